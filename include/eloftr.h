/* SPDX-License-Identifier: Unlicense */

/* Efficient LoFTR on a B200: the reference's eloftr.h API (eloftr.h:66-82
 * of i.coregistration.opencl) with the same entry points, semantics and
 * the public result fields its matcher glue reads (matcher_eloftr.c).
 *
 *   eloftr_load   replaces eloftr.c:228  (RepVGG blocks and BatchNorms
 *                                         folded into 3 x 3 convolutions,
 *                                         transformer, fine fusion)
 *   eloftr_alloc  replaces eloftr.c:293  (tiles of H x W, multiples of 32)
 *   eloftr_match  replaces eloftr.c:681  (backbone, 4 x self / cross
 *                                         aggregated attention with 2-D
 *                                         RoPE, coarse dual softmax by
 *                                         blocks of rows, mutual matches,
 *                                         fusion, two-stage fine matching)
 *   eloftr_free   replaces eloftr.c:707
 *
 * The network runs on this build's ops.h kernels (float32 channel-major,
 * as the reference); the coarse-matching and fine-matching kernels are
 * CUDA kernels with the semantics of eloftr_kernels.cl. */

#ifndef I_COREGISTRATION_B200_ELOFTR_H
#define I_COREGISTRATION_B200_ELOFTR_H

#include "ops.h"
#include "pth_loader.h"

#ifdef __cplusplus
extern "C" {
#endif

#define ELOFTR_MULTIPLE 32   /* Tile sides: 1/8 features, aggregated by 4. */
#define ELOFTR_DIM 256       /* Coarse feature dimension. */
#define ELOFTR_FINE_DIM 64   /* Fine feature dimension. */
#define ELOFTR_BLOCKS 21     /* RepVGG blocks: 1 + 2 + 4 + 14. */
#define ELOFTR_LAYERS 4      /* Transformer layers (self + cross each). */
#define ELOFTR_TRAIN_RES 832 /* Training resolution of the "npe". */

struct eloftr_impl;

struct eloftr_model {
    struct ops *ops;
    struct ocl_backend *ocl;
    /* Scale of the RoPE positions, set before eloftr_alloc: 1 as
     * Transformers; the authors' "npe" is 832 / the long side. */
    float pos_scale;
    /* Tile size, 1/8 grid, aggregated (1/32) grid, match capacity. */
    int H, W, h, w, ah, aw, nmax;
    /* Last eloftr_match: nm coarse matches, cells mi (image 0) and mj
     * (image 1) of the 1/8 grid, confidence mconf, and kp = x0, y0, x1, y1
     * per match in pixels (the reference's convention: pixel index - 3.5).
     * Host arrays owned by the model. */
    int nm;
    int *mi, *mj;
    float *mconf, *kp;
    struct eloftr_impl *impl;
};

/* Read the weights (EfficientLoFTRForKeypointMatching's names:
 * "efficientloftr.backbone.*", "efficientloftr.local_feature_transformer.*",
 * "refinement_layer.*"), fold the BatchNorms and upload. */
void eloftr_load(struct eloftr_model *m, struct ops *ops, struct pth_file *pf);

/* Work buffers for tiles of H x W cells (multiples of ELOFTR_MULTIPLE). */
void eloftr_alloc(struct eloftr_model *m, int H, int W);

/* Match two grey images (host H x W floats in 0..1): coarse mutual
 * matches above confidence 0.2 away from a 2-cell border, refined to a
 * fraction of a cell. Results in m->nm, m->mi, m->mj, m->mconf, m->kp.
 * With dump set (a folder), writes tileNNN_eloftr_<what>.f32 for the 1/8
 * backbone features (backbone_0/1, 256 x H/8 x W/8), the transformer
 * output (coarse_0/1) and the fine features (fine_0/1, 64 x H x W). */
void eloftr_match(struct eloftr_model *m, const float *grey0, const float *grey1,
                  const char *dump, int tile);

void eloftr_free(struct eloftr_model *m);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_ELOFTR_H */
