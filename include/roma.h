/* SPDX-License-Identifier: Unlicense */

/* RoMa on a B200: the reference's roma.h API (roma.h:110-128 of
 * i.coregistration.opencl) with the same entry points, argument meaning
 * and results, computed by this build's CUDA kernels.
 *
 *   roma_load     replaces roma.c:398   (VGG19-BN, DINOv2, projections, GP,
 *                                        decoder, refiners; BN / LayerScale
 *                                        folding on the host)
 *   roma_load_v2  replaces roma.c:533   (RoMa v2 refiners and their VGG)
 *   roma_alloc    replaces roma.c:559
 *   roma_match    replaces roma.c:1357  (host images in, host results out)
 *   roma_free     replaces roma.c:1464
 *
 * Differences of design, not of results: every step of a tile runs on
 * the device (the reference's host steps, the Pillow resampling
 * roma.c:1106-1186, the Gaussian-process Cholesky roma.c:772-836 and the
 * final sigmoid / clamp / standard deviation roma.c:1333-1349 and
 * 1419-1429, are CUDA kernels here); feature maps are token-major
 * (cells x channels) on the device; with ops->precision OPS_BF16 at
 * roma_load, the matrix products run on tcgen05 tensor cores with
 * bfloat16 operands and activations. */

#ifndef I_COREGISTRATION_B200_ROMA_H
#define I_COREGISTRATION_B200_ROMA_H

#include "ops.h"
#include "pth_loader.h"

#ifdef __cplusplus
extern "C" {
#endif

#define ROMA_MULTIPLE 8   /* Tile sides: VGG features down to 1/8. */
#define ROMA_COARSE 560   /* Side of the coarse pass (training size). */
#define ROMA_PATCH 14     /* DINOv2 patch size. */
#define ROMA_VIT_DIM 1024 /* DINOv2 ViT-L/14 width. */
#define ROMA_VIT_DEPTH 24 /* DINOv2 blocks. */
#define ROMA_DEC_DIM 1024 /* Coordinate decoder width (GP 512 + 512). */
#define ROMA_DEC_DEPTH 5  /* Coordinate decoder blocks. */
#define ROMA_CLS_RES 64   /* Coarse warp classes: 64 x 64 anchors. */
#define ROMA_SCALES 5     /* Refiners at 1/16, 1/8, 1/4, 1/2, 1/1. */
#define ROMA_HIDDEN 8     /* Hidden blocks per refiner. */
#define ROMA2_SCALES 3    /* RoMa v2's refiners at 1/4, 1/2, 1/1. */
#define ROMA2_ANCHOR 512  /* Their displacement scale: side / 512. */

struct roma_impl;

struct roma_model {
    struct ops *ops;
    struct ocl_backend *ocl;
    /* Inputs normalized with the ImageNet mean and deviation (RoMa's
     * transforms); MatchAnything's weights were trained on 0..1. */
    int imagenet;
    /* With RoMa v2's refiners (roma_load_v2). */
    int v2;
    /* OPS_FP32 or OPS_BF16, taken from ops->precision at roma_load. */
    int precision;
    /* Side of the coarse pass: ROMA_COARSE unless changed by
     * roma_set_coarse before roma_alloc. */
    int coarse;
    /* Tile size of roma_alloc. */
    int H, W;
    /* Last run, host side: flow (2, H, W) normalized to -1..1 in image B,
     * certainty (H, W) in 0..1, and with v2 the predicted standard
     * deviation (H, W) in cells (NAN where not positive definite). */
    float *flow, *cert, *sd;
    struct roma_impl *impl;
};

void roma_load(struct roma_model *m, struct ops *ops, struct pth_file *pf,
               struct pth_file *dino);
void roma_load_v2(struct roma_model *m, struct pth_file *pf);
void roma_alloc(struct roma_model *m, int H, int W);

/* Dense warp of image A onto image B, both (3, H, W) floats in 0..1 at
 * the alloc size (host memory): results in m->flow, m->cert, m->sd. With
 * dump set (a folder), the inputs and intermediate tensors are written
 * there as tileNNN_roma_<what>.f32 in the reference's layouts and names
 * (roma.c:1188-1227). Without dump and with profiling off, the tile runs
 * as one CUDA graph of the model, captured on the first such call (and
 * again when m->imagenet changes), so that call must not come inside a
 * stream capture of the calling thread. */
void roma_match(struct roma_model *m, const float *imgA, const float *imgB,
                const char *dump, int tile);

void roma_free(struct roma_model *m);

/* CUDA-native additions (no reference counterpart). */

/* Coarse-pass side (a multiple of 56: 14 for the patches, 8 for the
 * refiner grids), before roma_alloc; ROMA_COARSE by default. */
void roma_set_coarse(struct roma_model *m, int side);

/* roma_match on device-resident images (device pointers to (3, H, W)
 * floats), asynchronous on the model's stream, results left on the device
 * (roma_results_dev); no host transfer, no synchronisation. */
void roma_match_dev(struct roma_model *m, const float *imgA,
                    const float *imgB);

/* Device pointers of the last results: flow (2, H, W), cert (H, W), sd
 * (H, W, v2 only, else NULL). */
void roma_results_dev(struct roma_model *m, float **flow, float **cert,
                      float **sd);

/* Waits for the model's stream and reports a Gaussian-process kernel that
 * was not positive definite (the reference's fatal error, roma.c:785-787)
 * during the tiles run since the last call; 0 when all is well. */
int roma_sync(struct roma_model *m);

/* Capture one tile (roma_match_dev on these device images) into a CUDA
 * graph held by the model, replacing any previous one; returns the number
 * of kernel launches it holds, or -1 on error. roma_graph_launch replays
 * it on the model's stream (asynchronous; the images are read at replay
 * time, so new tiles are written into the same device buffers). */
int roma_graph_build(struct roma_model *m, const float *imgA,
                     const float *imgB);
void roma_graph_launch(struct roma_model *m);

/* Pinned host memory (for asynchronous host <-> device copies). */
void *coreg_host_alloc(size_t bytes);
void coreg_host_free(void *p);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_ROMA_H */
