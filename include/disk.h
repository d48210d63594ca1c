/* SPDX-License-Identifier: Unlicense */

/* DISK local features on a B200: the reference's disk.h API (disk.h:34-52
 * of i.coregistration.opencl) with the same entry points and semantics.
 *
 *   disk_load    replaces disk.c:42   (the "unet.path_down/up" weights)
 *   disk_alloc   replaces disk.c:84   (tiles of up to H x W cells)
 *   disk_detect  replaces disk.c:163  (U-Net, 5 x 5 NMS, the n best in
 *                                      raster order, L2-normalized
 *                                      descriptors)
 *   disk_free    replaces disk.c:285
 *
 * The U-Net runs on this build's ops.h kernels (float32, channel-major, as
 * the reference); the NMS and descriptor gather are CUDA kernels with the
 * semantics of disk_kernels.cl:10-60.
 *
 * Additions without a counterpart in the reference: disk_output_dev (the
 * network output on the device, for parity checks) and desc_nearest, the
 * descriptor-distance stage that the reference runs on the host inside
 * adalam_match (adalam.c:38-98), here on the device. */

#ifndef I_COREGISTRATION_B200_DISK_H
#define I_COREGISTRATION_B200_DISK_H

#include "ocl_backend.h"
#include "ops.h"
#include "pth_loader.h"

#ifdef __cplusplus
extern "C" {
#endif

#define DISK_DESC 128    /* Descriptor dimension. */
#define DISK_LAYERS 9    /* Five down blocks, four up blocks. */
#define DISK_MULTIPLE 16 /* Input sides must be multiples of this. */

struct disk_impl;

/* DISK (kornia.feature.DISK's U-Net: 5 x 5 kernels, down 16-32-64-64-64,
 * up 64-64-64-129). */
struct disk_model {
    struct ocl_backend *ocl;
    struct ops *ops;
    int cin[DISK_LAYERS], cout[DISK_LAYERS];
    /* Tile capacity of disk_alloc. */
    int H, W, nmax;
    struct disk_impl *impl;
};

/* Read the DISK weights from pf ("unet.path_down.{0..4}.1.{1,3}",
 * "unet.path_up.{0..3}.conv.{1,3}") and upload them. Errors as the ops.h
 * entry points (fatal, or recorded). */
void disk_load(struct disk_model *m, struct ops *ops, struct pth_file *pf);

/* Work buffers for tiles of up to H x W cells (multiples of
 * DISK_MULTIPLE) and up to nmax keypoints. */
void disk_alloc(struct disk_model *m, int H, int W, int nmax);

/* Keypoints of img, a host (3, H, W) float image in 0..1 whose content
 * covers its top-left h x w cells: 5 x 5 non-maxima suppression of the
 * heatmap cropped to h x w (the 2-cell border excluded), cells above
 * thresh, skipping cells where valid (h x w bytes, may be NULL) is 0; of
 * those the ones above the (n + 1)-th highest score, in raster order (at
 * most n). Writes xy (x, y pairs), score and the L2-normalized descriptors
 * (n x DISK_DESC) to host memory; returns the number of keypoints. */
int disk_detect(struct disk_model *m, const float *img, int H, int W, int h,
                int w, int n, float thresh, const unsigned char *valid, int *xy,
                float *score, float *desc);

void disk_free(struct disk_model *m);

/* Device pointer to the last disk_detect's network output ((DISK_DESC + 1,
 * H, W) float32: descriptors, then the heatmap). No reference
 * counterpart. */
const float *disk_output_dev(const struct disk_model *m);

/* Nearest neighbour of each of the n1 descriptors d1 among the n2 of d2
 * (dim floats each, host arrays) by the squared distance |a|^2 + |b|^2 -
 * 2 a.b, computed on the device: nn12 (n1 indices), score (the ratio of
 * the two smallest distances, the second clamped below at 1e-3) and, when
 * nn21 is not NULL, the nearest d1 of each d2 (n2 indices). Ties keep the
 * lowest index. The reference computes this on the host in adalam_match
 * (adalam.c:38-98); no counterpart in its headers. */
void desc_nearest(struct ops *o, const float *d1, int n1, const float *d2, int n2, int dim,
                  int *nn12, float *score, int *nn21);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_DISK_H */
