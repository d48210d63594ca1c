/* SPDX-License-Identifier: Unlicense */

/* A tile queue for the RoMa device stage over several GPUs (no reference
 * counterpart: it stands in for the per-tile loop of the reference's
 * main.c:776-896, which runs one roma_match after another on one OpenCL
 * device, for callers with several GPUs or several pipelines per GPU).
 *
 * Each pipeline is a backend (CUDA stream), an ops context, a roma_model
 * (roma_load, roma_load_v2 when v2 weights are given, roma_alloc) and a
 * host thread on one device. Tiles are independent (each roma_match is
 * self-contained), so a tile goes to whichever pipeline is free, and no
 * data moves between GPUs. Results come back to the caller in tile-index
 * order, the raster order that the reference's matcher.match and
 * dense_add need (dense.h:14-19, main.c:792-793).
 *
 * Errors: as the other entry points (ocl_backend.h). In the recorded mode
 * the first error of any pipeline is recorded on the calling thread once
 * the call has stopped its pipelines. */

#ifndef I_COREGISTRATION_B200_ROMA_TILES_H
#define I_COREGISTRATION_B200_ROMA_TILES_H

#ifdef __cplusplus
extern "C" {
#endif

struct roma_tiles;

/* Fill imgA and imgB (host, (3, H, W) floats in 0..1 each, pinned) with
 * tile `index`. Called from the pipelines' threads, several at a time. */
typedef void (*roma_tile_get)(void *ctx, int index, float *imgA, float *imgB);

/* Take the results of tile `index`: flow (2, H, W), cert (H, W) and sd
 * (H, W; NULL without RoMa v2's refiners), valid during the call. Called
 * once per tile, in increasing index order, one call at a time. */
typedef void (*roma_tile_put)(void *ctx, int index, const float *flow, const float *cert,
                              const float *sd);

/* per_device pipelines on each of the ndev CUDA devices in devices, the
 * RoMa weights main_w and dino_w (and RoMa v2's refiners v2_w, or NULL)
 * read by pth_open, precision OPS_FP32 or OPS_BF16, tiles of H x W cells
 * with the coarse pass at `coarse` (ROMA_COARSE for the reference's),
 * ImageNet normalization when imagenet is set. NULL after an error. */
struct roma_tiles *roma_tiles_create(const int *devices, int ndev, int per_device,
                                     int precision, const char *main_w, const char *dino_w,
                                     const char *v2_w, int H, int W, int coarse, int imagenet);

/* roma_match of tiles 0 .. ntiles - 1 over the pipelines: get fills a
 * free pipeline's pinned inputs, put receives the results in index order.
 * Returns the number of tiles delivered (ntiles unless an error stopped
 * the run). */
int roma_tiles_run(struct roma_tiles *t, int ntiles, roma_tile_get get, roma_tile_put put,
                   void *ctx);

/* Number of pipelines. */
int roma_tiles_pipelines(const struct roma_tiles *t);

void roma_tiles_free(struct roma_tiles *t);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_ROMA_TILES_H */
