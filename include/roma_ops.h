/* SPDX-License-Identifier: Unlicense */

/* RoMa's own kernels as C functions. The reference creates them from
 * roma_kernels.cl with ocl_kernel and sets their arguments itself
 * (roma.c:440-448, 848-855, 911-918, 938-994, 1048-1103); here each is a
 * function with the kernel's argument list, preceded by the ops context
 * (its stream) and with the counts the reference passes as launch sizes
 * made explicit. Buffers are float32 in the reference's channel-major
 * layouts; the model itself (roma.cu) runs the same kernels on its
 * token-major maps.
 *
 *   roma_row_norm     replaces roma_kernels.cl:10  (rows of X)
 *   roma_cos_exp      replaces roma_kernels.cl:27
 *   roma_cls_to_flow  replaces roma_kernels.cl:46  (n tokens)
 *   roma_warp_sample  replaces roma_kernels.cl:130
 *   roma_local_corr   replaces roma_kernels.cl:153
 *   roma_disp         replaces roma_kernels.cl:196
 *   roma_update       replaces roma_kernels.cl:213
 *   roma2_update      replaces roma_kernels.cl:232
 *   roma_dwconv5      replaces roma_kernels.cl:256 (C channels)
 *   roma_gp_solve     replaces roma.c:772-836 (the host solve, on the device) */

#ifndef I_COREGISTRATION_B200_ROMA_OPS_H
#define I_COREGISTRATION_B200_ROMA_OPS_H

#include "ops.h"

#ifdef __cplusplus
extern "C" {
#endif

void roma_row_norm(struct ops *o, cl_mem X, int rows, int C, cl_mem out);
void roma_cos_exp(struct ops *o, cl_mem S, cl_mem nx, cl_mem ny, int N, int M,
                  float T, float eps);
void roma_cls_to_flow(struct ops *o, cl_mem L, int ld, int C, int res, int n,
                      cl_mem flow, cl_mem cert);
void roma_warp_sample(struct ops *o, cl_mem in, int C, int H, int W,
                      cl_mem flow, cl_mem out, int coff);
void roma_local_corr(struct ops *o, cl_mem f1, cl_mem f2, int C, int H, int W,
                     int r, cl_mem flow, cl_mem out, int coff);
void roma_disp(struct ops *o, cl_mem flow, int H, int W, float fx, float fy,
               cl_mem out);
void roma_update(struct ops *o, cl_mem flow, cl_mem cert, cl_mem d, int n,
                 float scale, float Wf, float Hf);
void roma2_update(struct ops *o, cl_mem flow, cl_mem conf, cl_mem d, int n,
                  float W, float H);
void roma_dwconv5(struct ops *o, cl_mem in, int C, int H, int W, cl_mem wt,
                  cl_mem bias, cl_mem out);

/* The Gaussian process's solve, X = (K + noise I)^-1 F, for the n x n
 * kernel matrix K (symmetric, row-major) and the n x d right-hand sides F,
 * in double precision on the device (blocked Cholesky, then the two
 * triangular solves); X may not alias F. Synchronous. Returns 0, or 1
 * when K + noise I is not positive definite (the reference stops there
 * with "kernel not positive definite"; X is then meaningless). */
int roma_gp_solve(struct ops *o, cl_mem K, int n, cl_mem F, int d, double noise, cl_mem X);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_ROMA_OPS_H */
