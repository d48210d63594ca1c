/* SPDX-License-Identifier: Unlicense */

/* Generic tensor operations of the B200 build: the reference's ops.h
 * (ops.h:41-164 of i.coregistration.opencl) with the same entry points,
 * argument order and meaning, run as hand-written sm_100a CUDA kernels
 * on the stream of the ocl_backend. Tensors are float32, channel-major
 * (C, H, W) for image-like data and token-major (tokens, channels) for
 * sequences; offsets, leading dimensions and strides are in elements.
 *
 * Entry point                 replaces (reference file:line)
 *   ops_init / ops_free        ops.c:86 / ops.c:112
 *   ops_mat / ops_bmat         ops.c:125 / ops.c:132
 *   ops_gemm                   ops.c:139  (kernels gemm/gemm_big, ops.cl:53-284)
 *   ops_linear                 ops.c:190
 *   ops_conv1x1                ops.c:199
 *   ops_geom / ops_conv_out    ops.c:206 / ops.c:213
 *   ops_conv2d                 ops.c:267  (conv5x5/conv2d/unfold, ops.cl:328-448, 799)
 *   ops_chan_stats             ops.c:338  (ops.cl:453)
 *   ops_chan_affine            ops.c:354  (ops.cl:499)
 *   ops_prelu / ops_act        ops.c:375 / ops.c:388 (ops.cl:522, 535)
 *   ops_layernorm              ops.c:412  (ops.cl:547)
 *   ops_softmax_rows           ops.c:431  (ops.cl:583)
 *   ops_attention              ops.c:444  (ops.cl:616)
 *   ops_rope                   ops.c:476  (ops.cl:695)
 *   ops_resize                 ops.c:496  (ops.cl:723)
 *   ops_grid_sample            ops.c:518  (ops.cl:759)
 *   ops_unfold                 ops.c:536  (ops.cl:799)
 *   ops_avgpool2 / ops_pool2d  ops.c:546 / ops.c:559 (ops.cl:819, 835)
 *   ops_transpose              ops.c:580  (ops.cl:864)
 *   ops_axpby                  ops.c:595  (ops.cl:884)
 *   ops_fold_bn                ops.c:612  (host)
 *   ops_report                 ops.c:60
 * ops_run (enqueue an OpenCL kernel object) has no counterpart here. */

#ifndef I_COREGISTRATION_B200_OPS_H
#define I_COREGISTRATION_B200_OPS_H

#include "ocl_backend.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Activations, applied after the bias. */
#define ACT_NONE 0
#define ACT_GELU 1 /* Exact (erf) GELU. */
#define ACT_RELU 2
#define ACT_LEAKY 3
#define ACT_GELU_TANH 4

/* Largest attention head dimension of ops_attention. */
#define OPS_MAX_HEAD_DIM 128

/* Arithmetic of the matrix products (ops_gemm and everything built on
 * it): OPS_FP32 (default) is float32 FMA as the reference; OPS_BF16
 * rounds both operands to bfloat16 and runs tcgen05 tensor-core tiles
 * with float32 accumulation. */
#define OPS_FP32 0
#define OPS_BF16 1

struct ops {
    struct ocl_backend *ocl;
    int precision;
    /* Work buffer of the im2col convolutions, grown on demand up to
     * im2col_bytes (256 MiB by default) per block of output positions. */
    cl_mem scratch;
    size_t scratch_bytes, im2col_bytes;
    /* Work buffer of the bfloat16 operand copies (OPS_BF16). */
    cl_mem scratch16;
    size_t scratch16_bytes;
};

/* One GEMM operand: buffer, element offset, leading dimension and the
 * two batch strides. */
struct opnd {
    cl_mem buf;
    cl_long off;
    cl_int ld;
    cl_long s0, s1;
};

struct opnd ops_mat(cl_mem buf, long off, int ld);
struct opnd ops_bmat(cl_mem buf, long off, int ld, long s0, long s1);

void ops_init(struct ops *o, struct ocl_backend *ocl);
void ops_free(struct ops *o);

/* With I_COREGISTRATION_OPENCL_PROFILE set at ocl_init, every launch is
 * timed with CUDA events under its operation name; this prints the
 * totals (name, ms, calls) on stderr. */
void ops_report(void);

/* Batched C = act(alpha * A * op(B) + bias) + R over nb = nb0 * nb1
 * products, product b at batch offsets (b / nb1) * s0 + (b % nb1) * s1 of
 * every operand; A is M x K row-major, B is N x K (transb) or K x N;
 * bias per column, or per row with biasrow; R (NULL for none) has C's
 * layout from element offset roff and may alias C. */
void ops_gemm(struct ops *o, int M, int N, int K, struct opnd A, struct opnd B,
              int transb, struct opnd C, int nb, int nb1, cl_mem bias,
              int biasrow, cl_mem R, long roff, float alpha, int act,
              float slope);

/* Token-major Y[rows, out] = act(X[rows, in] W^T + b) (+ Y when
 * residual), W the PyTorch [out, in] weight. */
void ops_linear(struct ops *o, int rows, int in, int out, cl_mem X, long xoff,
                cl_mem W, cl_mem b, cl_mem Y, long yoff, int act, float slope,
                int residual);

/* 1x1 convolution of a channel-major (C, HW) tensor into (K, HW). */
void ops_conv1x1(struct ops *o, cl_mem X, long xoff, int C, int HW, cl_mem W,
                 cl_mem b, int K, cl_mem Y, long yoff, int act, float slope);

struct conv_geom {
    int kh, kw, sy, sx, py, px, dy, dx, groups;
};

struct conv_geom ops_geom(int k, int s, int p);
int ops_conv_out(int n, int k, int s, int p, int d);

/* General convolution of in (C, H, W) into out (K, Ho, Wo); weights
 * (K, C / groups, kh, kw). mean/rstd/alpha (NULL for none) normalize and
 * gate the input, prelu((x - mean[c]) * rstd[c], alpha[c]), before the
 * zero padding. */
void ops_conv2d(struct ops *o, cl_mem in, int C, int H, int W, cl_mem w,
                cl_mem b, int K, const struct conv_geom *g, cl_mem mean,
                cl_mem rstd, cl_mem alpha, int act, float slope, cl_mem out);

void ops_chan_stats(struct ops *o, cl_mem x, int C, int HW, float eps,
                    cl_mem mean, cl_mem rstd);
void ops_chan_affine(struct ops *o, cl_mem X, cl_mem Y, int C, int HW,
                     cl_mem mean, cl_mem rstd, cl_mem g, cl_mem b, int act,
                     float slope);
void ops_prelu(struct ops *o, cl_mem X, cl_mem Y, int C, int HW, cl_mem alpha);
void ops_act(struct ops *o, cl_mem X, cl_mem Y, long n, int act, float slope);
void ops_layernorm(struct ops *o, long rows, int C, cl_mem X, cl_mem Y,
                   cl_mem g, cl_mem b, float eps, int act, float slope);
void ops_softmax_rows(struct ops *o, cl_mem S, long rows, int L, float scale);
void ops_attention(struct ops *o, struct opnd Q, struct opnd K, struct opnd V,
                   struct opnd O, int Nq, int Nk, int nh, int d, float scale,
                   cl_mem kmask);
void ops_rope(struct ops *o, cl_mem X, long off, int ld, long rows, int nh,
              int d, int npos, cl_mem cs, int interleaved);
void ops_resize(struct ops *o, cl_mem in, int C, int h, int w, cl_mem out,
                int H, int W, int coff, int align_corners, float scale);
void ops_grid_sample(struct ops *o, cl_mem in, int C, int H, int W, cl_mem grid,
                     int n, int align_corners, cl_mem out);
void ops_unfold(struct ops *o, cl_mem in, int C, int H, int W,
                const struct conv_geom *g, cl_mem out);
void ops_avgpool2(struct ops *o, cl_mem in, int C, int H, int W, cl_mem out);
void ops_pool2d(struct ops *o, cl_mem in, int C, int H, int W, int k, int s,
                int p, int max, cl_mem out);
void ops_transpose(struct ops *o, cl_mem in, cl_mem out, int B, int R, int C);
void ops_axpby(struct ops *o, cl_mem out, cl_mem a, float alpha, cl_mem b,
               float beta, long n, long bmod);
void ops_fold_bn(float *w, float *b, int K, long per, const float *gamma,
                 const float *beta, const float *mean, const float *var,
                 float eps);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_OPS_H */
