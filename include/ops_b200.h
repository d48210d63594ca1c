/* SPDX-License-Identifier: Unlicense */

/* Operations of the B200 build without a counterpart in the reference's
 * ops.h: the channels-last ("token-major") 3 x 3 convolution the models
 * run (the reference's VGG convolutions, roma.c:742-768 and 1000-1027,
 * go through ops_conv2d on channel-major maps; this build keeps feature
 * maps channels-last so that every convolution is an implicit GEMM with
 * K-major operands), and the tensor-core status of the library. */

#ifndef I_COREGISTRATION_B200_OPS_B200_H
#define I_COREGISTRATION_B200_OPS_B200_H

#include "ops.h"

#ifdef __cplusplus
extern "C" {
#endif

/* 3 x 3 convolution, stride 1, zero padding 1, of a channels-last
 * (H, W, C) float32 map into (H, W, K): weights in the PyTorch layout
 * (K, C, 3, 3), bias per output channel (may be NULL), activation after
 * the bias. With o->precision OPS_BF16 and C a multiple of 64 it runs
 * as an implicit GEMM on tcgen05 tensor cores (the input and weights
 * rounded to bfloat16, 3-D TMA boxes of the map per tap, no im2col
 * buffer); otherwise in float32. */
void ops_conv3x3_cl(struct ops *o, cl_mem in, int H, int W, int C, cl_mem w,
                    cl_mem b, int K, int act, float slope, cl_mem out);

/* Multi-head attention of a fused token-major qkv buffer (N rows of 3 Dm
 * float32: queries, keys, values; head h at columns h (Dm / heads) of
 * each) into out (N x Dm): O = softmax(scale Q K^T) V per head, the
 * transformer attention of the models (the reference computes it with
 * two ops_gemm and ops_softmax_rows, roma.c:675-694). With o->precision
 * OPS_BF16 and a head size of 64 or 128 it runs the fused tcgen05 kernel
 * (bfloat16 operands, the probabilities rounded to bfloat16, float32
 * accumulation, no score matrix); otherwise the float32 kernel of
 * ops_attention. */
void ops_attention_qkv(struct ops *o, cl_mem qkv, int N, int Dm, int heads,
                       float scale, cl_mem out);

/* Depthwise 5 x 5 convolution, zero padding 2, + bias + ReLU of a
 * channels-last (H, W, C) float32 map into (H, W, C): the first half of a
 * RoMa refiner block with its BatchNorm folded (roma_dwconv5,
 * roma_kernels.cl:256-284, on channel-major maps). Weights (C, 1, 5, 5),
 * bias C floats. With o->precision OPS_BF16 the map is rounded to
 * bfloat16 and the model's bfloat16 kernel runs (float32 arithmetic,
 * bfloat16 result), as inside roma_match. */
void roma_dwconv5_cl(struct ops *o, cl_mem in, int H, int W, int C, cl_mem wt,
                     cl_mem bias, cl_mem out);

/* One hidden block of a RoMa refiner on a channels-last (H, W, C)
 * float32 map: out = W_pw relu(dw5x5(in) + b_dw) + b_pw, the depthwise
 * 5 x 5 convolution of roma_dwconv5_cl followed by the 1 x 1 convolution
 * the reference runs after it (roma.c:970-985, 1080-1094). pw_w is
 * (C, C) output-major, pw_b C floats. With o->precision OPS_BF16 and C
 * 32, 64 or 128 the model's fused tensor-core kernel runs (the depthwise
 * result rounded to bfloat16 in shared memory, float32 accumulation,
 * bfloat16 result); otherwise the two steps run one after the other. No
 * reference counterpart. */
void roma_refiner_block_cl(struct ops *o, cl_mem in, int H, int W, int C, cl_mem dw_w,
                           cl_mem dw_b, cl_mem pw_w, cl_mem pw_b, cl_mem out);

/* Local correlation of channels-last (H, W, C) float32 maps f1 and f2 at
 * the warp flow ((2, H, W) normalized coordinates, channel-major as in
 * the models) into out, channels-last (H, W, (2r + 1)^2): roma_local_corr
 * (roma_kernels.cl:153-192) on the models' layout. With o->precision
 * OPS_BF16 the maps are rounded to bfloat16 and the model's bfloat16
 * kernel runs (float32 arithmetic), as inside roma_match. */
void roma_local_corr_cl(struct ops *o, cl_mem f1, cl_mem f2, int C, int H, int W, int r,
                        cl_mem flow, cl_mem out);

/* ops_gemm that allocates no device memory; it has no counterpart in the
 * reference. Same arguments, meaning and results as ops_gemm. With
 * o->precision OPS_BF16, ops_gemm packs the operands to bfloat16 in a
 * buffer it grows with cudaMalloc; this variant packs them into a fixed
 * device array of ops_gemm_noalloc_max_bytes() bytes (16 MiB) that is part
 * of the library. It is meant for callers that must not allocate while
 * they run: a plug-in whose host framework's caching allocator already
 * holds the device's free memory, or a pipeline that does all allocation at
 * start-up because cudaMalloc synchronises the device. A product whose
 * packed operands, 2 (M + N) K nb bytes plus alignment, exceed the array is
 * rejected with an error naming the sizes (ops_gemm still runs it). The
 * first call on each device looks up the array's address and may load
 * the library's module there, so make it before any stream capture. All
 * calls on a device share the one array: calls that overlap in time
 * (several streams, host threads or ops contexts) corrupt each other's
 * results and must be serialised by the caller. Float32 products
 * (OPS_FP32, or shapes the tensor-core path does not take) stage nothing. */
void ops_gemm_noalloc(struct ops *o, int M, int N, int K, struct opnd A,
                      struct opnd B, int transb, struct opnd C, int nb, int nb1,
                      cl_mem bias, int biasrow, cl_mem R, long roff, float alpha,
                      int act, float slope);

/* Size in bytes of ops_gemm_noalloc's scratch array. */
size_t ops_gemm_noalloc_max_bytes(void);

/* Non-zero when a bounded wait of a tensor-core kernel ran out since the
 * last call (the kernel then stopped and its results are invalid); the
 * code is cleared. */
int coreg_tc_status(void);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_OPS_B200_H */
