// SPDX-License-Identifier: Unlicense
//
// Internal GEMM interface shared by ops_gemm (ops.h) and the models.
//
// C = act(alpha * A * op(B) + bias) + R, batched, with the contract of
// the reference's gemm / gemm_big kernels (ops.cl:39-52): A is M x K
// row-major (lda); B is N x K (transb, the PyTorch Linear weight layout)
// or K x N; batch b at offsets (b / nb1) * s0 + (b % nb1) * s1; bias per
// column (biasrow 0) or per row (biasrow 1); R has C's layout (ldc,
// batch strides of C) from its own base pointer and may alias C.
//
// Element types: A and B are float or bfloat16 (both the same), C and R
// float or bfloat16.

#pragma once

#include "common.cuh"

namespace coreg {

enum DType { DT_F32 = 0, DT_BF16 = 1 };

struct GemmArgs {
    int M, N, K;
    const void *A;
    long lda, sa0, sa1;
    const void *B;
    long ldb, sb0, sb1;
    int transb;
    void *C;
    long ldc, sc0, sc1;
    int nb, nb1;
    const float *bias;
    int biasrow;
    const void *R; // C's layout and type
    float alpha;
    int act;
    float slope;
    DType ab;  // type of A and B
    DType c;   // type of C and R
    // A operand mode: 0 dense row-major; 1 implicit im2col of a 3x3 /
    // stride 1 / padding 1 convolution over a channels-last (cH, cW, cC)
    // image (row m = pixel, column k = (ky, kx, c)); 2 implicit im2col of
    // a patchify convolution (cP x cP, stride cP) over a channels-last
    // (cH, cW, cC) image (row m = patch, column k = (c, ky, kx)).
    // amode 1: cK is the kernel size, 3 (also when 0: padding 1) or 5
    // (padding 2, column k = (ky, kx, c) likewise).
    int amode;
    int cH, cW, cC, cP, cK;
};

inline GemmArgs gemm_args(int M, int N, int K)
{
    GemmArgs g = {};
    g.M = M;
    g.N = N;
    g.K = K;
    g.nb = 1;
    g.nb1 = 1;
    g.alpha = 1.0f;
    return g;
}

// The rule by which ops_gemm (and ops_gemm_noalloc, which must give the
// same results) rounds float32 operands to bfloat16 for the tensor-core
// tiles: an OPS_BF16 context and a shape the tiles take. B is packed
// K-major whichever its layout (transb or not).
inline bool gemm_packs_bf16(int precision, int M, int N, int K)
{
    return precision == OPS_BF16 && M >= 64 && N >= 1 && K >= 16 && K % 8 == 0;
}

// Float32 rows x cols of each of nb batch products (batch b at
// (b / nb1) s0 + (b % nb1) s1, rows ld apart) into packed bfloat16 rows of
// `cols`, batch after batch; rows are walked by a grid-stride loop, so any
// row count launches.
void pack_bf16_rows(cudaStream_t st, const float *src, long ld, long s0, long s1, int nb,
                    int nb1, int rows, int cols, __nv_bfloat16 *dst);

// The transpose of the same: float32 rows x cols of each batch product into
// packed bfloat16 rows of `rows` (cols x rows per product), so that a
// K x N operand becomes N x K.
void pack_bf16_cols(cudaStream_t st, const float *src, long ld, long s0, long s1, int nb,
                    int nb1, int rows, int cols, __nv_bfloat16 *dst);

// Float32 FMA tiles (the accurate path): any strides, any type mix.
void gemm_simt(cudaStream_t st, const GemmArgs &g);

// tcgen05 tensor-core tiles for bfloat16 A and B, both K-major
// (transb), with float32 accumulation; returns false (nothing launched)
// when the shape or alignment is not supported, so that the caller can
// use gemm_simt.
bool gemm_tc(cudaStream_t st, const GemmArgs &g, int sm_count);

// Dispatch: tensor cores when bf16 operands allow it, else SIMT.
void gemm_run(const struct ocl_backend *ocl, const GemmArgs &g,
              const char *what);

// Internal launchers of ops.cu shared with the models.
void layernorm_rows(cudaStream_t st, const float *X, void *Y, DType ty,
                    const float *g, const float *b, long rows, int C, float eps,
                    int act, float slope);
void attention_l(cudaStream_t st, const void *Q, long ldq, const void *K,
                 long ldk, const void *V, long ldv, void *O, long ldo, int Nq,
                 int Nk, int nh, int d, float scale, const unsigned char *kmask,
                 DType t);
void resize_planes(cudaStream_t st, const float *in, int C, int h, int w,
                   float *out, int H, int W, int coff, int align, float scale);
void transpose_f32(cudaStream_t st, const float *in, float *out, int B, int R,
                   int C);
// Fused attention of a token-major qkv buffer (nimg images of N x 3 Dm,
// bfloat16, one after the other) into out (per image N rows of ldo,
// bfloat16) on tcgen05 tensor cores (tc_attention.cu); false when the head
// size (64 or 128) or alignment is not supported.
bool attention_tc(cudaStream_t st, const void *qkv, int N, int Dm, int heads, void *out,
                  long ldo, float scale, int nimg = 1);
// 3 x 3 / stride 1 / padding 1 convolution of a channels-last bfloat16
// (H, W, C) map with few channels (9 C <= kp, kp a multiple of 16) on the
// tensor cores: an explicit im2col into col (H W x kp bfloat16), then the
// GEMM with wk, the weights as (K, kp) bfloat16 rows in (tap, channel)
// order and zero beyond 9 C; out (H W x K) of type ot, bias and activation
// applied (ops.cu).
void conv3x3_im2col_tc(cudaStream_t st, const __nv_bfloat16 *in, int H, int W, int C, int kp,
                       const __nv_bfloat16 *wk, const float *bias, int K, int act,
                       float slope, void *out, DType ot, __nv_bfloat16 *col, int sm_count);

// The 3 -> 64 channel 3 x 3 convolution with bias and ReLU over a
// three-channel map, on the tensor cores without an im2col buffer
// (tc_conv_rgb.cu): wk is 64 x 32 (column j = tap 3 + c); false where it
// does not apply.
bool conv_rgb_tc(cudaStream_t st, const __nv_bfloat16 *in, int H, int W,
                 const __nv_bfloat16 *wk, const float *bias, void *out, DType ot, int sm_count);
// One hidden block of RoMa's refiners, out = W relu(dw5x5(in) + b_dw) + b_pw,
// over a channels-last bfloat16 (H, W, C) map in one tensor-core kernel
// (tc_dwpw.cu): dw_w (C x 25) and dw_b float32, pw_w (C x C, output-major)
// bfloat16, pw_b float32; false (nothing launched) unless C is 32, 64 or
// 128 and the pointers are 16-byte aligned.
bool dwpw_tc(cudaStream_t st, const void *in, int H, int W, int C, const float *dw_w,
             const float *dw_b, const void *pw_w, const float *pw_b, void *out, int sm_count);
// The depthwise 5 x 5 convolution + bias + ReLU of a refiner block alone
// (tc_dwpw.cu), channels-last bfloat16 in and out, C a multiple of 64;
// false (nothing launched) otherwise.
bool dw5_tc(cudaStream_t st, const void *in, int H, int W, int C, const float *dw_w,
            const float *dw_b, void *out, int sm_count);
// Double-precision GP solve (gp_chol.cu); work holds gp_work_doubles(n, d).
size_t gp_work_doubles(int n, int d);
void gp_solve_dev(cudaStream_t st, const float *K, int n, const float *F, int d,
                  double noise, float *X, double *work, int *flag);

}  // namespace coreg
