// SPDX-License-Identifier: Unlicense
//
// Launchers of RoMa's own kernels (roma_kernels.cu), used by the model
// (roma.cu) and by the C functions of roma_ops.h.
//
// Feature maps are addressed through two strides: element (c, i) of a map
// of n = H W cells is at base[c * cs + i * ps]. The reference's
// channel-major (C, n) layout is cs = n, ps = 1; this build's token-major
// (n, C) layout is cs = 1, ps = C. Warps, certainties and refiner outputs
// are planar: (k, n) with plane k at k * n.

#pragma once

#include "gemm.cuh"

namespace coreg {

struct Map {
    const void *p;
    long cs, ps;
    DType t;
};

struct MapOut {
    void *p;
    long cs, ps;
    DType t;
};

inline Map cm_map(const void *p, long n, DType t = DT_F32)
{
    return {p, n, 1, t};
}
inline Map tm_map(const void *p, long C, DType t = DT_F32)
{
    return {p, 1, C, t};
}
inline MapOut cm_out(void *p, long n, DType t = DT_F32)
{
    return {p, n, 1, t};
}
inline MapOut tm_out(void *p, long C, DType t = DT_F32)
{
    return {p, 1, C, t};
}

void roma_row_norm_l(cudaStream_t st, const float *X, int rows, int C,
                     float *out);
void roma_cos_exp_l(cudaStream_t st, float *S, const float *nx,
                    const float *ny, int N, int M, float T, float eps);
void roma_cls_to_flow_l(cudaStream_t st, const float *L, int ld, int C,
                        int res, int n, float *flow, float *cert);
// out channels coff .. coff + C - 1 = in (C channels, H x W grid) sampled
// at the warp flow (2, n).
void roma_warp_sample_l(cudaStream_t st, Map in, int C, int H, int W,
                        const float *flow, MapOut out, int coff);
void roma_local_corr_l(cudaStream_t st, Map f1, Map f2, int C, int H, int W,
                       int r, const float *flow, MapOut out, int coff);
// (fx, fy) (warp - own cell centre) into out (2, n) (planar) or, with
// emb_w set, the displacement embedding emb = W (emb, 2) disp + b into
// channels coff .. of out.
void roma_disp_l(cudaStream_t st, const float *flow, int H, int W, float fx,
                 float fy, float *out);
void roma_disp_emb_l(cudaStream_t st, const float *flow, int H, int W, float fx,
                     float fy, const float *emb_w, const float *emb_b, int emb,
                     MapOut out, int coff);
void roma_update_l(cudaStream_t st, float *flow, float *cert, Map d, int n,
                   float scale, float Wf, float Hf);
void roma2_update_l(cudaStream_t st, float *flow, float *conf, Map d, int n,
                    float W, float H);
// Depthwise 5 x 5, stride 1, padding 2, + bias, ReLU.
void roma_dwconv5_l(cudaStream_t st, Map in, int C, int H, int W,
                    const float *w, const float *b, MapOut out);

// Token-major helpers of the model.
// 2 x 2 / stride 2 max pooling of a channels-last (H, W, C) map.
void maxpool2_tm(cudaStream_t st, const void *in, DType t, int H, int W, int C,
                 void *out);
// Copy of rows x cols elements between row-major matrices (pitches in
// elements), with type conversion.
void copy2d(cudaStream_t st, const void *src, DType ts, long spitch, void *dst,
            DType td, long dpitch, long rows, long cols);
// Separable Pillow resampling of one (3, H, W) float image (weights
// precomputed per output index) into a channels-last (h, w, 3) map,
// normalized with (v - mean[c]) / std[c] when norm is set.
struct PilAxis {
    int n_out, taps;
    const int *start;     // n_out
    const double *weight; // n_out x taps
};
void pil_resize_norm(cudaStream_t st, const float *in, int H, int W, float *tmp,
                     PilAxis ax, PilAxis ay, int norm, void *out, DType t);
// The final host-side steps of roma_match on the device: certainty
// sigmoid (v2: of the overlap logit; v1: after the coarse attenuation),
// zero outside image B, warp clamped; v2 also sd = det(P)^(-1/4).
void roma_finish_l(cudaStream_t st, float *flow, float *cert, const float *prec,
                   const float *low, float *sd, long n);

}  // namespace coreg
