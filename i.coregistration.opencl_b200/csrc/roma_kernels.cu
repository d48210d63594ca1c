// SPDX-License-Identifier: Unlicense
//
// RoMa's own kernels on CUDA: Gaussian-process kernel, coarse warp from
// the anchor classes, warp sampling, local correlation, displacement
// embedding, warp updates (v1 and v2), depthwise 5 x 5 convolution, and
// the model's layout helpers (token-major pooling, Pillow resampling,
// the final certainty / standard-deviation step). Each kernel keeps the
// semantics of the reference's roma_kernels.cl kernel it replaces (cited
// per kernel); the index layouts are this build's (see roma_kernels.cuh).

#include <math.h>

#include "gemm.cuh"
#include "roma_kernels.cuh"

namespace coreg {

// Packed float32 pair FMA of sm_100 (a * b + c on both lanes).
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c)
{
    unsigned long long aa, bb, cc, dd;
    asm("mov.b64 %0, {%1, %2};" : "=l"(aa) : "f"(a.x), "f"(a.y));
    asm("mov.b64 %0, {%1, %2};" : "=l"(bb) : "f"(b.x), "f"(b.y));
    asm("mov.b64 %0, {%1, %2};" : "=l"(cc) : "f"(c.x), "f"(c.y));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(dd) : "l"(aa), "l"(bb), "l"(cc));
    float2 d;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(dd));
    return d;
}


template <typename T>
__device__ __forceinline__ float at_map(const T *p, long cs, long ps, int c,
                                        long i)
{
    return ldf(p + c * cs + i * ps);
}

// ------------------------------------------------------------- GP kernel

// roma_row_norm, roma_kernels.cl:10-23: Euclidean norm of each row.
__global__ void row_norm_k(const float *X, int rows, int C, float *out)
{
    const int r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r >= rows)
        return;
    const float *x = X + (size_t)r * C;
    float s = 0.0f;
    for (int c = lane; c < C; c += 32)
        s = fmaf(x[c], x[c], s);
    s = warp_sum(s);
    if (lane == 0)
        out[r] = sqrtf(s);
}

void roma_row_norm_l(cudaStream_t st, const float *X, int rows, int C,
                     float *out)
{
    if (rows > 0)
        row_norm_k<<<cdiv(rows, 8), 256, 0, st>>>(X, rows, C, out);
}

// roma_cos_exp, roma_kernels.cl:27-38: RoMa's CosKernel in place.
__global__ void cos_exp_k(float *S, const float *nx, const float *ny, int N,
                          int M, float T, float eps)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= (long)N * M)
        return;
    const int i = (int)(e / M), j = (int)(e % M);
    const float c = S[e] / (nx[i] * ny[j] + eps);
    S[e] = expf((c - 1.0f) / T);
}

void roma_cos_exp_l(cudaStream_t st, float *S, const float *nx,
                    const float *ny, int N, int M, float T, float eps)
{
    const long n = (long)N * M;
    if (n > 0)
        cos_exp_k<<<cdiv(n, 256), 256, 0, st>>>(S, nx, ny, N, M, T, eps);
}

// ------------------------------------------------------------ cls_to_flow

// roma_cls_to_flow, roma_kernels.cl:46-102: per token, softmax over the C
// = res x res anchor logits, their mode (first index among equal maxima),
// and the probability-weighted mean position of the mode and its four
// neighbours, indices clamped to 0 .. C - 1 (a clamped neighbour counts
// twice); the certainty logit (column C) copied. One block per token.
__global__ void __launch_bounds__(256)
cls_to_flow_k(const float *L, int ld, int C, int res, int n, float *flow,
              float *cert)
{
    __shared__ float vm[256], vs[256];
    __shared__ int vi[256];
    const int t = blockIdx.x, l = threadIdx.x;
    const float *p = L + (size_t)t * ld;
    float m = -INFINITY, s = 0.0f;
    int arg = 0;

    for (int j = l; j < C; j += 256)
        if (p[j] > m) {
            m = p[j];
            arg = j;
        }
    vm[l] = m;
    vi[l] = arg;
    __syncthreads();
    for (int k = 128; k > 0; k >>= 1) {
        if (l < k &&
            (vm[l + k] > vm[l] || (vm[l + k] == vm[l] && vi[l + k] < vi[l]))) {
            vm[l] = vm[l + k];
            vi[l] = vi[l + k];
        }
        __syncthreads();
    }
    m = vm[0];
    for (int j = l; j < C; j += 256)
        s += expf(p[j] - m);
    vs[l] = s;
    __syncthreads();
    for (int k = 128; k > 0; k >>= 1) {
        if (l < k)
            vs[l] += vs[l + k];
        __syncthreads();
    }
    if (l == 0) {
        const int mode = vi[0];
        const int nb[5] = {mode - 1, mode, mode + 1, mode - res, mode + res};
        float fx = 0.0f, fy = 0.0f, tot = 0.0f;
        for (int k = 0; k < 5; k++) {
            const int c = min(max(nb[k], 0), C - 1);
            const float pr = expf(p[c] - m) / vs[0];
            fx += pr * (-1.0f + (2 * (c % res) + 1) / (float)res);
            fy += pr * (-1.0f + (2 * (c / res) + 1) / (float)res);
            tot += pr;
        }
        flow[t] = fx / tot;
        flow[n + t] = fy / tot;
        cert[t] = p[C];
    }
}

void roma_cls_to_flow_l(cudaStream_t st, const float *L, int ld, int C,
                        int res, int n, float *flow, float *cert)
{
    if (n > 0)
        cls_to_flow_k<<<n, 256, 0, st>>>(L, ld, C, res, n, flow, cert);
}

// ------------------------------------------------------------ warp sample

// Bilinear value at normalized (x, y), align_corners=False, zero padding,
// non-finite points 0 (bilinear0, roma_kernels.cl:106-128).
template <typename T>
__device__ __forceinline__ float bilinear0(const T *p, long cs, long ps, int c,
                                           int H, int W, float x, float y)
{
    const float ix = ((x + 1.0f) * W - 1.0f) * 0.5f;
    const float iy = ((y + 1.0f) * H - 1.0f) * 0.5f;
    if (!isfinite(ix) || !isfinite(iy))
        return 0.0f;
    const int x0 = (int)floorf(ix), y0 = (int)floorf(iy);
    const float fx = ix - x0, fy = iy - y0;
    auto at = [&](int yy, int xx) {
        return xx >= 0 && xx < W && yy >= 0 && yy < H
                   ? at_map(p, cs, ps, c, (long)yy * W + xx)
                   : 0.0f;
    };
    const float v00 = at(y0, x0), v01 = at(y0, x0 + 1);
    const float v10 = at(y0 + 1, x0), v11 = at(y0 + 1, x0 + 1);
    return (1.0f - fy) * ((1.0f - fx) * v00 + fx * v01) +
           fy * ((1.0f - fx) * v10 + fx * v11);
}

// roma_warp_sample, roma_kernels.cl:130-141. Channel-fastest thread order
// for token-major maps (coalesced over channels), cell-fastest otherwise.
template <typename TI, typename TO>
__global__ void warp_sample_k(const TI *in, long cs, long ps, int C, int H,
                              int W, const float *flow, TO *out, long ocs,
                              long ops, int coff, int chan_fast)
{
    const long n = (long)H * W;
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n * C)
        return;
    int c;
    long i;
    if (chan_fast) {
        c = (int)(e % C);
        i = e / C;
    }
    else {
        i = e % n;
        c = (int)(e / n);
    }
    stf(out + (long)(coff + c) * ocs + i * ops,
        bilinear0(in, cs, ps, c, H, W, flow[i], flow[n + i]));
}

// The same for dense bfloat16 maps, 4 channels a thread (8-byte loads and
// store), the bilinear weights computed once per cell; the arithmetic per
// channel is bilinear0's.
__global__ void warp_sample4_k(const uint2 *in, long ps4, int C4, int H, int W, const float *flow,
                               uint2 *out, long ops4, int coff4, int total)
{
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= total)
        return;
    const int g = e % C4, i = e / C4, n = H * W;
    const float ix = ((flow[i] + 1.0f) * W - 1.0f) * 0.5f;
    const float iy = ((flow[n + i] + 1.0f) * H - 1.0f) * 0.5f;
    float v[4][4] = {};
    float fx = 0.0f, fy = 0.0f;
    if (isfinite(ix) && isfinite(iy)) {
        const int x0 = (int)floorf(ix), y0 = (int)floorf(iy);
        fx = ix - x0;
        fy = iy - y0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int yy = y0 + (k >> 1), xx = x0 + (k & 1);
            if (xx >= 0 && xx < W && yy >= 0 && yy < H) {
                const uint2 u = in[((long)yy * W + xx) * ps4 + g];
                v[k][0] = __uint_as_float(u.x << 16);
                v[k][1] = __uint_as_float(u.x & 0xffff0000u);
                v[k][2] = __uint_as_float(u.y << 16);
                v[k][3] = __uint_as_float(u.y & 0xffff0000u);
            }
        }
    }
    float r[4];
#pragma unroll
    for (int c = 0; c < 4; c++)
        r[c] = (1.0f - fy) * ((1.0f - fx) * v[0][c] + fx * v[1][c]) +
               fy * ((1.0f - fx) * v[2][c] + fx * v[3][c]);
    const __nv_bfloat162 a = __floats2bfloat162_rn(r[0], r[1]), b = __floats2bfloat162_rn(r[2], r[3]);
    uint2 o;
    o.x = *(const uint32_t *)&a;
    o.y = *(const uint32_t *)&b;
    out[(long)i * ops4 + coff4 + g] = o;
}

template <typename TI, typename TO>
static void warp_sample_t(cudaStream_t st, Map in, int C, int H, int W,
                          const float *flow, MapOut out, int coff)
{
    const long tot = (long)H * W * C;
    if (sizeof(TI) == 2 && sizeof(TO) == 2 && in.cs == 1 && out.cs == 1 && C % 4 == 0 &&
        in.ps % 4 == 0 && out.ps % 4 == 0 && coff % 4 == 0 && ((uintptr_t)in.p & 7) == 0 &&
        ((uintptr_t)out.p & 7) == 0 && tot / 4 < (1L << 30)) {
        const int total = (int)(tot / 4);
        warp_sample4_k<<<cdiv(total, 256), 256, 0, st>>>(
            (const uint2 *)in.p, in.ps / 4, C / 4, H, W, flow, (uint2 *)out.p, out.ps / 4,
            coff / 4, total);
        return;
    }
    warp_sample_k<TI, TO><<<cdiv(tot, 256), 256, 0, st>>>(
        (const TI *)in.p, in.cs, in.ps, C, H, W, flow, (TO *)out.p, out.cs,
        out.ps, coff, in.cs == 1);
}

void roma_warp_sample_l(cudaStream_t st, Map in, int C, int H, int W,
                        const float *flow, MapOut out, int coff)
{
    if ((long)H * W * C <= 0)
        return;
    if (in.t == DT_F32 && out.t == DT_F32)
        warp_sample_t<float, float>(st, in, C, H, W, flow, out, coff);
    else if (in.t == DT_BF16 && out.t == DT_BF16)
        warp_sample_t<__nv_bfloat16, __nv_bfloat16>(st, in, C, H, W, flow, out,
                                                    coff);
    else if (in.t == DT_F32)
        warp_sample_t<float, __nv_bfloat16>(st, in, C, H, W, flow, out, coff);
    else
        warp_sample_t<__nv_bfloat16, float>(st, in, C, H, W, flow, out, coff);
}

// ------------------------------------------------------ local correlation

// roma_local_corr, roma_kernels.cl:153-192: for window offset k = (a, b)
// of (2r + 1)^2 (a the row), f1 / sqrt(C) dotted with f2 sampled at the
// warp shifted by (b - r, a - r) cells. The offsets are whole cells, so
// the dot products are taken once at the (2r + 2)^2 cells around the warp
// and combined with the shared bilinear weights. One warp per cell: lanes
// split the channels.
#define CORR_MAXC 512
#define CORR_MAXPS 16
template <typename TI, typename TO>
__global__ void __launch_bounds__(128)
local_corr_k(const TI *f1, long cs1, long ps1, const TI *f2, long cs2,
             long ps2, int C, int H, int W, int r, const float *flow, TO *out,
             long ocs, long ops, int coff)
{
    __shared__ float S[4][CORR_MAXPS * CORR_MAXPS];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const long n = (long)H * W;
    const long i = (long)blockIdx.x * 4 + w;
    if (i >= n)
        return;
    const int side = 2 * r + 1, ps = 2 * r + 2;
    const float rc = rsqrtf((float)C);
    const float ix = ((flow[i] + 1.0f) * W - 1.0f) * 0.5f;
    const float iy = ((flow[n + i] + 1.0f) * H - 1.0f) * 0.5f;
    const bool ok = isfinite(ix) && isfinite(iy);
    const int x0 = ok ? (int)floorf(ix) : 0, y0 = ok ? (int)floorf(iy) : 0;
    const float fx = ok ? ix - x0 : 0.0f, fy = ok ? iy - y0 : 0.0f;
    float a1[CORR_MAXC / 32];

#pragma unroll
    for (int j = 0; j < CORR_MAXC / 32; j++) {
        const int c = lane + 32 * j;
        a1[j] = c < C ? at_map(f1, cs1, ps1, c, i) * rc : 0.0f;
    }
    for (int e = 0; e < ps * ps; e++) {
        const int yy = y0 - r + e / ps, xx = x0 - r + e % ps;
        float s = 0.0f;
        if (ok && xx >= 0 && xx < W && yy >= 0 && yy < H) {
            const long cell = (long)yy * W + xx;
#pragma unroll
            for (int j = 0; j < CORR_MAXC / 32; j++) {
                const int c = lane + 32 * j;
                if (c < C)
                    s = fmaf(a1[j], at_map(f2, cs2, ps2, c, cell), s);
            }
            s = warp_sum(s);
        }
        if (lane == 0)
            S[w][e] = s;
    }
    __syncwarp();
    for (int k = lane; k < side * side; k += 32) {
        const int e0 = (k / side) * ps + k % side, e1 = e0 + ps;
        const float v = (1.0f - fy) * ((1.0f - fx) * S[w][e0] + fx * S[w][e0 + 1]) +
                        fy * ((1.0f - fx) * S[w][e1] + fx * S[w][e1 + 1]);
        stf(out + (long)(coff + k) * ocs + i * ops, v);
    }
}

// The same for bfloat16 channels-last maps with C a multiple of 8 (the
// model's layout): one warp per cell, whose scaled f1 row sits in shared
// memory as float; the lanes split the (2r + 2)^2 positions (and, when
// there are fewer than 32, the channels into G groups), each taking a whole
// dot product with 16-byte loads of f2 and packed FMAs, then one shuffle
// reduction over its G lanes.
template <typename TO>
__global__ void __launch_bounds__(128)
local_corr_bf16_k(const __nv_bfloat16 *f1, long ps1, const __nv_bfloat16 *f2, long ps2, int C,
                  int H, int W, int r, const float *flow, TO *out, long ocs, long ops, int coff)
{
    __shared__ __align__(16) float a_s[4][CORR_MAXC];
    __shared__ float S[4][CORR_MAXPS * CORR_MAXPS];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const long n = (long)H * W;
    const long i = (long)blockIdx.x * 4 + w;
    if (i >= n)
        return;
    const int side = 2 * r + 1, ps = 2 * r + 2, P = ps * ps;
    const float rc = rsqrtf((float)C);
    const float ix = ((flow[i] + 1.0f) * W - 1.0f) * 0.5f;
    const float iy = ((flow[n + i] + 1.0f) * H - 1.0f) * 0.5f;
    const bool ok = isfinite(ix) && isfinite(iy);
    const int x0 = ok ? (int)floorf(ix) : 0, y0 = ok ? (int)floorf(iy) : 0;
    const float fx = ok ? ix - x0 : 0.0f, fy = ok ? iy - y0 : 0.0f;
    const __nv_bfloat16 *a = f1 + i * ps1;
    for (int c = lane; c < C; c += 32)
        a_s[w][c] = __bfloat162float(a[c]) * rc;
    __syncwarp();
    // G lanes per position (a power of two), positions per round 32 / G.
    const int G = P >= 32 ? 1 : (P > 8 ? 2 : (P > 4 ? 4 : 8));
    const int per = 32 / G, g = lane % G;
    const int nv = C / 8;
    for (int e0 = 0; e0 < P; e0 += per) {
        const int e = e0 + lane / G;
        const int yy = y0 - r + e / ps, xx = x0 - r + e % ps;
        float2 acc = make_float2(0.0f, 0.0f);
        if (e < P && ok && xx >= 0 && xx < W && yy >= 0 && yy < H) {
            const __nv_bfloat16 *b = f2 + ((long)yy * W + xx) * ps2;
            for (int v = g; v < nv; v += G) {
                const uint4 u = *(const uint4 *)(b + 8 * v);
                const float4 p0 = *(const float4 *)&a_s[w][8 * v];
                const float4 p1 = *(const float4 *)&a_s[w][8 * v + 4];
                acc = fma2(make_float2(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u)),
                           make_float2(p0.x, p0.y), acc);
                acc = fma2(make_float2(__uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u)),
                           make_float2(p0.z, p0.w), acc);
                acc = fma2(make_float2(__uint_as_float(u.z << 16), __uint_as_float(u.z & 0xffff0000u)),
                           make_float2(p1.x, p1.y), acc);
                acc = fma2(make_float2(__uint_as_float(u.w << 16), __uint_as_float(u.w & 0xffff0000u)),
                           make_float2(p1.z, p1.w), acc);
            }
        }
        float s = acc.x + acc.y;
        for (int o = G / 2; o > 0; o /= 2)
            s += __shfl_xor_sync(0xffffffffu, s, o);
        if (g == 0 && e < P)
            S[w][e] = s;
    }
    __syncwarp();
    for (int k = lane; k < side * side; k += 32) {
        const int e0 = (k / side) * ps + k % side, e1 = e0 + ps;
        const float v = (1.0f - fy) * ((1.0f - fx) * S[w][e0] + fx * S[w][e0 + 1]) +
                        fy * ((1.0f - fx) * S[w][e1] + fx * S[w][e1 + 1]);
        stf(out + (long)(coff + k) * ocs + i * ops, v);
    }
}

// The same with the channel count (NV 8-channel groups) and the lanes per
// position (G) fixed at compile time: the G lanes of a position read
// consecutive 16-byte pieces of its f2 row (coalesced), a few each,
// unrolled; bfloat16 (one 16-byte load a group) or float (two) maps, dense
// rows.
__device__ __forceinline__ void load8(const __nv_bfloat16 *b, float v[8])
{
    const uint4 u = *(const uint4 *)b;
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; k++) {
        v[2 * k] = __uint_as_float(w[k] << 16);
        v[2 * k + 1] = __uint_as_float(w[k] & 0xffff0000u);
    }
}

__device__ __forceinline__ void load8(const float *b, float v[8])
{
    const float4 x = *(const float4 *)b, y = *(const float4 *)(b + 4);
    v[0] = x.x, v[1] = x.y, v[2] = x.z, v[3] = x.w;
    v[4] = y.x, v[5] = y.y, v[6] = y.z, v[7] = y.w;
}

template <typename TI, typename TO, int NV, int G>
__global__ void __launch_bounds__(128)
local_corr_v_k(const TI *f1, long ps1, const TI *f2, long ps2, int H, int W, int r,
               const float *flow, TO *out, long ocs, long ops, int coff)
{
    constexpr int C = 8 * NV;
    __shared__ __align__(16) float a_s[4][C];
    __shared__ float S[4][CORR_MAXPS * CORR_MAXPS];
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const long n = (long)H * W;
    const long i = (long)blockIdx.x * 4 + w;
    if (i >= n)
        return;
    const int side = 2 * r + 1, ps = 2 * r + 2, P = ps * ps;
    const float rc = rsqrtf((float)C);
    const float ix = ((flow[i] + 1.0f) * W - 1.0f) * 0.5f;
    const float iy = ((flow[n + i] + 1.0f) * H - 1.0f) * 0.5f;
    const bool ok = isfinite(ix) && isfinite(iy);
    const int x0 = ok ? (int)floorf(ix) : 0, y0 = ok ? (int)floorf(iy) : 0;
    const float fx = ok ? ix - x0 : 0.0f, fy = ok ? iy - y0 : 0.0f;
    const TI *a = f1 + i * ps1;
    for (int c = lane; c < C; c += 32)
        a_s[w][c] = ldf(a + c) * rc;
    __syncwarp();
    constexpr int per = 32 / G;
    const int g = lane % G;
    for (int e0 = 0; e0 < P; e0 += per) {
        const int e = e0 + lane / G;
        const int yy = y0 - r + e / ps, xx = x0 - r + e % ps;
        float2 acc = make_float2(0.0f, 0.0f);
        if (e < P && ok && xx >= 0 && xx < W && yy >= 0 && yy < H) {
            const TI *b = f2 + ((long)yy * W + xx) * ps2;
#pragma unroll
            for (int v = g; v < NV; v += G) {
                float x[8];
                load8(b + 8 * v, x);
                const float4 p0 = *(const float4 *)&a_s[w][8 * v];
                const float4 p1 = *(const float4 *)&a_s[w][8 * v + 4];
                acc = fma2(make_float2(x[0], x[1]), make_float2(p0.x, p0.y), acc);
                acc = fma2(make_float2(x[2], x[3]), make_float2(p0.z, p0.w), acc);
                acc = fma2(make_float2(x[4], x[5]), make_float2(p1.x, p1.y), acc);
                acc = fma2(make_float2(x[6], x[7]), make_float2(p1.z, p1.w), acc);
            }
        }
        float sum = acc.x + acc.y;
#pragma unroll
        for (int o = G / 2; o > 0; o /= 2)
            sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (g == 0 && e < P)
            S[w][e] = sum;
    }
    __syncwarp();
    for (int k = lane; k < side * side; k += 32) {
        const int e0 = (k / side) * ps + k % side, e1 = e0 + ps;
        const float v = (1.0f - fy) * ((1.0f - fx) * S[w][e0] + fx * S[w][e0 + 1]) +
                        fy * ((1.0f - fx) * S[w][e1] + fx * S[w][e1 + 1]);
        stf(out + (long)(coff + k) * ocs + i * ops, v);
    }
}

// The compiled (channels, lanes per position) pairs of local_corr_v_k.
template <typename TI, typename TO>
static bool local_corr_v(cudaStream_t st, Map f1, Map f2, int C, int H, int W, int r,
                         const float *flow, MapOut out, int coff)
{
    if (r + 1 > CORR_MAXPS / 2 || f1.cs != 1 || f2.cs != 1 || f1.ps % 8 || f2.ps % 8 || ((uintptr_t)f1.p & 15) ||
        ((uintptr_t)f2.p & 15))
        return false;
    const long n = (long)H * W;
#define LCV(NV_, G_)                                                                          \
    if (C == 8 * NV_) {                                                            \
        local_corr_v_k<TI, TO, NV_, G_><<<cdiv(n, 4), 128, 0, st>>>(                          \
            (const TI *)f1.p, f1.ps, (const TI *)f2.p, f2.ps, H, W, r, flow, (TO *)out.p,      \
            out.cs, out.ps, coff);                                                            \
        return true;                                                                          \
    }
    LCV(64, 32)
    LCV(32, 16)
    LCV(24, 8)
    LCV(6, 2)
#undef LCV
    return false;
}

template <typename TI, typename TO>
static void local_corr_t(cudaStream_t st, Map f1, Map f2, int C, int H, int W,
                         int r, const float *flow, MapOut out, int coff)
{
    const long n = (long)H * W;
    if (local_corr_v<TI, TO>(st, f1, f2, C, H, W, r, flow, out, coff))
        return;
    if (sizeof(TI) == 2 && f1.cs == 1 && f2.cs == 1 && C % 8 == 0 && f1.ps % 8 == 0 &&
        f2.ps % 8 == 0 && ((uintptr_t)f1.p & 15) == 0 && ((uintptr_t)f2.p & 15) == 0) {
        local_corr_bf16_k<TO><<<cdiv(n, 4), 128, 0, st>>>(
            (const __nv_bfloat16 *)f1.p, f1.ps, (const __nv_bfloat16 *)f2.p, f2.ps, C, H, W, r,
            flow, (TO *)out.p, out.cs, out.ps, coff);
        return;
    }
    local_corr_k<TI, TO><<<cdiv(n, 4), 128, 0, st>>>(
        (const TI *)f1.p, f1.cs, f1.ps, (const TI *)f2.p, f2.cs, f2.ps, C, H, W,
        r, flow, (TO *)out.p, out.cs, out.ps, coff);
}

void roma_local_corr_l(cudaStream_t st, Map f1, Map f2, int C, int H, int W,
                       int r, const float *flow, MapOut out, int coff)
{
    if (C > CORR_MAXC || 2 * r + 2 > CORR_MAXPS || r < 0) {
        fail("roma_local_corr: C = %d > %d or radius %d > %d", C, CORR_MAXC, r,
             CORR_MAXPS / 2 - 1);
        return;
    }
    if ((long)H * W <= 0)
        return;
    if (f1.t == DT_F32 && out.t == DT_F32)
        local_corr_t<float, float>(st, f1, f2, C, H, W, r, flow, out, coff);
    else if (f1.t == DT_BF16 && out.t == DT_BF16)
        local_corr_t<__nv_bfloat16, __nv_bfloat16>(st, f1, f2, C, H, W, r, flow,
                                                   out, coff);
    else if (f1.t == DT_F32)
        local_corr_t<float, __nv_bfloat16>(st, f1, f2, C, H, W, r, flow, out,
                                           coff);
    else
        local_corr_t<__nv_bfloat16, float>(st, f1, f2, C, H, W, r, flow, out,
                                           coff);
}

// ----------------------------------------------------- displacement input

// Own cell centre of cell i of an H x W grid, normalized, align_corners
// False (roma_disp, roma_kernels.cl:196-208).
__device__ __forceinline__ void cell_centre(long i, int H, int W, float *gx,
                                            float *gy)
{
    *gx = -1.0f + 1.0f / W + (i % W) * (2.0f - 2.0f / W) / (W - 1);
    *gy = -1.0f + 1.0f / H + (i / W) * (2.0f - 2.0f / H) / (H - 1);
}

__global__ void disp_k(const float *flow, int H, int W, float fx, float fy,
                       float *out)
{
    const long n = (long)H * W;
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n)
        return;
    float gx, gy;
    cell_centre(i, H, W, &gx, &gy);
    out[i] = fx * (flow[i] - gx);
    out[n + i] = fy * (flow[n + i] - gy);
}

void roma_disp_l(cudaStream_t st, const float *flow, int H, int W, float fx,
                 float fy, float *out)
{
    const long n = (long)H * W;
    if (n > 0)
        disp_k<<<cdiv(n, 256), 256, 0, st>>>(flow, H, W, fx, fy, out);
}

// The displacement (as disp_k) through the refiner's disp_emb 1 x 1
// convolution (2 -> emb, the reference's ops_conv1x1 at roma.c:953-954),
// written into channels coff .. coff + emb - 1.
template <typename TO>
__global__ void disp_emb_k(const float *flow, int H, int W, float fx, float fy,
                           const float *ew, const float *eb, int emb, TO *out,
                           long ocs, long ops, int coff, int chan_fast)
{
    const long n = (long)H * W;
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n * emb)
        return;
    int k;
    long i;
    if (chan_fast) {
        k = (int)(e % emb);
        i = e / emb;
    }
    else {
        i = e % n;
        k = (int)(e / n);
    }
    float gx, gy;
    cell_centre(i, H, W, &gx, &gy);
    const float dx = fx * (flow[i] - gx), dy = fy * (flow[n + i] - gy);
    float acc = ew[2 * k] * dx;
    acc = fmaf(ew[2 * k + 1], dy, acc);
    stf(out + (long)(coff + k) * ocs + i * ops, acc + eb[k]);
}

// The same into a dense bfloat16 map, one thread per cell and 4
// embedding channels (8-byte stores), the displacement computed once.
__global__ void disp_emb4_k(const float *flow, int H, int W, float fx, float fy, const float *ew,
                            const float *eb, int emb4, uint2 *out, long ops4, int coff4,
                            int total)
{
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= total)
        return;
    const int g = e % emb4, i = e / emb4, n = H * W;
    float gx, gy;
    cell_centre(i, H, W, &gx, &gy);
    const float dx = fx * (flow[i] - gx), dy = fy * (flow[n + i] - gy);
    float r[4];
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const int k = 4 * g + c;
        float acc = ew[2 * k] * dx;
        acc = fmaf(ew[2 * k + 1], dy, acc);
        r[c] = acc + eb[k];
    }
    const __nv_bfloat162 a = __floats2bfloat162_rn(r[0], r[1]), b = __floats2bfloat162_rn(r[2], r[3]);
    uint2 o;
    o.x = *(const uint32_t *)&a;
    o.y = *(const uint32_t *)&b;
    out[(long)i * ops4 + coff4 + g] = o;
}

// The same for any embedding width and channel offset (RoMa v2's 79 and
// 23 channels): one thread per cell and 4 channels (the last group
// shorter), 32-bit indices, the displacement computed once per thread and
// the channels stored one by one.
template <typename TO>
__global__ void disp_emb_g_k(const float *flow, int H, int W, float fx, float fy,
                             const float *ew, const float *eb, int emb, TO *out, long ops,
                             int coff, int total)
{
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= total)
        return;
    const int groups = (emb + 3) / 4;
    const int g = e % groups, i = e / groups, n = H * W;
    float gx, gy;
    cell_centre(i, H, W, &gx, &gy);
    const float dx = fx * (flow[i] - gx), dy = fy * (flow[n + i] - gy);
    TO *o = out + (long)i * ops + coff;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const int k = 4 * g + c;
        if (k < emb) {
            float acc = ew[2 * k] * dx;
            acc = fmaf(ew[2 * k + 1], dy, acc);
            stf(o + k, acc + eb[k]);
        }
    }
}

void roma_disp_emb_l(cudaStream_t st, const float *flow, int H, int W, float fx,
                     float fy, const float *emb_w, const float *emb_b, int emb,
                     MapOut out, int coff)
{
    const long tot = (long)H * W * emb;
    if (tot <= 0)
        return;
    if (out.t == DT_BF16 && out.cs == 1 && emb % 4 == 0 && out.ps % 4 == 0 && coff % 4 == 0 &&
        ((uintptr_t)out.p & 7) == 0 && tot / 4 < (1L << 30)) {
        const int total = (int)(tot / 4);
        disp_emb4_k<<<cdiv(total, 256), 256, 0, st>>>(flow, H, W, fx, fy, emb_w, emb_b, emb / 4,
                                                      (uint2 *)out.p, out.ps / 4, coff / 4,
                                                      total);
        return;
    }
    const long groups = (long)H * W * ((emb + 3) / 4);
    if (out.cs == 1 && groups < (1L << 30) && (long)H * W < (1L << 30)) {
        if (out.t == DT_BF16)
            disp_emb_g_k<<<cdiv(groups, 256), 256, 0, st>>>(
                flow, H, W, fx, fy, emb_w, emb_b, emb, (__nv_bfloat16 *)out.p, out.ps, coff,
                (int)groups);
        else
            disp_emb_g_k<<<cdiv(groups, 256), 256, 0, st>>>(
                flow, H, W, fx, fy, emb_w, emb_b, emb, (float *)out.p, out.ps, coff,
                (int)groups);
        return;
    }
    if (out.t == DT_BF16)
        disp_emb_k<__nv_bfloat16><<<cdiv(tot, 256), 256, 0, st>>>(
            flow, H, W, fx, fy, emb_w, emb_b, emb, (__nv_bfloat16 *)out.p,
            out.cs, out.ps, coff, out.cs == 1);
    else
        disp_emb_k<float><<<cdiv(tot, 256), 256, 0, st>>>(
            flow, H, W, fx, fy, emb_w, emb_b, emb, (float *)out.p, out.cs,
            out.ps, coff, out.cs == 1);
}

// ---------------------------------------------------------------- updates

// roma_update, roma_kernels.cl:213-224.
__global__ void update_k(float *flow, float *cert, const float *d, long dcs,
                         long dps, int n, float scale, float Wf, float Hf)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n)
        return;
    flow[i] += scale * (d[i * dps] / (4.0f * Wf));
    flow[n + i] += scale * (d[dcs + i * dps] / (4.0f * Hf));
    cert[i] += d[2 * dcs + i * dps];
}

void roma_update_l(cudaStream_t st, float *flow, float *cert, Map d, int n,
                   float scale, float Wf, float Hf)
{
    if (n > 0)
        update_k<<<cdiv(n, 256), 256, 0, st>>>(flow, cert, (const float *)d.p,
                                               d.cs, d.ps, n, scale, Wf, Hf);
}

// softplus with torch's threshold 20 (roma_kernels.cl:230).
__device__ __forceinline__ float softplus20(float x)
{
    return x > 20.0f ? x : log1pf(expf(x));
}

// roma2_update, roma_kernels.cl:232-250.
__global__ void update2_k(float *flow, float *conf, const float *d, long dcs,
                          long dps, int n, float W, float H)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n)
        return;
    const float *di = d + (long)i * dps;
    flow[i] += di[0] / (4.0f * W);
    flow[n + i] += di[dcs] / (4.0f * H);
    const float l00 = softplus20(di[3 * dcs]) + 1e-6f;
    const float l10 = di[4 * dcs];
    const float l11 = softplus20(di[5 * dcs]) + 1e-6f;
    conf[i] += di[2 * dcs];
    conf[n + i] += l00 * l00;
    conf[2 * n + i] += l00 * l10;
    conf[3 * n + i] += l10 * l10 + l11 * l11;
}

void roma2_update_l(cudaStream_t st, float *flow, float *conf, Map d, int n,
                    float W, float H)
{
    if (n > 0)
        update2_k<<<cdiv(n, 256), 256, 0, st>>>(flow, conf, (const float *)d.p,
                                                d.cs, d.ps, n, W, H);
}

// --------------------------------------------------------------- dwconv5

// roma_dwconv5, roma_kernels.cl:256-284: depthwise 5 x 5, stride 1, zero
// padding 2, bias, ReLU; weights (C, 25).
template <typename TI, typename TO>
__global__ void dwconv5_k(const TI *in, long cs, long ps, int C, int H, int W,
                          const float *wt, const float *bias, TO *out, long ocs,
                          long ops, int chan_fast)
{
    const long n = (long)H * W;
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n * C)
        return;
    int c;
    long i;
    if (chan_fast) {
        c = (int)(e % C);
        i = e / C;
    }
    else {
        i = e % n;
        c = (int)(e / n);
    }
    const int y = (int)(i / W), x = (int)(i % W);
    const float *w = wt + c * 25;
    float acc = bias[c];
#pragma unroll
    for (int a = 0; a < 5; a++) {
        const int yy = y + a - 2;
        if (yy < 0 || yy >= H)
            continue;
#pragma unroll
        for (int b = 0; b < 5; b++) {
            const int xx = x + b - 2;
            if (xx < 0 || xx >= W)
                continue;
            acc = fmaf(at_map(in, cs, ps, c, (long)yy * W + xx), w[a * 5 + b],
                       acc);
        }
    }
    stf(out + (long)c * ocs + i * ops, fmaxf(acc, 0.0f));
}

// The same on token-major maps (channel stride 1, cell stride ps / ops):
// a 16 x 16 cell x 32 channel tile per block, its 20 x 20 input halo in
// shared memory; lane = channel, each thread two rows of 16 outputs with
// a sliding 5 x 5 window in registers (5 shared-memory reads per output
// instead of 25).
#define DW_T 16
template <typename TI, typename TO, int DW_C>
__global__ void __launch_bounds__(256)
dwconv5_tm_k(const TI *in, long ps, int C, int H, int W, const float *wt,
             const float *bias, TO *out, long ops)
{
    __shared__ TI tile[DW_T + 4][DW_T + 4][DW_C];
    const int tid = threadIdx.x, c0 = blockIdx.z * DW_C;
    const int x0 = blockIdx.x * DW_T - 2, y0 = blockIdx.y * DW_T - 2;
    for (int e = tid; e < (DW_T + 4) * (DW_T + 4) * DW_C; e += 256) {
        const int c = e % DW_C, px = (e / DW_C) % (DW_T + 4), py = e / (DW_C * (DW_T + 4));
        const int x = x0 + px, y = y0 + py;
        TI v = TI(0.0f);
        if (x >= 0 && x < W && y >= 0 && y < H && c0 + c < C)
            v = in[((long)y * W + x) * ps + c0 + c];
        tile[py][px][c] = v;
    }
    __syncthreads();
    const int c = tid % DW_C, cg = c0 + c;
    if (cg >= C)
        return;
    float w[25];
#pragma unroll
    for (int i = 0; i < 25; i++)
        w[i] = wt[cg * 25 + i];
    const float b = bias[cg];
    for (int oy = tid / DW_C; oy < DW_T; oy += 256 / DW_C) {
        const int y = blockIdx.y * DW_T + oy;
        if (y >= H)
            break;
        float win[5][5];
#pragma unroll
        for (int a = 0; a < 5; a++)
#pragma unroll
            for (int k = 0; k < 4; k++)
                win[a][k + 1] = ldf(&tile[oy + a][k][c]);
        for (int ox = 0; ox < DW_T; ox++) {
#pragma unroll
            for (int a = 0; a < 5; a++) {
#pragma unroll
                for (int k = 0; k < 4; k++)
                    win[a][k] = win[a][k + 1];
                win[a][4] = ldf(&tile[oy + a][ox + 4][c]);
            }
            const int x = blockIdx.x * DW_T + ox;
            if (x >= W)
                break;
            float acc = b;
#pragma unroll
            for (int a = 0; a < 5; a++)
#pragma unroll
                for (int k = 0; k < 5; k++)
                    acc = fmaf(win[a][k], w[a * 5 + k], acc);
            stf(out + ((long)y * W + x) * ops + cg, fmaxf(acc, 0.0f));
        }
    }
}

// bfloat16 channels-last depthwise 5 x 5 (+ bias, ReLU) for maps whose
// pixel pitch and channel count are multiples of 8: a 16 x 16 pixel x 32
// channel block stages its 20 x 20 halo tile with 16-byte loads into shared
// memory as bfloat16 pairs (rows padded by 16 words, so that the two
// output rows of a warp read different banks); each thread then computes
// one output row of 16 pixels for one channel pair, accumulating the 5
// input rows in turn (every input pixel feeds up to 5 outputs of the row)
// with packed float32 FMAs.
constexpr int DWP_T = 16, DWP_C = 32, DWP_TW = DWP_T + 4;
constexpr int DWP_RP = DWP_TW * (DWP_C / 2) + 16;  // words per tile row

__global__ void __launch_bounds__(256)
dwconv5_pair_k(const __nv_bfloat16 *in, long ps, int C, int H, int W, const float *wt,
               const float *bias, __nv_bfloat16 *out, long ops)
{
    __shared__ __align__(16) uint32_t tile[DWP_TW * DWP_RP];
    // The block's taps, tap-major with channel pairs innermost (a row's five
    // taps are five conflict-free 8-byte reads; global loads there stalled
    // every row on their latency).
    __shared__ float2 wsm[25][DWP_C / 2];
    const int tid = threadIdx.x, c0 = blockIdx.z * DWP_C;
    const int x0 = blockIdx.x * DWP_T - 2, y0 = blockIdx.y * DWP_T - 2;
    for (int e = tid; e < 25 * (DWP_C / 2); e += 256) {
        const int q = e % (DWP_C / 2), tap = e / (DWP_C / 2), c = c0 + 2 * q;
        wsm[tap][q] = c < C ? make_float2(wt[c * 25 + tap], wt[(c + 1) * 25 + tap])
                            : make_float2(0.0f, 0.0f);
    }
    for (int e = tid; e < DWP_TW * DWP_TW * (DWP_C / 8); e += 256) {
        const int j = e % (DWP_C / 8), px = (e / (DWP_C / 8)) % DWP_TW;
        const int py = e / ((DWP_C / 8) * DWP_TW);
        const int x = x0 + px, y = y0 + py, c = c0 + 8 * j;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (x >= 0 && x < W && y >= 0 && y < H && c < C)
            v = *(const uint4 *)(in + ((long)y * W + x) * ps + c);
        *(uint4 *)&tile[py * DWP_RP + px * (DWP_C / 2) + 4 * j] = v;
    }
    __syncthreads();
    const int pr = tid % (DWP_C / 2), oy = tid / (DWP_C / 2);
    const int cg = c0 + 2 * pr, y = blockIdx.y * DWP_T + oy;
    if (cg >= C || y >= H)
        return;
    float2 acc[DWP_T];
    const float2 b = make_float2(bias[cg], bias[cg + 1]);
#pragma unroll
    for (int i = 0; i < DWP_T; i++)
        acc[i] = b;
#pragma unroll 1
    for (int a = 0; a < 5; a++) {
        float2 w[5];
#pragma unroll
        for (int k = 0; k < 5; k++)
            w[k] = wsm[a * 5 + k][pr];
        const uint32_t *row = tile + (oy + a) * DWP_RP + pr;
#pragma unroll
        for (int x = 0; x < DWP_TW; x++) {
            const uint32_t u = row[x * (DWP_C / 2)];
            const float2 v = make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
#pragma unroll
            for (int k = 0; k < 5; k++) {
                const int ox = x - k;
                if (ox >= 0 && ox < DWP_T)
                    acc[ox] = fma2(v, w[k], acc[ox]);
            }
        }
    }
    __nv_bfloat16 *o = out + (long)y * W * ops + cg;
#pragma unroll
    for (int i = 0; i < DWP_T; i++) {
        const int x = blockIdx.x * DWP_T + i;
        if (x < W)
            *(__nv_bfloat162 *)(o + (long)x * ops) =
                __floats2bfloat162_rn(fmaxf(acc[i].x, 0.0f), fmaxf(acc[i].y, 0.0f));
    }
}

template <typename TI, typename TO>
static void dwconv5_t(cudaStream_t st, Map in, int C, int H, int W,
                      const float *w, const float *b, MapOut out)
{
    // Dense bfloat16 maps of a multiple of 64 channels: the TMA-fed kernel
    // (tc_dwpw.cu).
    if (sizeof(TI) == 2 && sizeof(TO) == 2 && in.cs == 1 && out.cs == 1 && in.ps == C &&
        out.ps == C && C % 64 == 0 && dw5_tc(st, in.p, H, W, C, w, b, out.p, 0))
        return;
    if (sizeof(TI) == 2 && sizeof(TO) == 2 && in.cs == 1 && out.cs == 1 && C % 8 == 0 &&
        in.ps % 8 == 0 && out.ps % 2 == 0 && ((uintptr_t)in.p & 15) == 0 &&
        ((uintptr_t)out.p & 3) == 0) {
        dim3 grid(cdiv(W, DWP_T), cdiv(H, DWP_T), cdiv(C, DWP_C));
        dwconv5_pair_k<<<grid, 256, 0, st>>>((const __nv_bfloat16 *)in.p, in.ps, C, H, W, w,
                                             b, (__nv_bfloat16 *)out.p, out.ps);
        return;
    }
    if (in.cs == 1 && out.cs == 1) {
        // 32 channels per block for 2-byte inputs, 16 for float (the
        // halo tile stays within 48 KB of shared memory).
        constexpr int CB = sizeof(TI) == 2 ? 32 : 16;
        dim3 grid(cdiv(W, DW_T), cdiv(H, DW_T), cdiv(C, CB));
        dwconv5_tm_k<TI, TO, CB><<<grid, 256, 0, st>>>((const TI *)in.p, in.ps, C, H, W, w,
                                                       b, (TO *)out.p, out.ps);
        return;
    }
    const long tot = (long)H * W * C;
    dwconv5_k<TI, TO><<<cdiv(tot, 256), 256, 0, st>>>(
        (const TI *)in.p, in.cs, in.ps, C, H, W, w, b, (TO *)out.p, out.cs,
        out.ps, in.cs == 1);
}

void roma_dwconv5_l(cudaStream_t st, Map in, int C, int H, int W,
                    const float *w, const float *b, MapOut out)
{
    if ((long)H * W * C <= 0)
        return;
    if (in.t == DT_F32 && out.t == DT_F32)
        dwconv5_t<float, float>(st, in, C, H, W, w, b, out);
    else if (in.t == DT_BF16 && out.t == DT_BF16)
        dwconv5_t<__nv_bfloat16, __nv_bfloat16>(st, in, C, H, W, w, b, out);
    else if (in.t == DT_F32)
        dwconv5_t<float, __nv_bfloat16>(st, in, C, H, W, w, b, out);
    else
        dwconv5_t<__nv_bfloat16, float>(st, in, C, H, W, w, b, out);
}

// ------------------------------------------------------- layout helpers

template <typename T>
__global__ void maxpool2_tm_k(const T *in, int H, int W, int C, T *out)
{
    const int w2 = W / 2, h2 = H / 2;
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= (long)h2 * w2 * C)
        return;
    const int c = (int)(e % C);
    const long o = e / C;
    const int x = (int)(o % w2), y = (int)(o / w2);
    const T *p = in + ((long)(2 * y) * W + 2 * x) * C + c;
    float v = -INFINITY;
    v = fmaxf(v, ldf(p));
    v = fmaxf(v, ldf(p + C));
    v = fmaxf(v, ldf(p + (long)W * C));
    v = fmaxf(v, ldf(p + (long)W * C + C));
    stf(out + e, v);
}

// bfloat16 with C a multiple of 8: one thread per output pixel and 8
// channels, 16-byte loads and store (max of bfloat16 values is exact in
// bfloat16).
__global__ void maxpool2_tm8_k(const uint4 *in, int H, int W, int C8, uint4 *out)
{
    const int w2 = W / 2, h2 = H / 2;
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= (long)h2 * w2 * C8)
        return;
    const int c = (int)(e % C8);
    const long o = e / C8;
    const int x = (int)(o % w2), y = (int)(o / w2);
    const uint4 *p = in + ((long)(2 * y) * W + 2 * x) * C8 + c;
    const uint4 a = p[0], b = p[C8], d = p[(long)W * C8], f = p[(long)W * C8 + C8];
    const __nv_bfloat162 *pa = (const __nv_bfloat162 *)&a, *pb = (const __nv_bfloat162 *)&b,
                         *pd = (const __nv_bfloat162 *)&d, *pf = (const __nv_bfloat162 *)&f;
    uint4 r;
    __nv_bfloat162 *pr = (__nv_bfloat162 *)&r;
#pragma unroll
    for (int i = 0; i < 4; i++)
        pr[i] = __hmax2(__hmax2(pa[i], pb[i]), __hmax2(pd[i], pf[i]));
    out[e] = r;
}

void maxpool2_tm(cudaStream_t st, const void *in, DType t, int H, int W, int C,
                 void *out)
{
    const long tot = (long)(H / 2) * (W / 2) * C;
    if (tot <= 0)
        return;
    if (t == DT_BF16 && C % 8 == 0 && ((uintptr_t)in & 15) == 0 && ((uintptr_t)out & 15) == 0) {
        maxpool2_tm8_k<<<cdiv(tot / 8, 256), 256, 0, st>>>((const uint4 *)in, H, W, C / 8,
                                                          (uint4 *)out);
        return;
    }
    if (t == DT_BF16)
        maxpool2_tm_k<__nv_bfloat16><<<cdiv(tot, 256), 256, 0, st>>>(
            (const __nv_bfloat16 *)in, H, W, C, (__nv_bfloat16 *)out);
    else
        maxpool2_tm_k<float><<<cdiv(tot, 256), 256, 0, st>>>(
            (const float *)in, H, W, C, (float *)out);
}

template <typename TS, typename TD>
__global__ void copy2d_k(const TS *src, long sp, TD *dst, long dp, long rows,
                         long cols)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= rows * cols)
        return;
    const long r = e / cols, c = e % cols;
    stf(dst + r * dp + c, ldf(src + r * sp + c));
}

// The same-type copy in chunks of V elements (V * element size = 16, 8 or
// 4 bytes) per thread, for pitches, widths and addresses that allow it:
// one vector load and store each instead of V scalar ones, and the
// 64-bit index division once per chunk.
template <typename W>
__global__ void copy2d_vec_k(const W *src, long sp, W *dst, long dp, long rows, long cols)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= rows * cols)
        return;
    const long r = e / cols, c = e % cols;
    dst[r * dp + c] = src[r * sp + c];
}

// Chunk bytes (16, 8 or 4) that divide every pitch, the width and both
// addresses, in bytes; 0 if none does.
static int copy_chunk(const void *src, long spb, const void *dst, long dpb, long colsb)
{
    for (int b = 16; b >= 4; b /= 2)
        if (((uintptr_t)src % b) == 0 && ((uintptr_t)dst % b) == 0 && spb % b == 0 &&
            dpb % b == 0 && colsb % b == 0)
            return b;
    return 0;
}

void copy2d(cudaStream_t st, const void *src, DType ts, long spitch, void *dst,
            DType td, long dpitch, long rows, long cols)
{
    const long tot = rows * cols;
    if (tot <= 0)
        return;
    if (ts == td) {
        const long es = ts == DT_F32 ? 4 : 2;
        const int b = copy_chunk(src, spitch * es, dst, dpitch * es, cols * es);
        const long cw = cols * es / (b ? b : 1), sw = spitch * es / (b ? b : 1),
                   dw = dpitch * es / (b ? b : 1);
        const unsigned gv = cdiv(rows * cw, 256);
        if (b == 16) {
            copy2d_vec_k<<<gv, 256, 0, st>>>((const uint4 *)src, sw, (uint4 *)dst, dw, rows, cw);
            return;
        }
        if (b == 8) {
            copy2d_vec_k<<<gv, 256, 0, st>>>((const uint2 *)src, sw, (uint2 *)dst, dw, rows, cw);
            return;
        }
        if (b == 4) {
            copy2d_vec_k<<<gv, 256, 0, st>>>((const uint32_t *)src, sw, (uint32_t *)dst, dw,
                                             rows, cw);
            return;
        }
    }
    const unsigned g = cdiv(tot, 256);
    if (ts == DT_F32 && td == DT_F32)
        copy2d_k<<<g, 256, 0, st>>>((const float *)src, spitch, (float *)dst,
                                     dpitch, rows, cols);
    else if (ts == DT_F32)
        copy2d_k<<<g, 256, 0, st>>>((const float *)src, spitch,
                                     (__nv_bfloat16 *)dst, dpitch, rows, cols);
    else if (td == DT_F32)
        copy2d_k<<<g, 256, 0, st>>>((const __nv_bfloat16 *)src, spitch,
                                     (float *)dst, dpitch, rows, cols);
    else
        copy2d_k<<<g, 256, 0, st>>>((const __nv_bfloat16 *)src, spitch,
                                     (__nv_bfloat16 *)dst, dpitch, rows, cols);
}

// Pillow's antialiased resampling (the reference's resize_axis,
// roma.c:1120-1155: double accumulation of precomputed, normalized taps),
// rows first into tmp (3, H, w), then columns into the channels-last
// output, normalized as prepare (roma.c:1178-1185).
__constant__ float c_mean[3] = {0.485f, 0.456f, 0.406f};
__constant__ float c_std[3] = {0.229f, 0.224f, 0.225f};

__global__ void pil_rows_k(const float *in, int H, int W, PilAxis ax,
                           float *tmp)
{
    const int o = blockIdx.x * blockDim.x + threadIdx.x;
    const int y = blockIdx.y, c = blockIdx.z;
    if (o >= ax.n_out)
        return;
    const float *src = in + ((size_t)c * H + y) * W + ax.start[o];
    const double *k = ax.weight + (size_t)o * ax.taps;
    double s = 0;
    for (int t = 0; t < ax.taps; t++)
        s += k[t] * src[t];
    tmp[((size_t)c * H + y) * ax.n_out + o] = (float)s;
}

template <typename TO>
__global__ void pil_cols_k(const float *tmp, int H, int w, PilAxis ay,
                           int identity, int norm, TO *out)
{
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int o = blockIdx.y, c = blockIdx.z;
    if (x >= w)
        return;
    float v;
    if (identity)
        v = tmp[((size_t)c * H + o) * w + x];
    else {
        const double *k = ay.weight + (size_t)o * ay.taps;
        const float *src = tmp + ((size_t)c * H + ay.start[o]) * w + x;
        double s = 0;
        for (int t = 0; t < ay.taps; t++)
            s += k[t] * src[(size_t)t * w];
        v = (float)s;
    }
    if (norm)
        v = (v - c_mean[c]) / c_std[c];
    stf(out + ((size_t)o * w + x) * 3 + c, v);
}

void pil_resize_norm(cudaStream_t st, const float *in, int H, int W, float *tmp,
                     PilAxis ax, PilAxis ay, int norm, void *out, DType t)
{
    const int w = ax.n_out, h = ay.n_out;
    const int identity = h == H && w == W;
    const float *rows = in;
    if (!identity) {
        pil_rows_k<<<dim3(cdiv(w, 128), H, 3), 128, 0, st>>>(in, H, W, ax, tmp);
        rows = tmp;
    }
    if (t == DT_BF16)
        pil_cols_k<__nv_bfloat16><<<dim3(cdiv(w, 128), h, 3), 128, 0, st>>>(
            rows, H, w, ay, identity, norm, (__nv_bfloat16 *)out);
    else
        pil_cols_k<float><<<dim3(cdiv(w, 128), h, 3), 128, 0, st>>>(
            rows, H, w, ay, identity, norm, (float *)out);
}

// The reference's host post-processing of roma_match on the device:
// match_v2 (roma.c:1333-1349): sd = det(P)^(-1/4) of the precision
// (p00, p10, p11) in prec (3, n), NAN if not positive; v1 (roma.c:1419-
// 1429): certainty attenuated by the upsampled coarse certainty low.
// Then sigmoid, zero where the warp leaves [-1, 1], warp clamped.
__global__ void finish_k(float *flow, float *cert, const float *prec,
                         const float *low, float *sd, long n)
{
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n)
        return;
    if (prec) {
        const double det = (double)prec[i] * prec[2 * n + i] -
                           (double)prec[n + i] * prec[n + i];
        sd[i] = det > 0 ? (float)pow(det, -0.25) : NAN;
    }
    float c = cert[i];
    if (low)
        c = c - (low[i] < 0 ? 0.5f * low[i] : 0.0f);
    c = 1.0f / (1.0f + expf(-c));
    float fx = flow[i], fy = flow[n + i];
    if (fabsf(fx) > 1 || fabsf(fy) > 1)
        c = 0;
    fx = fx < -1 ? -1 : fx > 1 ? 1 : fx;
    fy = fy < -1 ? -1 : fy > 1 ? 1 : fy;
    flow[i] = fx;
    flow[n + i] = fy;
    cert[i] = c;
}

void roma_finish_l(cudaStream_t st, float *flow, float *cert, const float *prec,
                   const float *low, float *sd, long n)
{
    if (n > 0)
        finish_k<<<cdiv(n, 256), 256, 0, st>>>(flow, cert, prec, low, sd, n);
}

}  // namespace coreg
