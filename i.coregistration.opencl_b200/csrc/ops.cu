// SPDX-License-Identifier: Unlicense
//
// The generic tensor operations of ops.h on CUDA. Each entry point keeps
// the argument meaning of the reference's ops.c / ops.cl entry point it
// replaces (cited per function); the kernels are this build's own.

#include <math.h>
#include <type_traits>
#include <string.h>

#include "gemm.cuh"

using namespace coreg;

// ------------------------------------------------------------------ setup

extern "C" void ops_init(struct ops *o, struct ocl_backend *ocl)
{
    memset(o, 0, sizeof(*o));
    o->ocl = ocl;
    o->precision = OPS_FP32;
    o->im2col_bytes = (size_t)256 << 20;
}

extern "C" void ops_free(struct ops *o)
{
    if (!o->ocl)
        return;
    ocl_release(&o->scratch);
    ocl_release(&o->scratch16);
    memset(o, 0, sizeof(*o));
}

extern "C" struct opnd ops_mat(cl_mem buf, long off, int ld)
{
    struct opnd m = {buf, off, ld, 0, 0};
    return m;
}

extern "C" struct opnd ops_bmat(cl_mem buf, long off, int ld, long s0, long s1)
{
    struct opnd m = {buf, off, ld, s0, s1};
    return m;
}

static bool need(cl_mem m, const char *what)
{
    if (!m) {
        fail("CUDA: %s: required buffer is NULL", what);
        return false;
    }
    return true;
}

static const int T256 = 256;

// ------------------------------------------------------------------- GEMM

// Float32 copy of an operand into bfloat16 (OPS_BF16 on ops_gemm and
// ops_gemm_noalloc): rows x cols of src (leading dimension ld) per batch
// product, packed; blockIdx.y walks the nb x rows rows with a stride of
// gridDim.y (at most 65535).
__global__ void to_bf16_kernel(const float *src, long ld, long s0, long s1,
                               int nb1, long nrows, int rows, int cols,
                               __nv_bfloat16 *dst)
{
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols)
        return;
    for (long br = blockIdx.y; br < nrows; br += gridDim.y) {
        const long b = br / rows, r = br % rows, b0 = b / nb1, b1 = b % nb1;
        dst[br * (long)cols + c] =
            __float2bfloat16_rn(src[b0 * s0 + b1 * s1 + r * ld + c]);
    }
}

// The same, eight columns per thread (two 16-byte loads, one 16-byte
// store) for rows whose starts are 16-byte aligned and cols a multiple of 8.
__global__ void to_bf16_v8_kernel(const float *src, long ld, long s0, long s1, int nb1,
                                  long nrows, int rows, int cols, __nv_bfloat16 *dst)
{
    const int c = 8 * (blockIdx.x * blockDim.x + threadIdx.x);
    if (c >= cols)
        return;
    for (long br = blockIdx.y; br < nrows; br += gridDim.y) {
        const long b = br / rows, r = br % rows, b0 = b / nb1, b1 = b % nb1;
        const float4 *p = (const float4 *)(src + b0 * s0 + b1 * s1 + r * ld + c);
        const float4 x = p[0], y = p[1];
        __nv_bfloat162 h[4] = {__floats2bfloat162_rn(x.x, x.y), __floats2bfloat162_rn(x.z, x.w),
                               __floats2bfloat162_rn(y.x, y.y), __floats2bfloat162_rn(y.z, y.w)};
        *(uint4 *)(dst + br * (long)cols + c) = *(const uint4 *)h;
    }
}

namespace coreg {

void pack_bf16_rows(cudaStream_t st, const float *src, long ld, long s0, long s1, int nb,
                    int nb1, int rows, int cols, __nv_bfloat16 *dst)
{
    const long nrows = (long)nb * rows;
    if (nrows <= 0 || cols <= 0)
        return;
    const unsigned gy = (unsigned)(nrows < 65535 ? nrows : 65535);
    if (cols % 8 == 0 && ld % 4 == 0 && s0 % 4 == 0 && s1 % 4 == 0 &&
        ((uintptr_t)src & 15) == 0 && ((uintptr_t)dst & 15) == 0) {
        to_bf16_v8_kernel<<<dim3(cdiv(cols / 8, 128), gy), 128, 0, st>>>(
            src, ld, s0, s1, nb1, nrows, rows, cols, dst);
        return;
    }
    to_bf16_kernel<<<dim3(cdiv(cols, 256), gy), 256, 0, st>>>(src, ld, s0, s1, nb1, nrows,
                                                               rows, cols, dst);
}


// 32 x 32 tiles of a float32 rows x cols batch product, transposed into
// bfloat16 (cols x rows); blockIdx.z is the batch.
__global__ void to_bf16_t_kernel(const float *src, long ld, long s0, long s1, int nb1,
                                 int rows, int cols, __nv_bfloat16 *dst)
{
    __shared__ float t[32][33];
    const long b = blockIdx.z, b0 = b / nb1, b1 = b % nb1;
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    const int x = threadIdx.x % 32, y = threadIdx.x / 32;
    const float *s = src + b0 * s0 + b1 * s1;
    for (int r = y; r < 32; r += blockDim.x / 32)
        t[r][x] = r0 + r < rows && c0 + x < cols ? s[(long)(r0 + r) * ld + c0 + x] : 0.0f;
    __syncthreads();
    __nv_bfloat16 *d = dst + b * (long)rows * cols;
    for (int c = y; c < 32; c += blockDim.x / 32)
        if (c0 + c < cols && r0 + x < rows)
            d[(long)(c0 + c) * rows + r0 + x] = __float2bfloat16_rn(t[x][c]);
}

void pack_bf16_cols(cudaStream_t st, const float *src, long ld, long s0, long s1, int nb,
                    int nb1, int rows, int cols, __nv_bfloat16 *dst)
{
    if (nb <= 0 || rows <= 0 || cols <= 0)
        return;
    to_bf16_t_kernel<<<dim3(cdiv(cols, 32), cdiv(rows, 32), nb), 256, 0, st>>>(
        src, ld, s0, s1, nb1, rows, cols, dst);
}

}  // namespace coreg

extern "C" void ops_gemm(struct ops *o, int M, int N, int K, struct opnd A,
                         struct opnd B, int transb, struct opnd C, int nb,
                         int nb1, cl_mem bias, int biasrow, cl_mem R, long roff,
                         float alpha, int act, float slope)
{
    GemmArgs g = gemm_args(M, N, K);

    if (pending() || !need(A.buf, "ops_gemm A") || !need(B.buf, "ops_gemm B") ||
        !need(C.buf, "ops_gemm C"))
        return;
    if (nb1 < 1 || nb < 1) {
        fail("ops_gemm: batch %d / %d", nb, nb1);
        return;
    }
    g.A = fptr(A.buf, A.off);
    g.lda = A.ld;
    g.sa0 = A.s0;
    g.sa1 = A.s1;
    g.B = fptr(B.buf, B.off);
    g.ldb = B.ld;
    g.sb0 = B.s0;
    g.sb1 = B.s1;
    g.transb = transb;
    g.C = fptr(C.buf, C.off);
    g.ldc = C.ld;
    g.sc0 = C.s0;
    g.sc1 = C.s1;
    g.nb = nb;
    g.nb1 = nb1;
    g.bias = fptr(bias);
    g.biasrow = biasrow;
    g.R = R ? fptr(R, roff) : nullptr;
    g.alpha = alpha;
    g.act = act;
    g.slope = slope;
    g.ab = DT_F32;
    g.c = DT_F32;
    if (gemm_packs_bf16(o->precision, M, N, K)) {
        // Pack both operands to bfloat16 (row-major, K contiguous), then
        // the tensor-core tiles.
        size_t ea = (size_t)nb * M * K, eb = (size_t)nb * N * K;
        size_t bytes = (ea + eb) * 2 + 256;

        if (bytes > o->scratch16_bytes) {
            ocl_release(&o->scratch16);
            o->scratch16 = ocl_alloc(o->ocl, bytes, "bf16 operands");
            o->scratch16_bytes = bytes;
            if (pending())
                return;
        }
        __nv_bfloat16 *a16 = (__nv_bfloat16 *)o->scratch16->ptr;
        __nv_bfloat16 *b16 = a16 + ((ea + 127) / 128) * 128;
        cudaStream_t st = stream_of(o->ocl);
        {
            Prof p(o->ocl, "gemm_pack_bf16");
            pack_bf16_rows(st, (const float *)g.A, g.lda, g.sa0, g.sa1, nb, nb1, M, K, a16);
            if (transb)
                pack_bf16_rows(st, (const float *)g.B, g.ldb, g.sb0, g.sb1, nb, nb1, N, K, b16);
            else
                pack_bf16_cols(st, (const float *)g.B, g.ldb, g.sb0, g.sb1, nb, nb1, K, N, b16);
            if (!launch_ok("gemm_pack_bf16"))
                return;
        }
        GemmArgs h = g;
        h.A = a16;
        h.lda = K;
        h.sa0 = (long)M * K * nb1;
        h.sa1 = (long)M * K;
        h.B = b16;
        h.ldb = K;
        h.sb0 = (long)N * K * nb1;
        h.sb1 = (long)N * K;
        h.transb = 1;
        h.ab = DT_BF16;
        gemm_run(o->ocl, h, "gemm_tc");
        return;
    }
    gemm_run(o->ocl, g, "gemm");
}

extern "C" void ops_linear(struct ops *o, int rows, int in, int out, cl_mem X,
                           long xoff, cl_mem W, cl_mem b, cl_mem Y, long yoff,
                           int act, float slope, int residual)
{
    ops_gemm(o, rows, out, in, ops_mat(X, xoff, in), ops_mat(W, 0, in), 1,
             ops_mat(Y, yoff, out), 1, 1, b, 0, residual ? Y : NULL, yoff, 1.0f,
             act, slope);
}

extern "C" void ops_conv1x1(struct ops *o, cl_mem X, long xoff, int C, int HW,
                            cl_mem W, cl_mem b, int K, cl_mem Y, long yoff,
                            int act, float slope)
{
    ops_gemm(o, K, HW, C, ops_mat(W, 0, C), ops_mat(X, xoff, HW), 0,
             ops_mat(Y, yoff, HW), 1, 1, b, 1, NULL, 0, 1.0f, act, slope);
}

// ------------------------------------------------------------ convolutions

extern "C" struct conv_geom ops_geom(int k, int s, int p)
{
    struct conv_geom g = {k, k, s, s, p, p, 1, 1, 1};
    return g;
}

extern "C" int ops_conv_out(int n, int k, int s, int p, int d)
{
    return (n + 2 * p - d * (k - 1) - 1) / s + 1;
}

// F.unfold of positions l0 .. l0 + n - 1 (ops.cl:799-816 semantics): row
// c * kh * kw + i * kw + j, column l - l0.
__global__ void unfold_kernel(const float *in, int C, int H, int W, int kh,
                              int kw, int sy, int sx, int py, int px, int dy,
                              int dx, int Wo, int l0, int n, float *out)
{
    const int t = blockIdx.x * blockDim.x + threadIdx.x;
    const int row = blockIdx.y;
    if (t >= n)
        return;
    const int c = row / (kh * kw), i = (row / kw) % kh, j = row % kw;
    const int l = l0 + t;
    const int iy = (l / Wo) * sy - py + i * dy;
    const int ix = (l % Wo) * sx - px + j * dx;
    out[(size_t)row * n + t] = iy >= 0 && iy < H && ix >= 0 && ix < W
                                   ? in[((size_t)c * H + iy) * W + ix]
                                   : 0.0f;
}

// Direct convolution, one thread per output value (ops.cl:397-448
// semantics, including the normalize-and-gate of the input before the
// zero padding).
__global__ void conv_direct_kernel(const float *in, int C, int H, int W,
                                   const float *wt, const float *bias, int K,
                                   int Ho, int Wo, int kh, int kw, int sy,
                                   int sx, int py, int px, int dy, int dx,
                                   int groups, const float *mean,
                                   const float *rstd, const float *alpha,
                                   int act, float slope, float *out)
{
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int y = blockIdx.y;
    const int k = blockIdx.z;
    if (x >= Wo)
        return;
    const int cg = C / groups, kg = K / groups, c0 = (k / kg) * cg;
    const float *w = wt + (size_t)k * cg * kh * kw;
    float acc = 0.0f;

    for (int c = 0; c < cg; c++) {
        const float *src = in + (size_t)(c0 + c) * H * W;
        float m = 0.0f, r = 1.0f, a = 1.0f;
        if (mean) {
            m = mean[c0 + c];
            r = rstd[c0 + c];
            if (alpha)
                a = alpha[c0 + c];
        }
        for (int i = 0; i < kh; i++) {
            const int iy = y * sy - py + i * dy;
            if (iy < 0 || iy >= H)
                continue;
            for (int j = 0; j < kw; j++) {
                const int ix = x * sx - px + j * dx;
                if (ix < 0 || ix >= W)
                    continue;
                float v = src[(size_t)iy * W + ix];
                if (mean) {
                    v = (v - m) * r;
                    v = v >= 0.0f ? v : a * v;
                }
                acc = fmaf(v, w[(c * kh + i) * kw + j], acc);
            }
        }
    }
    if (bias)
        acc += bias[k];
    out[((size_t)k * Ho + y) * Wo + x] = apply_act(acc, act, slope);
}

// Convolution as W (K, C kh kw) times the unfolded input, by blocks of
// output positions that fit the scratch buffer (the reference's
// conv_im2col, ops.c:238-265).
static void conv_im2col(struct ops *o, cl_mem in, int C, int H, int W, cl_mem w,
                        cl_mem b, int K, const struct conv_geom *g, int Ho,
                        int Wo, int act, float slope, cl_mem out)
{
    const int Kc = C * g->kh * g->kw, L = Ho * Wo;
    int blk = (int)(o->im2col_bytes / sizeof(float) / Kc) / 128 * 128;
    cudaStream_t st = stream_of(o->ocl);

    if (blk < 128)
        blk = 128;
    if (blk > L)
        blk = L;
    size_t bytes = (size_t)Kc * blk * sizeof(float);
    if (bytes > o->scratch_bytes) {
        ocl_release(&o->scratch);
        o->scratch = ocl_alloc(o->ocl, bytes, "im2col");
        o->scratch_bytes = bytes;
        if (pending())
            return;
    }
    for (int l0 = 0; l0 < L; l0 += blk) {
        const int n = L - l0 < blk ? L - l0 : blk;
        {
            Prof p(o->ocl, "unfold");
            unfold_kernel<<<dim3(cdiv(n, T256), Kc), T256, 0, st>>>(
                fptr(in), C, H, W, g->kh, g->kw, g->sy, g->sx, g->py, g->px,
                g->dy, g->dx, Wo, l0, n, fptr(o->scratch));
            if (!launch_ok("unfold"))
                return;
        }
        ops_gemm(o, K, n, Kc, ops_mat(w, 0, Kc), ops_mat(o->scratch, 0, n), 0,
                 ops_mat(out, l0, L), 1, 1, b, 1, NULL, 0, 1.0f, act, slope);
    }
}

// ------------------------------------- bfloat16 convolutions, tensor cores
//
// OPS_BF16 contexts run the stride-1 3 x 3 (padding 1) and 5 x 5 (padding
// 2) convolutions of ops_conv2d, normalized input included, on the tcgen05
// GEMM's implicit-convolution mode, keeping ops_conv2d's channel-major
// float32 layout on both sides:
//   1. the weights (K, C, k, k) float32 -> (K, k, k, Cp) bfloat16, C padded
//      to Cp, a multiple of 64, with zeros;
//   2. the input (C, H, W) float32 -> (H W, Cp) bfloat16, normalized and
//      PReLU-gated on the way when mean is given (the same arithmetic as
//      the float32 kernel: the gate before the zero padding, ops.cl:328-387);
//   3. the GEMM over k k Cp columns (one 3-D TMA box per tap and 64-channel
//      chunk, zeros outside the map) with bias and activation, into a
//      channels-last float32 map of 16-byte rows;
//   4. a transpose into out (K, H, W).
// Steps 1, 2 and 4 move the operands once; the product is the tensor
// cores'. All four buffers come from o->scratch16.

namespace {

int conv_cpad(int C) { return (C + 63) / 64 * 64; }
int conv_opitch(int K) { return (K + 3) / 4 * 4; }

// (K, C, kk) float32 -> (K, kk, Cp) bfloat16, zero for c >= C.
__global__ void conv_w16_k(const float *w, int K, int C, int kk, int Cp, __nv_bfloat16 *out)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= (long)K * kk * Cp)
        return;
    const int c = (int)(e % Cp), tap = (int)(e / Cp % kk), k = (int)(e / ((long)Cp * kk));
    out[e] = __float2bfloat16_rn(c < C ? w[((long)k * C + c) * kk + tap] : 0.0f);
}

// Input (C, n) float32 into n x Cp bfloat16 rows, gated as described
// above; channels C..Cp-1 zero. One block of 256 threads per `cells` cells
// (64, 32 or 16, so that the Cp x (cells + 1) tile fits 48 KB of shared
// memory): coalesced reads along the cells of a channel, coalesced writes
// along the channels of a cell.
__host__ __device__ inline int gate_cells(int Cp) { return Cp <= 128 ? 64 : Cp <= 256 ? 32 : 16; }
__global__ void __launch_bounds__(256)
conv_gate_cl_k(const float *in, int C, long n, const float *mean, const float *rstd,
               const float *alpha, int Cp, __nv_bfloat16 *out)
{
    extern __shared__ float tile[];  // Cp x (cells + 1)
    const int cells = gate_cells(Cp);
    const long p0 = (long)blockIdx.x * cells;
    const int tx = threadIdx.x % cells, ty = threadIdx.x / cells;
    for (int c = ty; c < Cp; c += blockDim.x / cells) {
        float v = 0.0f;
        if (c < C && p0 + tx < n) {
            v = in[(long)c * n + p0 + tx];
            if (mean) {
                v = (v - mean[c]) * rstd[c];
                const float a = alpha ? alpha[c] : 1.0f;
                v = v >= 0.0f ? v : a * v;
            }
        }
        tile[c * (cells + 1) + tx] = v;
    }
    __syncthreads();
    const int pairs = Cp / 2;
    for (int e = threadIdx.x; e < cells * pairs; e += blockDim.x) {
        const int px = e / pairs, c = 2 * (e % pairs);
        if (p0 + px < n)
            *(__nv_bfloat162 *)(out + (p0 + px) * Cp + c) = __floats2bfloat162_rn(
                tile[c * (cells + 1) + px], tile[(c + 1) * (cells + 1) + px]);
    }
}

// Channels-last (n x ld) float32 -> channel-major (K, n), 32 x 32 tiles.
__global__ void conv_to_cm_k(const float *in, long n, int ld, int K, float *out)
{
    __shared__ float t[32][33];
    const long p0 = (long)blockIdx.x * 32;
    const int k0 = blockIdx.y * 32, x = threadIdx.x % 32, y = threadIdx.x / 32;
    for (int r = y; r < 32; r += blockDim.x / 32)
        if (p0 + r < n && k0 + x < K)
            t[r][x] = in[(p0 + r) * ld + k0 + x];
    __syncthreads();
    for (int r = y; r < 32; r += blockDim.x / 32)
        if (k0 + r < K && p0 + x < n)
            out[(long)(k0 + r) * n + p0 + x] = t[x][r];
}

// Whether ops_conv2d takes the tensor-core path: a bfloat16 context, a
// stride-1 3 x 3 / padding 1 or 5 x 5 / padding 2 convolution without
// groups or dilation, at most 512 input channels (the gate tile's shared
// memory) and at least 64 output positions (one tensor-core row block).
bool conv_tc_geometry(const struct ops *o, int C, int H, int W, const struct conv_geom *g)
{
    return o->precision == OPS_BF16 && g->groups == 1 && g->dy == 1 && g->dx == 1 &&
           g->sy == 1 && g->sx == 1 && g->kh == g->kw && (g->kh == 3 || g->kh == 5) &&
           g->py == g->kh / 2 && g->px == g->kw / 2 && (long)H * W >= 64 &&
           conv_cpad(C) <= 512;
}

// The tensor-core convolution; false (after recording an error, or with
// nothing launched when the GEMM does not take the shape) otherwise.
bool conv2d_tc(struct ops *o, cl_mem in, int C, int H, int W, cl_mem w, cl_mem b, int K,
               int ks, cl_mem mean, cl_mem rstd, cl_mem alpha, int act, float slope,
               cl_mem out)
{
    const long n = (long)H * W;
    const int Cp = conv_cpad(C), kk = ks * ks, ld = conv_opitch(K);
    const size_t wb = ((size_t)K * kk * Cp * 2 + 255) / 256 * 256;
    const size_t ib = ((size_t)n * Cp * 2 + 255) / 256 * 256;
    const size_t bytes = wb + ib + (size_t)n * ld * 4;
    if (n >= (1L << 31) / ld)
        return false;
    GemmArgs gg = gemm_args((int)n, K, kk * Cp);
    gg.amode = 1;
    gg.cK = ks;
    gg.cH = H;
    gg.cW = W;
    gg.cC = Cp;
    gg.ldb = kk * Cp;
    gg.transb = 1;
    gg.ldc = ld;
    gg.bias = fptr(b);
    gg.act = act;
    gg.slope = slope;
    gg.ab = DT_BF16;
    gg.c = DT_F32;
    if (bytes > o->scratch16_bytes) {
        ocl_release(&o->scratch16);
        o->scratch16 = ocl_alloc(o->ocl, bytes, "convolution operands");
        o->scratch16_bytes = bytes;
        if (pending())
            return false;
    }
    char *base = (char *)o->scratch16->ptr;
    __nv_bfloat16 *w16 = (__nv_bfloat16 *)base, *a16 = (__nv_bfloat16 *)(base + wb);
    float *cl = (float *)(base + wb + ib);
    gg.A = a16;
    gg.B = w16;
    gg.C = cl;
    cudaStream_t st = stream_of(o->ocl);
    Prof p(o->ocl, ks == 5 ? "conv5x5_tc" : "conv3x3_tc");
    const int cells = gate_cells(Cp);
    conv_w16_k<<<cdiv((long)K * kk * Cp, 256), 256, 0, st>>>(fptr(w), K, C, kk, Cp, w16);
    conv_gate_cl_k<<<cdiv(n, cells), 256, Cp * (cells + 1) * 4, st>>>(
        fptr(in), C, n, fptr(mean), fptr(rstd), fptr(alpha), Cp, a16);
    if (!launch_ok("convolution operands"))
        return false;
    if (!gemm_tc(st, gg, o->ocl->sm_count))
        return false;
    conv_to_cm_k<<<dim3(cdiv(n, 32), cdiv(K, 32)), 256, 0, st>>>(cl, n, ld, K, fptr(out));
    return launch_ok(ks == 5 ? "conv5x5_tc" : "conv3x3_tc");
}

}  // namespace

extern "C" void ops_conv2d(struct ops *o, cl_mem in, int C, int H, int W,
                           cl_mem w, cl_mem b, int K, const struct conv_geom *g,
                           cl_mem mean, cl_mem rstd, cl_mem alpha, int act,
                           float slope, cl_mem out)
{
    if (pending() || !need(in, "ops_conv2d in") || !need(w, "ops_conv2d w") ||
        !need(out, "ops_conv2d out"))
        return;
    const int Ho = ops_conv_out(H, g->kh, g->sy, g->py, g->dy);
    const int Wo = ops_conv_out(W, g->kw, g->sx, g->px, g->dx);

    if (g->groups < 1 || C % g->groups || K % g->groups) {
        fail("CUDA: %d -> %d channels in %d groups", C, K, g->groups);
        return;
    }
    if (mean && !rstd) {
        fail("ops_conv2d: mean without rstd");
        return;
    }
    if (!count_ok((long)C * H * W, "convolution input") ||
        !count_ok((long)K * Ho * Wo, "convolution output"))
        return;
    if (Ho <= 0 || Wo <= 0)
        return;
    if (conv_tc_geometry(o, C, H, W, g) &&
        conv2d_tc(o, in, C, H, W, w, b, K, g->kh, mean, rstd, alpha, act, slope, out))
        return;
    if (pending())
        return;
    if (g->groups == 1 && !mean && !alpha && g->dy == 1 && g->dx == 1 &&
        (long)C * g->kh * g->kw * Ho * Wo >= 4096) {
        if (!count_ok((long)C * g->kh * g->kw * 128, "im2col block"))
            return;
        conv_im2col(o, in, C, H, W, w, b, K, g, Ho, Wo, act, slope, out);
        return;
    }
    Prof p(o->ocl, "conv2d");
    conv_direct_kernel<<<dim3(cdiv(Wo, 64), Ho, K), 64, 0, stream_of(o->ocl)>>>(
        fptr(in), C, H, W, fptr(w), fptr(b), K, Ho, Wo, g->kh, g->kw, g->sy,
        g->sx, g->py, g->px, g->dy, g->dx, g->groups, fptr(mean), fptr(rstd),
        fptr(alpha), act, slope, fptr(out));
    launch_ok("conv2d");
}

// (K, C, 3, 3) -> (K, 3, 3, C), converted to T.
template <typename T>
__global__ void conv3_reorder_k(const float *w, int K, int C, T *out)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= (long)K * C * 9)
        return;
    const int c = (int)(e % C), t = (int)((e / C) % 9), k = (int)(e / (9L * C));
    stf(out + e, w[((long)k * C + c) * 9 + t]);
}

template <typename T>
__global__ void to_type_k(const float *in, long n, T *out)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < n)
        stf(out + e, in[e]);
}

// (K, C, 3, 3) float32 weights -> (K, kp) bfloat16 rows in (tap, channel)
// order, zero beyond 9 C: the B operand of the few-channel convolution.
__global__ void conv3_reorder_pad_k(const float *w, int K, int C, int kp, __nv_bfloat16 *out)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= (long)K * kp)
        return;
    const int k = (int)(e / kp), j = (int)(e % kp);
    float v = 0.0f;
    if (j < 9 * C)
        v = w[((long)k * C + j % C) * 9 + j / C];
    out[e] = __float2bfloat16_rn(v);
}

// Explicit im2col of a 3 x 3 / stride 1 / padding 1 convolution over a
// channels-last bfloat16 map: row = pixel, column j = tap * C + c for
// j < 9 C (zeros outside the map), zero up to kp (a multiple of 8). One
// thread per 8 columns of a row: one 16-byte store.
__global__ void im2col3_small_k(const __nv_bfloat16 *in, int H, int W, int C, int kp,
                                __nv_bfloat16 *col)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const int chunks = kp / 8;
    const long n = (long)H * W;
    if (e >= n * chunks)
        return;
    const long pix = e / chunks;
    const int j0 = (int)(e % chunks) * 8;
    const int px = (int)(pix % W), py = (int)(pix / W);
    __align__(16) __nv_bfloat16 v[8];
#pragma unroll
    for (int q = 0; q < 8; q++) {
        const int j = j0 + q;
        __nv_bfloat16 x = __float2bfloat16_rn(0.0f);
        if (j < 9 * C) {
            const int t = j / C, c = j % C;
            const int xx = px + t % 3 - 1, yy = py + t / 3 - 1;
            if (xx >= 0 && xx < W && yy >= 0 && yy < H)
                x = in[((long)yy * W + xx) * C + c];
        }
        v[q] = x;
    }
    *(uint4 *)(col + pix * kp + j0) = *(const uint4 *)v;
}

// The same for a compile-time channel count: one thread per pixel writes
// its whole row (9 C values, zeros up to KP) with 16-byte stores, the 3 x 3
// neighbourhood read once.
template <int C, int KP>
__global__ void im2col3_row_k(const __nv_bfloat16 *in, int H, int W, __nv_bfloat16 *col)
{
    const int pix = blockIdx.x * blockDim.x + threadIdx.x;
    if (pix >= H * W)
        return;
    const int px = pix % W, py = pix / W;
    __align__(16) __nv_bfloat16 v[KP];
#pragma unroll
    for (int t = 0; t < 9; t++) {
        const int xx = px + t % 3 - 1, yy = py + t / 3 - 1;
        const bool in_map = xx >= 0 && xx < W && yy >= 0 && yy < H;
        const __nv_bfloat16 *p = in + ((long)yy * W + xx) * C;
#pragma unroll
        for (int c = 0; c < C; c++)
            v[t * C + c] = in_map ? p[c] : __float2bfloat16_rn(0.0f);
    }
#pragma unroll
    for (int j = 9 * C; j < KP; j++)
        v[j] = __float2bfloat16_rn(0.0f);
    uint4 *dst = (uint4 *)(col + (long)pix * KP);
#pragma unroll
    for (int q = 0; q < KP / 8; q++)
        dst[q] = ((const uint4 *)v)[q];
}

namespace coreg {

void conv3x3_im2col_tc(cudaStream_t st, const __nv_bfloat16 *in, int H, int W, int C, int kp,
                       const __nv_bfloat16 *wk, const float *bias, int K, int act,
                       float slope, void *out, DType ot, __nv_bfloat16 *col, int sm_count)
{
    const long n = (long)H * W;
    // RGB to 64 channels with ReLU: one kernel, no im2col buffer.
    if (C == 3 && kp == 32 && K == 64 && act == ACTF_RELU &&
        conv_rgb_tc(st, in, H, W, wk, bias, out, ot, sm_count))
        return;
    if (C == 3 && kp == 32 && n < (1L << 31))
        im2col3_row_k<3, 32><<<cdiv(n, 256), 256, 0, st>>>(in, H, W, col);
    else
        im2col3_small_k<<<cdiv(n * (kp / 8), 256), 256, 0, st>>>(in, H, W, C, kp, col);
    GemmArgs g = gemm_args((int)n, K, kp);
    g.A = col;
    g.lda = kp;
    g.B = wk;
    g.ldb = kp;
    g.transb = 1;
    g.C = out;
    g.ldc = K;
    g.bias = bias;
    g.act = act;
    g.slope = slope;
    g.ab = DT_BF16;
    g.c = ot;
    if (!gemm_tc(st, g, sm_count))
        gemm_simt(st, g);
}

}  // namespace coreg

extern "C" void ops_conv3x3_cl(struct ops *o, cl_mem in, int H, int W, int C,
                               cl_mem w, cl_mem b, int K, int act, float slope,
                               cl_mem out)
{
    if (pending() || !need(in, "ops_conv3x3_cl in") || !need(w, "w") ||
        !need(out, "out"))
        return;
    const long n = (long)H * W;
    if (!count_ok(n * C, "conv3x3 input") || !count_ok(n * K, "conv3x3 output") ||
        n <= 0 || K <= 0 || C <= 0)
        return;
    const bool tc = o->precision == OPS_BF16 && C % 64 == 0;
    if (o->precision == OPS_BF16 && !tc && 9 * C <= 64) {
        // Few channels: explicit im2col of kp columns, then the tensor
        // cores.
        const int kp = (9 * C + 15) / 16 * 16;
        const size_t wb = ((size_t)K * kp * 2 + 255) / 256 * 256;
        const size_t ib = ((size_t)n * C * 2 + 255) / 256 * 256;
        const size_t bytes = wb + ib + (size_t)n * kp * 2;
        if (bytes > o->scratch16_bytes) {
            ocl_release(&o->scratch16);
            o->scratch16 = ocl_alloc(o->ocl, bytes, "conv3x3 operands");
            o->scratch16_bytes = bytes;
            if (pending())
                return;
        }
        char *base = (char *)o->scratch16->ptr;
        __nv_bfloat16 *wk = (__nv_bfloat16 *)base, *a16 = (__nv_bfloat16 *)(base + wb);
        __nv_bfloat16 *col = (__nv_bfloat16 *)(base + wb + ib);
        cudaStream_t st = stream_of(o->ocl);
        Prof p(o->ocl, "conv3x3_tc");
        conv3_reorder_pad_k<<<cdiv((long)K * kp, 256), 256, 0, st>>>(fptr(w), K, C, kp, wk);
        to_type_k<__nv_bfloat16><<<cdiv(n * C, 256), 256, 0, st>>>(fptr(in), n * C, a16);
        conv3x3_im2col_tc(st, a16, H, W, C, kp, wk, fptr(b), K, act, slope, out->ptr, DT_F32,
                          col, o->ocl->sm_count);
        launch_ok("conv3x3_tc");
        return;
    }
    const size_t es = tc ? 2 : 4;
    const size_t wbytes = ((size_t)K * 9 * C * es + 255) / 256 * 256;
    const size_t bytes = wbytes + (tc ? (size_t)n * C * 2 : 0);
    cl_mem *scr = tc ? &o->scratch16 : &o->scratch;
    size_t *cap = tc ? &o->scratch16_bytes : &o->scratch_bytes;
    if (bytes > *cap) {
        ocl_release(scr);
        *scr = ocl_alloc(o->ocl, bytes, "conv3x3 operands");
        *cap = bytes;
        if (pending())
            return;
    }
    cudaStream_t st = stream_of(o->ocl);
    void *wr = (*scr)->ptr, *a = in->ptr;
    const long nw = (long)K * 9 * C;
    {
        Prof p(o->ocl, "conv3x3_pack");
        if (tc) {
            conv3_reorder_k<__nv_bfloat16><<<cdiv(nw, 256), 256, 0, st>>>(
                fptr(w), K, C, (__nv_bfloat16 *)wr);
            a = (char *)wr + wbytes;
            to_type_k<__nv_bfloat16><<<cdiv(n * C, 256), 256, 0, st>>>(
                fptr(in), n * C, (__nv_bfloat16 *)a);
        }
        else
            conv3_reorder_k<float><<<cdiv(nw, 256), 256, 0, st>>>(fptr(w), K, C,
                                                                  (float *)wr);
        if (!launch_ok("conv3x3_pack"))
            return;
    }
    GemmArgs g = gemm_args((int)n, K, 9 * C);
    g.A = a;
    g.amode = 1;
    g.cH = H;
    g.cW = W;
    g.cC = C;
    g.B = wr;
    g.ldb = 9 * C;
    g.transb = 1;
    g.C = out->ptr;
    g.ldc = K;
    g.bias = fptr(b);
    g.act = act;
    g.slope = slope;
    g.ab = tc ? DT_BF16 : DT_F32;
    g.c = DT_F32;
    gemm_run(o->ocl, g, tc ? "conv3x3_tc" : "conv3x3");
}

template <typename T>
__global__ void from_type_k(const T *in, long n, float *out)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < n)
        out[e] = ldf(in + e);
}

extern "C" void ops_attention_qkv(struct ops *o, cl_mem qkv, int N, int Dm,
                                  int heads, float scale, cl_mem out)
{
    if (pending() || !need(qkv, "ops_attention_qkv qkv") || !need(out, "out"))
        return;
    if (N <= 0 || heads <= 0 || Dm % heads || Dm / heads > OPS_MAX_HEAD_DIM) {
        fail("ops_attention_qkv: %d tokens, %d channels, %d heads", N, Dm, heads);
        return;
    }
    const int d = Dm / heads;
    const long nin = (long)N * 3 * Dm, nout = (long)N * Dm;
    cudaStream_t st = stream_of(o->ocl);
    if (o->precision == OPS_BF16 && (d == 64 || d == 128) && Dm % 64 == 0) {
        const size_t bytes = (size_t)(nin + nout) * 2 + 256;
        if (bytes > o->scratch16_bytes) {
            ocl_release(&o->scratch16);
            o->scratch16 = ocl_alloc(o->ocl, bytes, "attention operands");
            o->scratch16_bytes = bytes;
            if (pending())
                return;
        }
        __nv_bfloat16 *q16 = (__nv_bfloat16 *)o->scratch16->ptr;
        __nv_bfloat16 *o16 = q16 + (nin + 127) / 128 * 128;
        Prof p(o->ocl, "attention_tc");
        to_type_k<__nv_bfloat16><<<cdiv(nin, 256), 256, 0, st>>>(fptr(qkv), nin, q16);
        if (!attention_tc(st, q16, N, Dm, heads, o16, Dm, scale)) {
            fail("ops_attention_qkv: tensor-core attention refused the operands");
            return;
        }
        from_type_k<__nv_bfloat16><<<cdiv(nout, 256), 256, 0, st>>>(o16, nout, fptr(out));
        launch_ok("attention_tc");
        return;
    }
    Prof p(o->ocl, "attention");
    attention_l(st, fptr(qkv), 3L * Dm, fptr(qkv) + Dm, 3L * Dm, fptr(qkv) + 2 * Dm,
                3L * Dm, fptr(out), Dm, N, N, heads, d, scale, nullptr, DT_F32);
    launch_ok("attention");
}

extern "C" void ops_unfold(struct ops *o, cl_mem in, int C, int H, int W,
                           const struct conv_geom *g, cl_mem out)
{
    if (pending() || !need(in, "ops_unfold in") || !need(out, "ops_unfold out"))
        return;
    const int Ho = ops_conv_out(H, g->kh, g->sy, g->py, 1);
    const int Wo = ops_conv_out(W, g->kw, g->sx, g->px, 1);
    if (!count_ok((long)C * g->kh * g->kw * Ho * Wo, "unfold output"))
        return;
    const int n = Ho * Wo;
    if (n <= 0)
        return;
    Prof p(o->ocl, "unfold");
    unfold_kernel<<<dim3(cdiv(n, T256), C * g->kh * g->kw), T256, 0,
                    stream_of(o->ocl)>>>(fptr(in), C, H, W, g->kh, g->kw,
                                         g->sy, g->sx, g->py, g->px, 1, 1, Wo,
                                         0, n, fptr(out));
    launch_ok("unfold");
}

// ------------------------------------------------------- channel statistics

// Mean and 1 / sqrt(biased variance + eps) of each channel (ops.cl:453-492
// semantics: two passes over the plane, the mean first, then the sum of
// squared deviations from it). Each pass splits every channel into S
// segments summed by their own blocks (vector loads where the plane
// allows), then one warp per channel adds the S partial sums in a fixed
// order: deterministic, and the whole device reads the planes.
__global__ void __launch_bounds__(256)
chan_partial_k(const float *x, long HW, long seg, const float *mean, float *part)
{
    __shared__ float red[32];
    const int c = blockIdx.y, S = gridDim.x;
    const long b0 = (long)blockIdx.x * seg, b1 = b0 + seg < HW ? b0 + seg : HW;
    const float *p = x + (size_t)c * HW;
    const float m = mean ? mean[c] : 0.0f;
    float s0 = 0.0f, s1 = 0.0f;
    if ((((uintptr_t)(p + b0)) & 15) == 0 && ((b1 - b0) & 3) == 0) {
        const float4 *q = (const float4 *)(p + b0);
        const long n4 = (b1 - b0) / 4;
        for (long i = threadIdx.x; i < n4; i += blockDim.x) {
            const float4 v = q[i];
            if (mean) {
                const float d0 = v.x - m, d1 = v.y - m, d2 = v.z - m, d3 = v.w - m;
                s0 = fmaf(d0, d0, s0);
                s1 = fmaf(d1, d1, s1);
                s0 = fmaf(d2, d2, s0);
                s1 = fmaf(d3, d3, s1);
            }
            else {
                s0 += v.x + v.z;
                s1 += v.y + v.w;
            }
        }
    }
    else
        for (long i = b0 + threadIdx.x; i < b1; i += blockDim.x) {
            const float v = p[i];
            if (mean)
                s0 = fmaf(v - m, v - m, s0);
            else
                s0 += v;
        }
    const float t = block_sum(s0 + s1, red);
    if (threadIdx.x == 0)
        part[(size_t)c * S + blockIdx.x] = t;
}

__global__ void chan_final_k(const float *part, int S, long HW, float eps, float *mean,
                             float *rstd)
{
    const int c = blockIdx.x;
    float s = 0.0f;
    for (int i = threadIdx.x; i < S; i += 32)
        s += part[(size_t)c * S + i];
    s = warp_sum(s);
    if (threadIdx.x == 0) {
        if (rstd)
            rstd[c] = rsqrtf(s / HW + eps);
        else
            mean[c] = s / HW;
    }
}

extern "C" void ops_chan_stats(struct ops *o, cl_mem x, int C, int HW, float eps,
                               cl_mem mean, cl_mem rstd)
{
    if (pending() || !need(x, "ops_chan_stats x") || !need(mean, "mean") ||
        !need(rstd, "rstd") || C <= 0)
        return;
    // Segments: about four blocks per SM over all channels, at least 2048
    // elements each.
    long seg = ((long)HW * C + 4L * 148 - 1) / (4L * 148);
    seg = seg < 2048 ? 2048 : seg;
    seg = (seg + 3) / 4 * 4;
    const int S = (int)((HW + seg - 1) / seg);
    const size_t bytes = (size_t)C * S * sizeof(float);
    if (bytes > o->scratch_bytes) {
        ocl_release(&o->scratch);
        o->scratch = ocl_alloc(o->ocl, bytes, "channel statistics");
        o->scratch_bytes = bytes;
        if (pending())
            return;
    }
    cudaStream_t st = stream_of(o->ocl);
    float *part = fptr(o->scratch);
    Prof p(o->ocl, "chan_stats");
    chan_partial_k<<<dim3(S, C), 256, 0, st>>>(fptr(x), HW, seg, nullptr, part);
    chan_final_k<<<C, 32, 0, st>>>(part, S, HW, eps, fptr(mean), nullptr);
    chan_partial_k<<<dim3(S, C), 256, 0, st>>>(fptr(x), HW, seg, fptr(mean), part);
    chan_final_k<<<C, 32, 0, st>>>(part, S, HW, eps, nullptr, fptr(rstd));
    launch_ok("chan_stats");
}

__global__ void chan_affine_kernel(const float *X, float *Y, int HW, int total,
                                   const float *mean, const float *rstd,
                                   const float *g, const float *b, int act,
                                   float slope)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total)
        return;
    const int c = i / HW;
    float v = X[i];
    if (mean)
        v = (v - mean[c]) * rstd[c];
    if (g)
        v *= g[c];
    if (b)
        v += b[c];
    Y[i] = apply_act(v, act, slope);
}

extern "C" void ops_chan_affine(struct ops *o, cl_mem X, cl_mem Y, int C,
                                int HW, cl_mem mean, cl_mem rstd, cl_mem g,
                                cl_mem b, int act, float slope)
{
    const long n = (long)C * HW;
    if (pending() || !need(X, "ops_chan_affine X") || !need(Y, "Y") ||
        !count_ok(n, "chan_affine") || n == 0)
        return;
    if (mean && !rstd) {
        fail("ops_chan_affine: mean without rstd");
        return;
    }
    Prof p(o->ocl, "chan_affine");
    chan_affine_kernel<<<cdiv(n, T256), T256, 0, stream_of(o->ocl)>>>(
        fptr(X), fptr(Y), HW, (int)n, fptr(mean), fptr(rstd), fptr(g), fptr(b),
        act, slope);
    launch_ok("chan_affine");
}

__global__ void prelu_kernel(const float *X, float *Y, int HW, int total,
                             const float *alpha)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total)
        return;
    const float v = X[i];
    Y[i] = v >= 0.0f ? v : alpha[i / HW] * v;
}

extern "C" void ops_prelu(struct ops *o, cl_mem X, cl_mem Y, int C, int HW,
                          cl_mem alpha)
{
    const long n = (long)C * HW;
    if (pending() || !need(X, "ops_prelu X") || !need(Y, "Y") ||
        !need(alpha, "alpha") || !count_ok(n, "prelu") || n == 0)
        return;
    Prof p(o->ocl, "prelu");
    prelu_kernel<<<cdiv(n, T256), T256, 0, stream_of(o->ocl)>>>(
        fptr(X), fptr(Y), HW, (int)n, fptr(alpha));
    launch_ok("prelu");
}

__global__ void act_kernel(const float *X, float *Y, int total, int act,
                           float slope)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < total)
        Y[i] = apply_act(X[i], act, slope);
}

extern "C" void ops_act(struct ops *o, cl_mem X, cl_mem Y, long n, int act,
                        float slope)
{
    if (pending() || !need(X, "ops_act X") || !need(Y, "Y") ||
        !count_ok(n, "act") || n == 0)
        return;
    Prof p(o->ocl, "act");
    act_kernel<<<cdiv(n, T256), T256, 0, stream_of(o->ocl)>>>(
        fptr(X), fptr(Y), (int)n, act, slope);
    launch_ok("act");
}

// ------------------------------------------------------ LayerNorm, softmax

// Row LayerNorm (ops.cl:547-578 semantics: two passes, rsqrt(var + eps),
// optional affine, activation); Y may alias X. One block per row.
template <typename TO>
__global__ void layernorm_kernel(const float *X, TO *Y, const float *g,
                                 const float *bt, int C, float eps, int act,
                                 float slope)
{
    __shared__ float red[32];
    const size_t row = blockIdx.x;
    const float *x = X + row * C;
    TO *y = Y + row * C;
    float s = 0.0f;

    for (int c = threadIdx.x; c < C; c += blockDim.x)
        s += x[c];
    const float mean = block_sum(s, red) / C;
    s = 0.0f;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const float d = x[c] - mean;
        s = fmaf(d, d, s);
    }
    const float r = rsqrtf(block_sum(s, red) / C + eps);
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        float v = (x[c] - mean) * r;
        if (g)
            v = v * g[c] + bt[c];
        stf(y + c, apply_act(v, act, slope));
    }
}

// The same for rows of C = 128 nv floats (nv <= 16): one warp per row,
// held in registers (lane l takes float4 l, l + 32, ...), both passes
// from registers with warp reductions, 8 rows per block. Y may alias X.
__device__ __forceinline__ void store4(float *y, float4 v) { *(float4 *)y = v; }

__device__ __forceinline__ void store4(__nv_bfloat16 *y, float4 v)
{
    const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *(const uint32_t *)&a;
    u.y = *(const uint32_t *)&b;
    *(uint2 *)y = u;
}

// NVMAX: the row's float4 per lane, a compile-time bound, so that a row
// of 1024 channels holds 32 registers of values and not 64 (at 93
// registers a thread only two 256-thread blocks fit an SM, and the 3202
// rows of the ViT took two waves).
template <typename TO, int NVMAX>
__global__ void __launch_bounds__(256)
layernorm_warp_k(const float *X, TO *Y, const float *g, const float *bt, long rows, int nv,
                 float eps, int act, float slope)
{
    const int lane = threadIdx.x % 32;
    const long row = (long)blockIdx.x * 8 + threadIdx.x / 32;
    if (row >= rows)
        return;
    const int C = 128 * nv;
    const float4 *x = (const float4 *)(X + row * C);
    float4 v[NVMAX];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < NVMAX; i++)
        if (i < nv) {
            v[i] = x[lane + 32 * i];
            s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / C;
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < NVMAX; i++)
        if (i < nv) {
            const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean,
                        d = v[i].w - mean;
            q = fmaf(a, a, q);
            q = fmaf(b, b, q);
            q = fmaf(c, c, q);
            q = fmaf(d, d, q);
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        q += __shfl_xor_sync(0xffffffffu, q, o);
    const float r = rsqrtf(q / C + eps);
    TO *y = Y + row * C;
#pragma unroll
    for (int i = 0; i < NVMAX; i++)
        if (i < nv) {
            const int c = 4 * (lane + 32 * i);
            float4 o = make_float4((v[i].x - mean) * r, (v[i].y - mean) * r,
                                   (v[i].z - mean) * r, (v[i].w - mean) * r);
            if (g) {
                const float4 gg = *(const float4 *)(g + c), bb = *(const float4 *)(bt + c);
                o = make_float4(o.x * gg.x + bb.x, o.y * gg.y + bb.y, o.z * gg.z + bb.z,
                                o.w * gg.w + bb.w);
            }
            o = make_float4(apply_act(o.x, act, slope), apply_act(o.y, act, slope),
                            apply_act(o.z, act, slope), apply_act(o.w, act, slope));
            store4(y + c, o);
        }
}

namespace coreg {
void layernorm_rows(cudaStream_t st, const float *X, void *Y, DType ty,
                    const float *g, const float *b, long rows, int C, float eps,
                    int act, float slope)
{
    const int t = C >= 512 ? 256 : C >= 128 ? 128 : 32;
    if (rows <= 0)
        return;
    if (C % 128 == 0 && C <= 2048 && ((uintptr_t)X & 15) == 0 && ((uintptr_t)Y & 15) == 0 &&
        (!g || (((uintptr_t)g & 15) == 0 && ((uintptr_t)b & 15) == 0))) {
        const unsigned blocks = (unsigned)((rows + 7) / 8);
        const int nv = C / 128;
        auto run = [&](auto nvmax) {
            constexpr int NV = decltype(nvmax)::value;
            if (ty == DT_BF16)
                layernorm_warp_k<__nv_bfloat16, NV><<<blocks, 256, 0, st>>>(
                    X, (__nv_bfloat16 *)Y, g, b, rows, nv, eps, act, slope);
            else
                layernorm_warp_k<float, NV><<<blocks, 256, 0, st>>>(X, (float *)Y, g, b, rows,
                                                                    nv, eps, act, slope);
        };
        if (nv <= 2)
            run(std::integral_constant<int, 2>());
        else if (nv <= 4)
            run(std::integral_constant<int, 4>());
        else if (nv <= 8)
            run(std::integral_constant<int, 8>());
        else
            run(std::integral_constant<int, 16>());
        return;
    }
    if (ty == DT_BF16)
        layernorm_kernel<__nv_bfloat16><<<(unsigned)rows, t, 0, st>>>(
            X, (__nv_bfloat16 *)Y, g, b, C, eps, act, slope);
    else
        layernorm_kernel<float><<<(unsigned)rows, t, 0, st>>>(
            X, (float *)Y, g, b, C, eps, act, slope);
}
}  // namespace coreg

extern "C" void ops_layernorm(struct ops *o, long rows, int C, cl_mem X,
                              cl_mem Y, cl_mem g, cl_mem b, float eps, int act,
                              float slope)
{
    if (pending() || !need(X, "ops_layernorm X") || !need(Y, "Y"))
        return;
    if (g && !b) {
        fail("ops_layernorm: gamma without beta");
        return;
    }
    Prof p(o->ocl, "layernorm");
    layernorm_rows(stream_of(o->ocl), fptr(X), fptr(Y), DT_F32, fptr(g),
                   fptr(b), rows, C, eps, act, slope);
    launch_ok("layernorm");
}

// In-place softmax(scale * x) over rows (ops.cl:583-602 semantics).
__global__ void softmax_kernel(float *S, int L, float scale)
{
    __shared__ float red[32];
    float *s = S + (size_t)blockIdx.x * L;
    float m = -INFINITY, sum = 0.0f;

    for (int j = threadIdx.x; j < L; j += blockDim.x)
        m = fmaxf(m, s[j] * scale);
    m = block_max(m, red);
    for (int j = threadIdx.x; j < L; j += blockDim.x) {
        const float v = expf(s[j] * scale - m);
        s[j] = v;
        sum += v;
    }
    const float inv = 1.0f / block_sum(sum, red);
    for (int j = threadIdx.x; j < L; j += blockDim.x)
        s[j] *= inv;
}

extern "C" void ops_softmax_rows(struct ops *o, cl_mem S, long rows, int L,
                                 float scale)
{
    if (pending() || !need(S, "ops_softmax_rows S") || rows <= 0)
        return;
    const int t = L >= 512 ? 256 : L >= 128 ? 128 : 32;
    Prof p(o->ocl, "softmax_rows");
    softmax_kernel<<<(unsigned)rows, t, 0, stream_of(o->ocl)>>>(fptr(S), L,
                                                                scale);
    launch_ok("softmax_rows");
}

// --------------------------------------------------------------- attention

// O = softmax(scale Q K^T) V per head, never storing the scores
// (ops.cl:604-687 semantics: key mask, a query without keys gets zeros).
// Block: 4 warps x 4 queries each (16 queries) of one head; keys in
// chunks of 32 through shared memory, lane j scoring key j of the chunk,
// each lane owning output columns lane, lane + 32, ...
#define ATT_Q 16
#define ATT_KC 32
template <typename T>
__global__ void __launch_bounds__(128)
attention_kernel(const T *Q, long ldq, const T *K, long ldk, const T *V,
                 long ldv, T *O, long ldo, int Nq, int Nk, int d, float scale,
                 const unsigned char *kmask)
{
    __shared__ float qs[ATT_Q][OPS_MAX_HEAD_DIM + 1];
    __shared__ float ks[ATT_KC][OPS_MAX_HEAD_DIM + 1];
    __shared__ float vs[ATT_KC][OPS_MAX_HEAD_DIM];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int h = blockIdx.y, q0 = blockIdx.x * ATT_Q;
    const int nd = (d + 31) / 32;
    float o[4][4], m[4], l[4];

    Q += (size_t)h * d;
    K += (size_t)h * d;
    V += (size_t)h * d;
    for (int e = threadIdx.x; e < ATT_Q * d; e += blockDim.x) {
        const int r = e / d, c = e % d, q = q0 + r;
        qs[r][c] = q < Nq ? ldf(Q + (size_t)q * ldq + c) * scale : 0.0f;
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        m[i] = -INFINITY;
        l[i] = 0.0f;
#pragma unroll
        for (int t = 0; t < 4; t++)
            o[i][t] = 0.0f;
    }
    for (int k0 = 0; k0 < Nk; k0 += ATT_KC) {
        __syncthreads();
        for (int e = threadIdx.x; e < ATT_KC * d; e += blockDim.x) {
            const int r = e / d, c = e % d, k = k0 + r;
            ks[r][c] = k < Nk ? ldf(K + (size_t)k * ldk + c) : 0.0f;
            vs[r][c] = k < Nk ? ldf(V + (size_t)k * ldv + c) : 0.0f;
        }
        __syncthreads();
        const int key = k0 + lane;
        const bool ok = key < Nk && (!kmask || kmask[key]);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int r = wid * 4 + i;
            float s = -INFINITY;
            if (ok) {
                s = 0.0f;
                for (int c = 0; c < d; c++)
                    s = fmaf(qs[r][c], ks[lane][c], s);
            }
            const float mn = fmaxf(m[i], warp_max(s));
            if (mn == -INFINITY)
                continue;
            const float corr = expf(m[i] - mn);
            const float e = ok ? expf(s - mn) : 0.0f;
            l[i] = l[i] * corr + warp_sum(e);
            m[i] = mn;
#pragma unroll
            for (int t = 0; t < 4; t++)
                o[i][t] *= corr;
            for (int j = 0; j < ATT_KC; j++) {
                const float pj = __shfl_sync(0xffffffffu, e, j);
#pragma unroll
                for (int t = 0; t < 4; t++)
                    if (t < nd && lane + 32 * t < d)
                        o[i][t] = fmaf(pj, vs[j][lane + 32 * t], o[i][t]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int q = q0 + wid * 4 + i;
        if (q >= Nq)
            continue;
#pragma unroll
        for (int t = 0; t < 4; t++) {
            const int c = lane + 32 * t;
            if (c < d)
                stf(O + (size_t)q * ldo + (size_t)h * d + c,
                    l[i] > 0.0f ? o[i][t] / l[i] : 0.0f);
        }
    }
}

namespace coreg {
void attention_l(cudaStream_t st, const void *Q, long ldq, const void *K,
                 long ldk, const void *V, long ldv, void *O, long ldo, int Nq,
                 int Nk, int nh, int d, float scale, const unsigned char *kmask,
                 DType t)
{
    dim3 grid(cdiv(Nq, ATT_Q), nh);
    if (t == DT_BF16)
        attention_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(
            (const __nv_bfloat16 *)Q, ldq, (const __nv_bfloat16 *)K, ldk,
            (const __nv_bfloat16 *)V, ldv, (__nv_bfloat16 *)O, ldo, Nq, Nk, d,
            scale, kmask);
    else
        attention_kernel<float><<<grid, 128, 0, st>>>(
            (const float *)Q, ldq, (const float *)K, ldk, (const float *)V, ldv,
            (float *)O, ldo, Nq, Nk, d, scale, kmask);
}
}  // namespace coreg

// OPS_BF16 contexts run unmasked self-sized attention (Nq = Nk) on the
// tcgen05 attention kernels (head size 64 or 128): the float32 Q, K, V are
// packed into one token-major bfloat16 qkv buffer, each head's d columns
// zero-padded to 64 (d <= 64) or 128 (zeros add nothing to the scores and
// give zero output columns), and the bfloat16 output is unpacked into O.
// Both buffers come from o->scratch16.
__global__ void attn_pack_k(const float *Q, long ldq, const float *K, long ldk, const float *V,
                            long ldv, int N, int nh, int d, int dp, __nv_bfloat16 *qkv)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const long dm = (long)nh * dp;
    if (e >= (long)N * 3 * dm)
        return;
    const long r = e / (3 * dm), j = e % (3 * dm);
    const int which = (int)(j / dm), h = (int)(j % dm / dp), c = (int)(j % dp);
    const float *src = which == 0 ? Q + r * ldq : which == 1 ? K + r * ldk : V + r * ldv;
    qkv[e] = __float2bfloat16_rn(c < d ? src[h * d + c] : 0.0f);
}

__global__ void attn_unpack_k(const __nv_bfloat16 *o16, int N, int nh, int d, int dp, float *O,
                              long ldo)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= (long)N * nh * d)
        return;
    const long r = e / ((long)nh * d);
    const int h = (int)(e % ((long)nh * d) / d), c = (int)(e % d);
    O[r * ldo + h * d + c] = __bfloat162float(o16[r * (long)nh * dp + h * dp + c]);
}

static bool attention_bf16_tc(struct ops *o, struct opnd Q, struct opnd K, struct opnd V,
                              struct opnd O, int N, int nh, int d, float scale)
{
    const int dp = d <= 64 ? 64 : 128;
    const long dm = (long)nh * dp;
    const size_t qb = ((size_t)N * 3 * dm * 2 + 255) / 256 * 256;
    const size_t bytes = qb + (size_t)N * dm * 2;
    if (bytes > o->scratch16_bytes) {
        ocl_release(&o->scratch16);
        o->scratch16 = ocl_alloc(o->ocl, bytes, "attention operands");
        o->scratch16_bytes = bytes;
        if (pending())
            return false;
    }
    __nv_bfloat16 *qkv = (__nv_bfloat16 *)o->scratch16->ptr;
    __nv_bfloat16 *o16 = (__nv_bfloat16 *)((char *)o->scratch16->ptr + qb);
    cudaStream_t st = stream_of(o->ocl);
    attn_pack_k<<<cdiv((long)N * 3 * dm, 256), 256, 0, st>>>(
        fptr(Q.buf, Q.off), Q.ld, fptr(K.buf, K.off), K.ld, fptr(V.buf, V.off), V.ld, N, nh, d,
        dp, qkv);
    if (!attention_tc(st, qkv, N, (int)dm, nh, o16, dm, scale, 1))
        return false;
    attn_unpack_k<<<cdiv((long)N * nh * d, 256), 256, 0, st>>>(o16, N, nh, d, dp,
                                                              fptr(O.buf, O.off), O.ld);
    return launch_ok("attention");
}

extern "C" void ops_attention(struct ops *o, struct opnd Q, struct opnd K,
                              struct opnd V, struct opnd O, int Nq, int Nk,
                              int nh, int d, float scale, cl_mem kmask)
{
    if (pending() || !need(Q.buf, "ops_attention Q") || !need(K.buf, "K") ||
        !need(V.buf, "V") || !need(O.buf, "O"))
        return;
    if (d < 1 || d > OPS_MAX_HEAD_DIM) {
        fail("CUDA: attention head dimension %d not in 1..%d", d,
             OPS_MAX_HEAD_DIM);
        return;
    }
    if (Nq <= 0 || nh <= 0)
        return;
    Prof p(o->ocl, "attention");
    if (o->precision == OPS_BF16 && Nq == Nk && !kmask &&
        attention_bf16_tc(o, Q, K, V, O, Nq, nh, d, scale))
        return;
    if (pending())
        return;
    attention_l(stream_of(o->ocl), fptr(Q.buf, Q.off), Q.ld, fptr(K.buf, K.off),
                K.ld, fptr(V.buf, V.off), V.ld, fptr(O.buf, O.off), O.ld, Nq, Nk,
                nh, d, scale, kmask ? (const unsigned char *)kmask->ptr : nullptr,
                DT_F32);
    launch_ok("attention");
}

// ------------------------------------------------------------------- RoPE

// Rotary encoding in place (ops.cl:695-716 semantics).
__global__ void rope_kernel(float *X, long ld, int nh, int d, int npos,
                            const float2 *cs, int interleaved, int total)
{
    const int gid = blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= total)
        return;
    const int nf = d / 2;
    const int f = gid % nf, h = (gid / nf) % nh, r = gid / (nf * nh);
    float *x = X + (size_t)r * ld + (size_t)h * d;
    const float2 rot = cs[(r % npos) * nf + f];
    const int i0 = interleaved ? 2 * f : f;
    const int i1 = interleaved ? 2 * f + 1 : f + nf;
    const float a = x[i0], b = x[i1];
    x[i0] = a * rot.x - b * rot.y;
    x[i1] = a * rot.y + b * rot.x;
}

extern "C" void ops_rope(struct ops *o, cl_mem X, long off, int ld, long rows,
                         int nh, int d, int npos, cl_mem cs, int interleaved)
{
    const long n = rows * nh * (d / 2);
    if (pending() || !need(X, "ops_rope X") || !need(cs, "cs") ||
        !count_ok(n, "rope") || n == 0)
        return;
    if (npos < 1) {
        fail("ops_rope: npos %d", npos);
        return;
    }
    Prof p(o->ocl, "rope");
    rope_kernel<<<cdiv(n, T256), T256, 0, stream_of(o->ocl)>>>(
        fptr(X, off), ld, nh, d, npos, (const float2 *)cs->ptr, interleaved,
        (int)n);
    launch_ok("rope");
}

// ------------------------------------------------------ resampling, pooling

// Bilinear resampling into channels coff.. of out (ops.cl:723-754
// semantics: align_corners, else source step sy/sx clamped at 0).
__global__ void resize_kernel(const float *in, int h, int w, float *out, int H,
                              int W, int coff, int align, float sy, float sx)
{
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int y = blockIdx.y, c = blockIdx.z;
    if (x >= W)
        return;
    float ux, uy;
    if (align) {
        ux = W > 1 ? x * (float)(w - 1) / (W - 1) : 0.0f;
        uy = H > 1 ? y * (float)(h - 1) / (H - 1) : 0.0f;
    }
    else {
        ux = fmaxf((x + 0.5f) * sx - 0.5f, 0.0f);
        uy = fmaxf((y + 0.5f) * sy - 0.5f, 0.0f);
    }
    const int x0 = (int)ux, y0 = (int)uy;
    const int x1 = min(x0 + 1, w - 1), y1 = min(y0 + 1, h - 1);
    const float fx = ux - x0, fy = uy - y0;
    const float *p = in + (size_t)c * h * w;
    out[((size_t)(c + coff) * H + y) * W + x] =
        (1.0f - fy) * ((1.0f - fx) * p[y0 * w + x0] + fx * p[y0 * w + x1]) +
        fy * ((1.0f - fx) * p[y1 * w + x0] + fx * p[y1 * w + x1]);
}

namespace coreg {
void resize_planes(cudaStream_t st, const float *in, int C, int h, int w,
                   float *out, int H, int W, int coff, int align, float scale)
{
    const float sy = scale > 0 ? 1.0f / scale : (float)h / H;
    const float sx = scale > 0 ? 1.0f / scale : (float)w / W;
    if (C <= 0 || H <= 0 || W <= 0)
        return;
    resize_kernel<<<dim3(cdiv(W, 128), H, C), 128, 0, st>>>(in, h, w, out, H, W,
                                                           coff, align, sy, sx);
}
}  // namespace coreg

extern "C" void ops_resize(struct ops *o, cl_mem in, int C, int h, int w,
                           cl_mem out, int H, int W, int coff,
                           int align_corners, float scale)
{
    if (pending() || !need(in, "ops_resize in") || !need(out, "out"))
        return;
    Prof p(o->ocl, "resize_bilinear");
    resize_planes(stream_of(o->ocl), fptr(in), C, h, w, fptr(out), H, W, coff,
                  align_corners, scale);
    launch_ok("resize_bilinear");
}

// Bilinear sampling at normalized points, zero padding (ops.cl:759-793).
__global__ void grid_sample_kernel(const float *in, int C, int H, int W,
                                   const float2 *grid, int n, int align,
                                   float *out)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int c = blockIdx.y;
    if (i >= n)
        return;
    const float *p = in + (size_t)c * H * W;
    const float2 g = grid[i];
    float ix, iy, v = 0.0f;
    if (align) {
        ix = (g.x + 1.0f) * 0.5f * (W - 1);
        iy = (g.y + 1.0f) * 0.5f * (H - 1);
    }
    else {
        ix = ((g.x + 1.0f) * W - 1.0f) * 0.5f;
        iy = ((g.y + 1.0f) * H - 1.0f) * 0.5f;
    }
    if (isfinite(ix) && isfinite(iy)) {
        const int x0 = (int)floorf(ix), y0 = (int)floorf(iy);
        const float fx = ix - x0, fy = iy - y0;
        auto at = [&](int yy, int xx) {
            return xx >= 0 && xx < W && yy >= 0 && yy < H ? p[yy * W + xx]
                                                          : 0.0f;
        };
        v = (1.0f - fy) * ((1.0f - fx) * at(y0, x0) + fx * at(y0, x0 + 1)) +
            fy * ((1.0f - fx) * at(y0 + 1, x0) + fx * at(y0 + 1, x0 + 1));
    }
    out[(size_t)c * n + i] = v;
}

extern "C" void ops_grid_sample(struct ops *o, cl_mem in, int C, int H, int W,
                                cl_mem grid, int n, int align_corners,
                                cl_mem out)
{
    if (pending() || !need(in, "ops_grid_sample in") || !need(grid, "grid") ||
        !need(out, "out") || n <= 0 || C <= 0)
        return;
    Prof p(o->ocl, "grid_sample");
    grid_sample_kernel<<<dim3(cdiv(n, T256), C), T256, 0, stream_of(o->ocl)>>>(
        fptr(in), C, H, W, (const float2 *)grid->ptr, n, align_corners,
        fptr(out));
    launch_ok("grid_sample");
}

__global__ void avgpool2_kernel(const float *in, int H, int W, float *out)
{
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int y = blockIdx.y, c = blockIdx.z;
    const int w = W / 2;
    if (x >= w)
        return;
    const float *p = in + ((size_t)c * H + 2 * y) * W + 2 * x;
    out[((size_t)c * (H / 2) + y) * w + x] =
        0.25f * (p[0] + p[1] + p[W] + p[W + 1]);
}

extern "C" void ops_avgpool2(struct ops *o, cl_mem in, int C, int H, int W,
                             cl_mem out)
{
    if (pending() || !need(in, "ops_avgpool2 in") || !need(out, "out") ||
        H < 2 || W < 2 || C <= 0)
        return;
    Prof p(o->ocl, "avgpool2");
    avgpool2_kernel<<<dim3(cdiv(W / 2, 128), H / 2, C), 128, 0,
                      stream_of(o->ocl)>>>(fptr(in), H, W, fptr(out));
    launch_ok("avgpool2");
}

// k x k pooling (ops.cl:835-860 semantics: max ignores the padding,
// average counts it).
__global__ void pool2d_kernel(const float *in, int H, int W, int Ho, int Wo,
                              int k, int s, int pad, int max, float *out)
{
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    const int y = blockIdx.y, c = blockIdx.z;
    if (x >= Wo)
        return;
    const float *p = in + (size_t)c * H * W;
    float acc = max ? -INFINITY : 0.0f;
    for (int i = 0; i < k; i++) {
        const int iy = y * s - pad + i;
        if (iy < 0 || iy >= H)
            continue;
        for (int j = 0; j < k; j++) {
            const int ix = x * s - pad + j;
            if (ix < 0 || ix >= W)
                continue;
            const float v = p[iy * W + ix];
            acc = max ? fmaxf(acc, v) : acc + v;
        }
    }
    out[((size_t)c * Ho + y) * Wo + x] = max ? acc : acc / (k * k);
}

extern "C" void ops_pool2d(struct ops *o, cl_mem in, int C, int H, int W, int k,
                           int s, int p, int max, cl_mem out)
{
    if (pending() || !need(in, "ops_pool2d in") || !need(out, "out"))
        return;
    const int Ho = ops_conv_out(H, k, s, p, 1), Wo = ops_conv_out(W, k, s, p, 1);
    if (Ho <= 0 || Wo <= 0 || C <= 0)
        return;
    Prof pr(o->ocl, max ? "maxpool" : "avgpool");
    pool2d_kernel<<<dim3(cdiv(Wo, 128), Ho, C), 128, 0, stream_of(o->ocl)>>>(
        fptr(in), H, W, Ho, Wo, k, s, p, max, fptr(out));
    launch_ok("pool2d");
}

// ----------------------------------------------------- transpose, axpby

__global__ void transpose_kernel(const float *in, float *out, int R, int C)
{
    __shared__ float t[32][33];
    const size_t base = (size_t)blockIdx.z * R * C;
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int r = r0 + i, c = c0 + threadIdx.x;
        if (r < R && c < C)
            t[i][threadIdx.x] = in[base + (size_t)r * C + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int c = c0 + i, r = r0 + threadIdx.x;
        if (r < R && c < C)
            out[base + (size_t)c * R + r] = t[threadIdx.x][i];
    }
}

namespace coreg {
void transpose_f32(cudaStream_t st, const float *in, float *out, int B, int R,
                   int C)
{
    if (B <= 0 || R <= 0 || C <= 0)
        return;
    transpose_kernel<<<dim3(cdiv(C, 32), cdiv(R, 32), B), dim3(32, 8), 0, st>>>(
        in, out, R, C);
}
}  // namespace coreg

extern "C" void ops_transpose(struct ops *o, cl_mem in, cl_mem out, int B, int R,
                              int C)
{
    if (pending() || !need(in, "ops_transpose in") || !need(out, "out") ||
        !count_ok((long)B * R * C, "transpose"))
        return;
    Prof p(o->ocl, "transpose");
    transpose_f32(stream_of(o->ocl), fptr(in), fptr(out), B, R, C);
    launch_ok("transpose");
}

__global__ void axpby_kernel(float *out, const float *a, float alpha,
                             const float *b, float beta, int n, int bmod)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n)
        return;
    out[i] = alpha * a[i] + (b ? beta * b[i % bmod] : 0.0f);
}

extern "C" void ops_axpby(struct ops *o, cl_mem out, cl_mem a, float alpha,
                          cl_mem b, float beta, long n, long bmod)
{
    if (pending() || !need(out, "ops_axpby out") || !need(a, "a") ||
        !count_ok(n, "axpby") || n == 0)
        return;
    Prof p(o->ocl, "axpby");
    axpby_kernel<<<cdiv(n, T256), T256, 0, stream_of(o->ocl)>>>(
        fptr(out), fptr(a), alpha, fptr(b), beta, (int)n,
        bmod > 0 ? (int)bmod : 1);
    launch_ok("axpby");
}

// ------------------------------------------------------------ BN folding

// Host BatchNorm folding in double (ops.c:612-626 semantics).
extern "C" void ops_fold_bn(float *w, float *b, int K, long per,
                            const float *gamma, const float *beta,
                            const float *mean, const float *var, float eps)
{
    for (int k = 0; k < K; k++) {
        const double s = gamma[k] / sqrt((double)var[k] + eps);
        for (long i = 0; i < per; i++)
            w[(size_t)k * per + i] = (float)(w[(size_t)k * per + i] * s);
        b[k] = (float)((b[k] - mean[k]) * s + beta[k]);
    }
}
