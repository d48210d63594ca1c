// SPDX-License-Identifier: Unlicense
//
// The first convolution of VGG19-BN (3 x 3, stride 1, padding 1, 3 -> 64
// channels, bias and ReLU: roma.c:742-768 over ops.cl's conv2d) on the
// tensor cores without an im2col buffer. A product of K = 27 (padded to 32)
// per output pixel writes 128 bytes and reads 6: the layer is bound by its
// output, and the explicit im2col plus a K = 32 GEMM spent most of their
// time on the im2col buffer and on per-tile epilogue latency.
//
// Persistent, 128-pixel tiles (consecutive pixels of the row-major map).
// Warps:
//   0..3   producers: thread t gathers the 3 x 3 x 3 neighbourhood of pixel
//          t of the tile (zeros outside the map) into row t of a 128 x 64
//          bfloat16 A buffer, 128-byte swizzled (columns j = tap 3 + c,
//          27..31 zero; the MMA reads 32 columns), in a ring of RC_NA;
//   4      tensor memory (two 64-column accumulators) and MMA issue: two
//          tcgen05.mma (K = 16 each) per tile against the weights, which
//          stay in shared memory for the kernel;
//   5..8   epilogue: warp w reads TMEM lanes 32 (w % 4) .. (rows = pixels),
//          frees the accumulator, adds the bias, applies ReLU and writes
//          the pixel's 64 channels.
// Every mbarrier wait is bounded; a wait that runs out records an error
// code (coreg_tc_status) and the warp leaves its loop.

#include "tc_common.cuh"

namespace coreg {
namespace tc {

namespace {

constexpr int RC_T = 288, RC_NA = 4, RC_K = 64;

struct RcSmem {
    alignas(1024) __nv_bfloat16 a[RC_NA][128 * 64];
    alignas(1024) __nv_bfloat16 b[RC_K * 64];
    float bias[RC_K];
    uint64_t afull[RC_NA], aempty[RC_NA], accfull[2], accempty[2];
    uint32_t tmem;
};

__device__ __forceinline__ uint32_t pack2(__nv_bfloat16 lo, __nv_bfloat16 hi)
{
    return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
}

__device__ __forceinline__ void store64(float *dst, const float v[RC_K])
{
#pragma unroll
    for (int j = 0; j < RC_K; j += 4)
        *reinterpret_cast<float4 *>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
}

__device__ __forceinline__ void store64(__nv_bfloat16 *dst, const float v[RC_K])
{
#pragma unroll
    for (int j = 0; j < RC_K; j += 8) {
        uint4 u;
        u.x = pack2(__float2bfloat16_rn(v[j]), __float2bfloat16_rn(v[j + 1]));
        u.y = pack2(__float2bfloat16_rn(v[j + 2]), __float2bfloat16_rn(v[j + 3]));
        u.z = pack2(__float2bfloat16_rn(v[j + 4]), __float2bfloat16_rn(v[j + 5]));
        u.w = pack2(__float2bfloat16_rn(v[j + 6]), __float2bfloat16_rn(v[j + 7]));
        *reinterpret_cast<uint4 *>(dst + j) = u;
    }
}

// in: H x W x 3 bfloat16; wk: 64 x 32 bfloat16 (column j = tap 3 + c, zeros
// from 27); out: H x W x 64.
template <typename TO>
__global__ void __launch_bounds__(RC_T, 1)
conv_rgb_kernel(const __nv_bfloat16 *in, int H, int W, const __nv_bfloat16 *wk,
                const float *bias, TO *out, long ntiles)
{
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    RcSmem &s = *reinterpret_cast<RcSmem *>(smem_raw + ((1024u - (su32(smem_raw) & 1023u)) & 1023u));
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const long npix = (long)H * W;
    const int my_tiles =
        ntiles > (long)blockIdx.x ? (int)((ntiles - blockIdx.x + gridDim.x - 1) / gridDim.x) : 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < RC_NA; i++) {
            mbar_init(&s.afull[i], 4);
            mbar_init(&s.aempty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&s.accfull[i], 1);
            mbar_init(&s.accempty[i], 4);
        }
        mbar_fence_init();
    }
    // The weights: row n (output channel), 16-byte chunk c < 4 of its 32
    // columns at chunk position c ^ (n % 8) (128-byte swizzle).
    for (int e = threadIdx.x; e < RC_K * 4; e += RC_T) {
        const int n = e / 4, c = e % 4;
        reinterpret_cast<uint4 *>(s.b + n * 64)[c ^ (n & 7)] =
            reinterpret_cast<const uint4 *>(wk + n * 32)[c];
    }
    for (int e = threadIdx.x; e < RC_K; e += RC_T)
        s.bias[e] = bias[e];
    fence_async_smem();
    if (warp == 4)
        tmem_alloc(&s.tmem, 2 * RC_K);
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = s.tmem;

    if (warp < 4) {
        // ------------------------------------------------------ producers
        const int t = threadIdx.x;
        for (int i = 0; i < my_tiles; i++) {
            const int slot = i % RC_NA, use = i / RC_NA;
            if (!__all_sync(0xffffffffu, use == 0 || mbar_wait(&s.aempty[slot], (use - 1) & 1, 41)))
                break;
            const long pix = ((long)blockIdx.x + (long)i * gridDim.x) * 128 + t;
            __nv_bfloat16 v[32];
#pragma unroll
            for (int j = 0; j < 32; j++)
                v[j] = __float2bfloat16_rn(0.0f);
            if (pix < npix) {
                const int px = (int)(pix % W), py = (int)(pix / W);
#pragma unroll
                for (int tap = 0; tap < 9; tap++) {
                    const int xx = px + tap % 3 - 1, yy = py + tap / 3 - 1;
                    if (xx >= 0 && xx < W && yy >= 0 && yy < H) {
                        const __nv_bfloat16 *p = in + ((long)yy * W + xx) * 3;
                        v[3 * tap] = p[0];
                        v[3 * tap + 1] = p[1];
                        v[3 * tap + 2] = p[2];
                    }
                }
            }
            uint4 *row = reinterpret_cast<uint4 *>(s.a[slot] + t * 64);
#pragma unroll
            for (int c = 0; c < 4; c++)
                row[c ^ (t & 7)] = make_uint4(pack2(v[8 * c], v[8 * c + 1]), pack2(v[8 * c + 2], v[8 * c + 3]),
                                              pack2(v[8 * c + 4], v[8 * c + 5]),
                                              pack2(v[8 * c + 6], v[8 * c + 7]));
            fence_async_smem();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&s.afull[slot]);
        }
    }
    else if (warp == 4) {
        // ------------------------------------------------------------ MMA
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(128, RC_K);
            const uint64_t db = sw128_desc(su32(s.b));
            for (int lt = 0; lt < my_tiles; lt++) {
                const int buf = lt & 1, use = lt >> 1, slot = lt % RC_NA;
                if (use > 0 && !mbar_wait(&s.accempty[buf], (use - 1) & 1, 42))
                    break;
                if (!mbar_wait(&s.afull[slot], (lt / RC_NA) & 1, 43))
                    break;
                fence_after();
                const uint64_t da = sw128_desc(su32(s.a[slot]));
                const uint32_t acc = tmem + (uint32_t)(buf * RC_K);
                mma_bf16(acc, da, db, idesc, 0u);
                mma_bf16(acc, da + 2, db + 2, idesc, 1u);
                mma_commit(&s.aempty[slot]);
                mma_commit(&s.accfull[buf]);
            }
        }
    }
    else {
        // ------------------------------------------------------- epilogue
        const int q = warp % 4, r = 32 * q + lane;
        for (int lt = 0; lt < my_tiles; lt++) {
            const int buf = lt & 1, use = lt >> 1;
            if (!__all_sync(0xffffffffu, mbar_wait_backoff(&s.accfull[buf], use & 1, 44)))
                break;
            fence_after();
            float v[RC_K];
            const uint32_t acc = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * RC_K);
            tmem_ld32(acc, v);
            tmem_ld32(acc + 32, v + 32);
            fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&s.accempty[buf]);
            const long pix = ((long)blockIdx.x + (long)lt * gridDim.x) * 128 + r;
            if (pix < npix) {
#pragma unroll
                for (int j = 0; j < RC_K; j++)
                    v[j] = fmaxf(v[j] + s.bias[j], 0.0f);
                store64(out + pix * RC_K, v);
            }
        }
    }
    fence_before();
    __syncthreads();
    if (warp == 4) {
        fence_after();
        tmem_dealloc(tmem, 2 * RC_K);
    }
}

template <typename TO>
bool run_rgb(cudaStream_t st, const __nv_bfloat16 *in, int H, int W, const __nv_bfloat16 *wk,
             const float *bias, TO *out, int sm_count)
{
    const size_t smem = sizeof(RcSmem) + 1024;
    static unsigned done = 0;
    if (!smem_opt_in((const void *)conv_rgb_kernel<TO>, smem, &done))
        return false;
    const long ntiles = ((long)H * W + 127) / 128;
    // Two CTAs per SM (128 TMEM columns and 74 KB of shared memory each).
    const long grid = ntiles < 2L * sm_count ? ntiles : 2L * sm_count;
    conv_rgb_kernel<TO><<<(unsigned)grid, RC_T, smem, st>>>(in, H, W, wk, bias, out, ntiles);
    return true;
}

}  // namespace

}  // namespace tc

// The 3 -> 64 channel 3 x 3 convolution with bias and ReLU (wk 64 x 32,
// column j = tap 3 + c); false where the kernel does not apply.
bool conv_rgb_tc(cudaStream_t st, const __nv_bfloat16 *in, int H, int W,
                 const __nv_bfloat16 *wk, const float *bias, void *out, DType ot, int sm_count)
{
    if (((uintptr_t)wk & 15) || ((uintptr_t)out & 15) || (long)H * W <= 0)
        return false;
    if (sm_count <= 0)
        sm_count = 148;
    if (ot == DT_BF16)
        return tc::run_rgb(st, in, H, W, wk, bias, (__nv_bfloat16 *)out, sm_count);
    return tc::run_rgb(st, in, H, W, wk, bias, (float *)out, sm_count);
}

}  // namespace coreg
