// SPDX-License-Identifier: Unlicense
//
// One hidden block of RoMa's convolutional refiners as a single sm_100a
// kernel over a channels-last bfloat16 (H, W, C) map, C in {32, 64, 128}:
//
//   out = W_pw relu(dw5x5(in) + b_dw) + b_pw
//
// that is the depthwise 5 x 5 convolution with its folded batch norm and
// ReLU (roma_kernels.cl:251-290) followed by the block's 1 x 1 convolution,
// the two steps the reference runs per block (roma.c:970-985,
// roma.c:1080-1094). The depthwise result is rounded to bfloat16, as the
// unfused path stores it, straight into shared memory as the A operand of
// the tcgen05 product: it never reaches global memory, so a block reads
// its input and writes its output once.
//
// Persistent: one CTA per SM walks 16 x 8-pixel output tiles (128 GEMM
// rows); a tile's channels are k-blocks of CK = min(C, 64). Warps:
//   0..15  producers: compute the depthwise convolution of each (tile,
//          k-block) in float32 (packed FMAs, weights from shared memory,
//          the taps in the reference's order) from its input patch and
//          write the bfloat16 result, 128-byte swizzled, into a ring of NA
//          A buffers. A thread takes one tile row of one channel pair, so
//          that every weight and patch value it reads from shared memory
//          (the bound of this stage) feeds 16 and up to 5 packed FMAs; an
//          item takes 8 warps (CK 64) or 4 (CK 32), and the sixteen warps
//          work on 2 or 4 consecutive items at once;
//   16     tensor-memory allocator, weight loader (one TMA load, resident
//          for the kernel) and MMA issuer into one of two 128 x C float32
//          accumulators (tiles alternate);
//   17..20 epilogue: tensor memory + bias -> bfloat16 -> swizzled shared
//          staging -> TMA store of the tile (clipped at the map border);
//   21     patch loader: the 20 x 12-pixel x CK-channel input patch of each
//          item by TMA (zeros outside the map) into a ring of NH buffers,
//          a buffer refilled once the producer warps of its last item have
//          released it.
// Producers, loader and MMA issuer meet only at mbarriers. Every wait is
// bounded (global time, about two seconds); a wait that runs out records
// an error code (coreg_tc_status) and the waiting warp leaves its loop,
// so that the others run out of their waits in turn; the epilogue warps
// leave together (a flag written before and read after their barrier).
// Then the CTA frees its tensor memory and returns.

#include <string.h>

#include "tc_common.cuh"

namespace coreg {
namespace tc {

bool make_map_2d(CUtensorMap *map, const void *base, long rows, long cols, long ld,
                 int box_rows);
bool make_map_hwc(CUtensorMap *map, void *base, int H, int W, int C, int box_c, int box_w,
                  int box_h, int swizzle_bytes);

namespace {

constexpr int TX = 16, TY = 8;              // output tile (TX TY = 128 rows)
constexpr int PX = TX + 4, PY = TY + 4;     // input patch
constexpr int PROD_WARPS = 16;              // warps 0..15
constexpr int MMA_WARP = 16;
constexpr int EPI_WARP0 = 17;               // warps 17..20
constexpr int LOAD_WARP = 21;
constexpr int DW_THREADS = 22 * 32;

template <int C>
struct DwCfg {
    static constexpr int CK = C < 64 ? C : 64;        // channels per k-block
    static constexpr int NKB = C / CK;
    static constexpr int NP = CK / 2;                 // channel pairs per k-block
    // A producer thread computes one whole tile row (TX pixels) of one
    // channel pair, so that its weights and each patch value it loads feed
    // TX and up to five outputs: CK 64, a warp per row (lane = pair), eight
    // warps per item; CK 32, a half warp per row, four warps per item. The
    // producer warps form PG groups that work on PG consecutive items at
    // once (group g takes items g, g + PG, ...).
    static constexpr int WI = CK == 64 ? 8 : 4;      // warps per item
    static constexpr int PG = PROD_WARPS / WI;       // items in flight
    // Patch width loaded (pixels) and row pitch in 32-bit words: with CK 32
    // the two half warps read adjacent patch rows, which one extra pixel
    // per row puts 16 banks apart.
    static constexpr int PXL = CK == 32 ? PX + 1 : PX;
    static constexpr int RPW = PXL * NP;
    static constexpr int PATCH_WORDS = PY * RPW;
    // Rings: with 32 channels one A slot and two patch slots more than the
    // items in flight; the wider blocks keep three of each (C 128 fills the
    // shared memory at that).
    static constexpr int NA = C == 32 ? PG + 1 : 3;   // A ring
    static constexpr int NH = C == 32 ? PG + 2 : 3;   // patch ring
    static constexpr int NO = C <= 64 ? 2 : 1;        // output staging buffers
    static constexpr int TMEM_COLS = 2 * C;           // two accumulators
    static constexpr int OSW = CK == 64 ? 128 : 64;   // output swizzle (bytes)
};

template <int C>
struct DwSmem {
    using G = DwCfg<C>;
    alignas(1024) __nv_bfloat16 b[G::NKB][C * 64];   // weights, per k-block C x 64
    alignas(1024) __nv_bfloat16 a[G::NA][128 * 64];  // depthwise result, 128 x 64
    alignas(1024) __nv_bfloat16 o[G::NO][128 * C];   // output tile, NKB boxes
    alignas(1024) uint32_t patch[G::NH][G::PATCH_WORDS];
    float2 dw[G::NKB][25][G::NP];  // depthwise taps, channel pairs innermost
    float dwb[C], pwb[C];
    uint64_t bfull, pfull[G::NH], pempty[G::NH], afull[G::NA], aempty[G::NA], accfull[2],
        accempty[2];
    uint32_t tmem;
    int eabort;
};

struct DwParams {
    int H, W, tiles_x, ntiles;
    const float *dw_w, *dw_b, *pw_b;
};

// Float32 pairs packed in one 64-bit register pair for the sm_100a f32x2
// FMA; the accumulators and weights stay packed through the convolution,
// so that no moves split and rejoin them around each instruction.
typedef unsigned long long u64;

__device__ __forceinline__ u64 pk2(float lo, float hi)
{
    u64 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}

__device__ __forceinline__ float2 upk2(u64 v)
{
    float2 d;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(v));
    return d;
}

__device__ __forceinline__ u64 fma2p(u64 a, u64 b, u64 c)
{
    u64 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

// A bfloat16 pair (low half first) as packed floats.
__device__ __forceinline__ u64 bf2(uint32_t u)
{
    return pk2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}

// relu of a packed pair, rounded to a bfloat16 pair.
__device__ __forceinline__ uint32_t relu_bf2(u64 v)
{
    const float2 f = upk2(v);
    const __nv_bfloat162 h = __floats2bfloat162_rn(fmaxf(f.x, 0.0f), fmaxf(f.y, 0.0f));
    return *(const uint32_t *)&h;
}

template <int C>
__global__ void __launch_bounds__(DW_THREADS, 1)
dwpw_kernel(const __grid_constant__ CUtensorMap tma_in, const __grid_constant__ CUtensorMap tma_b,
            const __grid_constant__ CUtensorMap tma_o, DwParams p)
{
    using G = DwCfg<C>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    DwSmem<C> &s = *reinterpret_cast<DwSmem<C> *>(
        (void *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023));
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int my_tiles =
        p.ntiles > (int)blockIdx.x ? (p.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x
                                   : 0;
    const int nitems = my_tiles * G::NKB;

    if (threadIdx.x == 0) {
        mbar_init(&s.bfull, 1);
        for (int i = 0; i < G::NA; i++) {
            mbar_init(&s.afull[i], G::WI);
            mbar_init(&s.aempty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&s.accfull[i], 1);
            mbar_init(&s.accempty[i], 4);
        }
        for (int i = 0; i < G::NH; i++) {
            mbar_init(&s.pfull[i], 1);
            mbar_init(&s.pempty[i], G::WI);
        }
        s.eabort = 0;
        mbar_fence_init();
    }
    for (int e = threadIdx.x; e < C * 25; e += DW_THREADS) {
        const int c = e / 25, tap = e % 25;
        float *d = (float *)&s.dw[c / G::CK][tap][(c % G::CK) / 2];
        d[c & 1] = p.dw_w[e];
    }
    for (int c = threadIdx.x; c < C; c += DW_THREADS) {
        s.dwb[c] = p.dw_b[c];
        s.pwb[c] = p.pw_b[c];
    }
    if (warp == MMA_WARP)
        tmem_alloc(&s.tmem, G::TMEM_COLS);
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = s.tmem;

    if (warp < PROD_WARPS) {
        // ------------------------------------------------------ producers
        const int grp = warp / G::WI, gw = warp % G::WI;
        int row, pair;
        if (G::CK == 64) {
            row = gw;
            pair = lane;
        }
        else {
            row = 2 * gw + (lane >> 4);
            pair = lane & 15;
        }
        for (int i = grp; i < nitems; i += G::PG) {
            const int slot = i % G::NA, use = i / G::NA;
            // The MMAs of this A buffer's previous item are done, and item
            // i's patch has landed.
            if (!__all_sync(0xffffffffu,
                            (use == 0 || mbar_wait(&s.aempty[slot], (use - 1) & 1, 21)) &&
                                mbar_wait(&s.pfull[i % G::NH], (i / G::NH) & 1, 26)))
                break;
            const uint32_t *pb = s.patch[i % G::NH];
            const int kb = i % G::NKB, c = kb * G::CK + 2 * pair;
            u64 acc[TX];
            const u64 bb = *(const u64 *)&s.dwb[c];
#pragma unroll
            for (int o = 0; o < TX; o++)
                acc[o] = bb;
#pragma unroll
            for (int a = 0; a < 5; a++) {
                u64 w[5];
#pragma unroll
                for (int k = 0; k < 5; k++)
                    w[k] = *(const u64 *)&s.dw[kb][a * 5 + k][pair];
                const uint32_t *rp = pb + (row + a) * G::RPW + pair;
#pragma unroll
                for (int x = 0; x < TX + 4; x++) {
                    const u64 v = bf2(rp[x * G::NP]);
#pragma unroll
                    for (int k = 0; k < 5; k++) {
                        const int ox = x - k;
                        if (ox >= 0 && ox < TX)
                            acc[ox] = fma2p(v, w[k], acc[ox]);
                    }
                }
            }
            // Row m = pixel of the tile, 16-byte chunk (pair / 4) of its
            // 128-byte row at position chunk ^ (m % 8): the layout of a
            // 128-byte-swizzled K-major operand.
            uint32_t *ab = (uint32_t *)s.a[slot];
            const int chunk = pair >> 2, sub = pair & 3;
#pragma unroll
            for (int o = 0; o < TX; o++) {
                const int m = row * TX + o;
                ab[m * 32 + ((chunk ^ (m & 7)) << 2) + sub] = relu_bf2(acc[o]);
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&s.afull[slot]);
                mbar_arrive(&s.pempty[i % G::NH]);
            }
        }
    }
    else if (warp == LOAD_WARP) {
        // ---------------------------------------------------- patch loads
        if (lane == 0) {
            for (int i = 0; i < nitems; i++) {
                const int buf = i % G::NH, use = i / G::NH;
                // Every producer warp is done with this buffer's last item.
                if (use > 0 && !mbar_wait(&s.pempty[buf], (use - 1) & 1, 27))
                    break;
                const int t = (int)blockIdx.x + (i / G::NKB) * (int)gridDim.x, kb = i % G::NKB;
                const int x0 = (t % p.tiles_x) * TX - 2, y0 = (t / p.tiles_x) * TY - 2;
                mbar_expect_tx(&s.pfull[buf], (uint32_t)(G::PATCH_WORDS * 4));
                tma_load_3d(s.patch[buf], &tma_in, &s.pfull[buf], kb * G::CK, x0, y0);
            }
        }
    }
    else if (warp == MMA_WARP) {
        // ------------------------------------------------------------ MMA
        if (lane == 0) {
            mbar_expect_tx(&s.bfull, (uint32_t)(G::NKB * C * 64 * 2));
            for (int kb = 0; kb < G::NKB; kb++)
                tma_load_2d(s.b[kb], &tma_b, &s.bfull, kb * 64, 0);
            bool ok = mbar_wait(&s.bfull, 0, 22);
            constexpr uint32_t idesc = idesc_bf16(128, C);
            int it = 0;
            for (int lt = 0; lt < my_tiles && ok; lt++) {
                const int buf = lt & 1, use = lt >> 1;
                // The epilogue has read this accumulator's previous tile.
                if (use > 0 && !mbar_wait(&s.accempty[buf], (use - 1) & 1, 23))
                    break;
                fence_after();
                const uint32_t acc = tmem + (uint32_t)(buf * C);
                for (int kb = 0; kb < G::NKB; kb++, it++) {
                    const int slot = it % G::NA;
                    if (!mbar_wait(&s.afull[slot], (it / G::NA) & 1, 24)) {
                        ok = false;
                        break;
                    }
                    fence_after();
                    const uint64_t da = sw128_desc(su32(s.a[slot]));
                    const uint64_t db = sw128_desc(su32(s.b[kb]));
#pragma unroll
                    for (int k = 0; k < G::CK / 16; k++)
                        mma_bf16(acc, da + 2 * k, db + 2 * k, idesc,
                                 (kb > 0 || k > 0) ? 1u : 0u);
                    mma_commit(&s.aempty[slot]);
                }
                if (ok)
                    mma_commit(&s.accfull[buf]);
            }
        }
    }
    else {
        // ------------------------------------------------------- epilogue
        const int q = warp % 4, m = 32 * q + lane;
        const bool leader = warp == EPI_WARP0 && lane == 0;
        for (int lt = 0; lt < my_tiles; lt++) {
            const int t = (int)blockIdx.x + lt * (int)gridDim.x;
            const int buf = lt & 1, use = lt >> 1;
            // Decided per warp: the tensor-memory loads are warp-collective.
            const bool ok =
                __all_sync(0xffffffffu, mbar_wait_backoff(&s.accfull[buf], use & 1, 25));
            if (!ok && lane == 0)
                s.eabort = 1;
            // The TMA store that last used this staging buffer has read it.
            if (leader)
                bulk_wait_read<G::NO - 1>();
            named_bar(1, 128);
            if (s.eabort)
                break;
            fence_after();
            __nv_bfloat16 *ob = s.o[lt % G::NO];
            const uint32_t acc = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * C);
#pragma unroll 1
            for (int c0 = 0; c0 < C; c0 += 32) {
                float v[32];
                tmem_ld32(acc + c0, v);
                uint32_t wv[16];
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const __nv_bfloat162 h =
                        __floats2bfloat162_rn(v[2 * j] + s.pwb[c0 + 2 * j],
                                              v[2 * j + 1] + s.pwb[c0 + 2 * j + 1]);
                    wv[j] = *(const uint32_t *)&h;
                }
                // Box c0 / CK holds rows of CK channels (CK * 2 bytes),
                // 16-byte chunks swizzled as the output tensor map reads
                // them: 128-byte rows chunk ^ (m % 8), 64-byte rows
                // chunk ^ ((m / 2) % 4).
                char *rowp = (char *)ob + (c0 / G::CK) * (128 * G::CK * 2) + m * (G::CK * 2);
                const int lc0 = (c0 % G::CK) / 8;
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    const int lc = lc0 + u;
                    const int pc = G::OSW == 128 ? (lc ^ (m & 7)) : (lc ^ ((m >> 1) & 3));
                    *(uint4 *)(rowp + pc * 16) =
                        make_uint4(wv[4 * u], wv[4 * u + 1], wv[4 * u + 2], wv[4 * u + 3]);
                }
            }
            // This warp's tensor-memory reads are complete: free the
            // accumulator for the tile after next.
            fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&s.accempty[buf]);
            fence_async_smem();
            named_bar(1, 128);
            if (leader) {
                const int x0 = (t % p.tiles_x) * TX, y0 = (t / p.tiles_x) * TY;
                for (int box = 0; box < G::NKB; box++)
                    tma_store_3d(&tma_o, ob + box * 128 * G::CK, box * G::CK, x0, y0);
                bulk_commit();
            }
        }
        if (leader)
            bulk_wait_all();
    }
    fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        fence_after();
        tmem_dealloc(tmem, G::TMEM_COLS);
    }
}

template <int C>
bool launch_dwpw(cudaStream_t st, const __nv_bfloat16 *in, int H, int W, const float *dw_w,
                 const float *dw_b, const __nv_bfloat16 *pw_w, const float *pw_b,
                 __nv_bfloat16 *out, int sm_count)
{
    using G = DwCfg<C>;
    CUtensorMap mi, mb, mo;
    if (!make_map_hwc(&mi, const_cast<__nv_bfloat16 *>(in), H, W, C, G::CK, G::PXL, PY, 0))
        return false;
    if (!make_map_2d(&mb, pw_w, C, C, C, C))
        return false;
    if (!make_map_hwc(&mo, out, H, W, C, G::CK, TX, TY, G::OSW))
        return false;
    DwParams p;
    memset(&p, 0, sizeof(p));
    p.H = H;
    p.W = W;
    p.tiles_x = cdiv(W, TX);
    const long ntiles = (long)p.tiles_x * cdiv(H, TY);
    if (ntiles >= (1L << 30))
        return false;
    p.ntiles = (int)ntiles;
    p.dw_w = dw_w;
    p.dw_b = dw_b;
    p.pw_b = pw_b;
    static_assert(sizeof(DwSmem<C>) + 1024 <= 227 * 1024, "shared memory of one CTA");
    const size_t smem = sizeof(DwSmem<C>) + 1024;
    static unsigned done = 0;
    if (!smem_opt_in((const void *)dwpw_kernel<C>, smem, &done))
        return false;
    const int grid = (int)(ntiles < sm_count ? ntiles : sm_count);
    dwpw_kernel<C><<<grid, DW_THREADS, smem, st>>>(mi, mb, mo, p);
    return true;
}

// ------------------------------------------------ depthwise convolution
//
// The depthwise 5 x 5 convolution + bias + ReLU alone, for the refiners too
// wide for the fused kernel (C a multiple of 64). Output tiles of 16 x 16
// pixels x 64 channels; the 20 x 20-pixel input patch of each (tile,
// k-block) arrives by TMA in a ring of three buffers. Each producer thread
// computes two adjacent output rows of 8 pixels for one channel pair, so
// that every patch value it loads feeds up to ten packed FMAs (float32, the
// taps in the reference's order), and writes the bfloat16 result straight
// to global memory (a warp stores the 64 channels of one pixel, 128
// contiguous bytes). The weights are staged once per CTA in shared memory,
// tap-major with channel pairs innermost, and a thread's 25 weight pairs
// are reloaded from there (conflict-free) when the k-block changes; items
// (tile, k-block) go in k-block-major order over all CTAs. For maps of at
// least one tile per CTA: smaller ones spend more on the staging than it
// saves.

constexpr int DW5_WARPS = 16;                    // producer warps (thread 0 loads)
constexpr int DW5_THREADS = DW5_WARPS * 32;
constexpr int DW5_NHMAX = 3;
constexpr int DW5_TY = 16, DW5_PY = DW5_TY + 4;  // tile rows, patch rows
constexpr int DW5_PATCH_WORDS = DW5_PY * PX * 32;  // 64 channels: 32 words a pixel

// Dynamic shared memory: nh patch buffers, then the weights (C / 64
// k-blocks x 25 taps x 32 channel pairs, float pairs), then the barriers.
struct Dw5Layout {
    int nh;
    size_t w_off, bar_off, bytes;
};

__host__ __device__ inline Dw5Layout dw5_layout(int C)
{
    Dw5Layout l;
    l.nh = C <= 512 ? 3 : 2;
    l.w_off = (size_t)l.nh * DW5_PATCH_WORDS * 4;
    l.bar_off = l.w_off + (size_t)C * 25 * 4;
    l.bytes = l.bar_off + 2 * DW5_NHMAX * 8;
    return l;
}

struct Dw5Params {
    __nv_bfloat16 *out;
    const float *dw_w, *dw_b;
    int H, W, C, tiles_x, ntiles;
};

__global__ void __launch_bounds__(DW5_THREADS, 1)
dw5_kernel(const __grid_constant__ CUtensorMap tma_in, Dw5Params p)
{
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char *base = smem_raw + ((1024u - (su32(smem_raw) & 1023u)) & 1023u);
    const Dw5Layout L = dw5_layout(p.C);
    const int NH = L.nh;
    uint32_t *patch = (uint32_t *)base;
    float2 *wsm = (float2 *)(base + L.w_off);
    uint64_t *pfull = (uint64_t *)(base + L.bar_off), *pempty = pfull + DW5_NHMAX;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const long nall = (long)p.ntiles * (p.C / 64);
    const int nitems =
        nall > (long)blockIdx.x ? (int)((nall - (long)blockIdx.x + gridDim.x - 1) / gridDim.x) : 0;
    if (threadIdx.x == 0) {
        for (int i = 0; i < NH; i++) {
            mbar_init(&pfull[i], 1);
            mbar_init(&pempty[i], DW5_WARPS);
        }
        mbar_fence_init();
    }
    // Weights [c][25] -> [c / 64][tap][(c % 64) / 2], coalesced reads.
    for (int e = threadIdx.x; e < p.C * 25; e += DW5_THREADS) {
        const int c = e / 25, tap = e - c * 25;
        float *d = (float *)&wsm[((c >> 6) * 25 + tap) * 32 + ((c & 63) >> 1)];
        d[c & 1] = __ldg(p.dw_w + e);
    }
    __syncthreads();
    auto item = [&](int i, int *t, int *kb) {
        const int g = (int)blockIdx.x + i * (int)gridDim.x;
        *kb = g / p.ntiles;
        *t = g - *kb * p.ntiles;
    };
    // Thread 0 loads item i into buffer i % NH once every warp has released
    // the buffer's previous item.
    auto fetch = [&](int i) -> bool {
        const int buf = i % NH, use = i / NH;
        if (use > 0 && !mbar_wait(&pempty[buf], (use - 1) & 1, 31))
            return false;
        int t, kb;
        item(i, &t, &kb);
        const int ty = t / p.tiles_x, x0 = (t - ty * p.tiles_x) * TX - 2;
        const int y0 = ty * DW5_TY - 2;
        mbar_expect_tx(&pfull[buf], (uint32_t)(DW5_PATCH_WORDS * 4));
        tma_load_3d(patch + (size_t)buf * DW5_PATCH_WORDS, &tma_in, &pfull[buf], kb * 64, x0, y0);
        return true;
    };
    bool loading = true;
    if (threadIdx.x == 0)
        for (int i = 0; i < NH - 1 && i < nitems && loading; i++)
            loading = fetch(i);
    {
        const int row = 2 * (warp >> 1), px0 = 8 * (warp & 1), pair = lane;
        int cur = -1;
        u64 w[25], bb = 0;
        for (int i = 0; i < nitems; i++) {
            int t, kb;
            item(i, &t, &kb);
            const int c = kb * 64 + 2 * pair;
            if (kb != cur) {
#pragma unroll
                for (int k = 0; k < 25; k++)
                    w[k] = *(const u64 *)&wsm[(kb * 25 + k) * 32 + pair];
                bb = pk2(__ldg(p.dw_b + c), __ldg(p.dw_b + c + 1));
                cur = kb;
            }
            if (threadIdx.x == 0 && loading && i + NH - 1 < nitems)
                loading = fetch(i + NH - 1);
            const int buf = i % NH;
            if (!__all_sync(0xffffffffu, mbar_wait(&pfull[buf], (i / NH) & 1, 32)))
                break;
            const uint32_t *pb = patch + (size_t)buf * DW5_PATCH_WORDS;
            // Output rows row (acc0) and row + 1 (acc1) from patch rows
            // row .. row + 5: patch row j is tap row j of the first and j - 1
            // of the second.
            u64 acc0[8], acc1[8];
#pragma unroll
            for (int o = 0; o < 8; o++)
                acc0[o] = acc1[o] = bb;
#pragma unroll
            for (int j = 0; j < 6; j++) {
                const uint32_t *rp = pb + (row + j) * (PX * 32) + px0 * 32 + pair;
#pragma unroll
                for (int x = 0; x < 12; x++) {
                    const u64 v = bf2(rp[x * 32]);
#pragma unroll
                    for (int k = 0; k < 5; k++) {
                        const int ox = x - k;
                        if (ox >= 0 && ox < 8) {
                            if (j < 5)
                                acc0[ox] = fma2p(v, w[j * 5 + k], acc0[ox]);
                            if (j > 0)
                                acc1[ox] = fma2p(v, w[(j - 1) * 5 + k], acc1[ox]);
                        }
                    }
                }
            }
            // This warp is done with the patch.
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&pempty[buf]);
            const int ty = t / p.tiles_x;
            const int y = ty * DW5_TY + row, xb = (t - ty * p.tiles_x) * TX + px0;
            if (y < p.H) {
                __nv_bfloat16 *o = p.out + ((long)y * p.W + xb) * p.C + c;
#pragma unroll
                for (int k = 0; k < 8; k++)
                    if (xb + k < p.W)
                        *(uint32_t *)(o + (long)k * p.C) = relu_bf2(acc0[k]);
            }
            if (y + 1 < p.H) {
                __nv_bfloat16 *o = p.out + ((long)(y + 1) * p.W + xb) * p.C + c;
#pragma unroll
                for (int k = 0; k < 8; k++)
                    if (xb + k < p.W)
                        *(uint32_t *)(o + (long)k * p.C) = relu_bf2(acc1[k]);
            }
        }
    }
}

}  // namespace

int dwpw_status()
{
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_error, sizeof(int));
    if (v)
        cudaMemcpyToSymbol(g_error, &z, sizeof(int));
    return v;
}

}  // namespace tc

bool dw5_tc(cudaStream_t st, const void *in, int H, int W, int C, const float *dw_w,
            const float *dw_b, void *out, int sm_count)
{
    if (sm_count <= 0)
        sm_count = 148;
    if (H < 1 || W < 1 || C < 64 || C % 64 || ((uintptr_t)in & 15) || ((uintptr_t)out & 3) ||
        ((uintptr_t)dw_w & 15))
        return false;
    CUtensorMap mi;
    if (!tc::make_map_hwc(&mi, const_cast<void *>(in), H, W, C, 64, tc::PX, tc::DW5_PY, 0))
        return false;
    tc::Dw5Params p;
    p.out = (__nv_bfloat16 *)out;
    p.dw_w = dw_w;
    p.dw_b = dw_b;
    p.H = H;
    p.W = W;
    p.C = C;
    p.tiles_x = cdiv(W, tc::TX);
    const long ntiles = (long)p.tiles_x * cdiv(H, tc::DW5_TY);
    const long nall = ntiles * (C / 64);
    if (nall >= (1L << 30) || ntiles < sm_count)
        return false;
    p.ntiles = (int)ntiles;
    const size_t smem = tc::dw5_layout(C).bytes + 1024;
    if (smem > 227 * 1024)
        return false;
    // The opt-in covers the largest layout once per device.
    static unsigned done = 0;
    if (!tc::smem_opt_in((const void *)tc::dw5_kernel, 227 * 1024, &done))
        return false;
    const int grid = (int)(nall < sm_count ? nall : sm_count);
    tc::dw5_kernel<<<grid, tc::DW5_THREADS, smem, st>>>(mi, p);
    return true;
}

bool dwpw_tc(cudaStream_t st, const void *in, int H, int W, int C, const float *dw_w,
             const float *dw_b, const void *pw_w, const float *pw_b, void *out, int sm_count)
{
    if (sm_count <= 0)
        sm_count = 148;
    if (H < 1 || W < 1 || ((uintptr_t)in & 15) || ((uintptr_t)out & 15) || ((uintptr_t)pw_w & 15))
        return false;
    const auto *i16 = (const __nv_bfloat16 *)in;
    const auto *w16 = (const __nv_bfloat16 *)pw_w;
    auto *o16 = (__nv_bfloat16 *)out;
    if (C == 32)
        return tc::launch_dwpw<32>(st, i16, H, W, dw_w, dw_b, w16, pw_b, o16, sm_count);
    if (C == 64)
        return tc::launch_dwpw<64>(st, i16, H, W, dw_w, dw_b, w16, pw_b, o16, sm_count);
    if (C == 128)
        return tc::launch_dwpw<128>(st, i16, H, W, dw_w, dw_b, w16, pw_b, o16, sm_count);
    return false;
}

}  // namespace coreg
