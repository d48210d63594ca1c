// SPDX-License-Identifier: Unlicense
//
// tcgen05 tensor-core GEMM for sm_100a: C = act(alpha A B^T + bias) + R
// with A (M x K) and B (N x K) bfloat16, K-major (row-major with K
// contiguous), float32 accumulation in tensor memory, float32 or
// bfloat16 C: the GemmArgs contract of gemm.cuh (one product, column
// bias). In convolution mode (GemmArgs::amode 1) A is the implicit im2col
// of a 3 x 3 / padding 1 or 5 x 5 / padding 2 convolution (stride 1) over a
// channels-last map, each k-block a 3-D TMA box of the map shifted by the
// tap, zeros read at the borders: no im2col buffer.
//
// Persistent: one CTA per SM walks the 128 x BN output tiles t = blockIdx.x,
// blockIdx.x + gridDim.x, ... (row blocks fastest, so that the CTAs running
// at one time share the weight columns in L2). Warp-specialized:
//   warp 0      TMA producer: A and B tiles of 64 K-elements per stage,
//               128-byte swizzled, into a ring of STAGES shared-memory
//               stages (mbarrier full[s], transaction bytes); the ring runs
//               on across tile boundaries;
//   warp 1      tensor-memory allocator and MMA issuer: one thread issues
//               4 tcgen05.mma (K = 16 each) per stage into one of two
//               128 x BN float32 accumulators in TMEM (tiles alternate),
//               commits each stage to empty[s] (the producer's refill
//               signal) and each finished tile to acc_full[buffer]
//               (two accumulators, four for tiles of at most 64 columns);
//   warps 2..9  epilogue, two warps per TMEM lane quadrant (alternate
//               32-column chunks): each reads its 32 lanes (rows) with
//               tcgen05.ld, transposes them through a padded shared-memory
//               block and writes every row with one coalesced warp store
//               (lane = column), bias, activation and residual applied on
//               the way, then frees the accumulator (acc_empty[buffer]).
//               Stores of one row per thread would make 32 separate memory
//               requests per instruction.
// With two or four accumulators the epilogue of a tile overlaps the main
// loops of the next ones.
// Every mbarrier wait is bounded (about two seconds); a wait that runs out
// records an error code (coreg_tc_status) and the CTA leaves its loops,
// frees its tensor memory and returns.

#include <mutex>
#include <stdlib.h>
#include <string.h>

#include "tc_common.cuh"

namespace coreg {
namespace tc {

namespace {

constexpr int BM = 128, BK = 64;
// Producer warp, MMA warp, eight epilogue warps.
constexpr int NTHREADS = 320;

struct TcParams {
    int M, N, K;
    void *C;
    long ldc;
    const float *bias;    // per column
    const float *bias_r;  // per row
    const void *R;
    float alpha;
    int act;
    float slope;
    int c_bf16;
    // Convolution mode (ksz x ksz, ksz 3 or 5, stride 1, padding ksz / 2,
    // channels-last input of cH x cW x cC, cC a multiple of 64): the tile
    // is TW x TH output pixels (TW TH = 128), k-block kb = (tap, 64-channel
    // chunk), tap = ky ksz + kx.
    int conv, cH, cW, cC, TW, TH, tiles_x, tiles_y, ksz;
    // Tap reuse (3 x 3 only): a stage is one (64-channel chunk, column tap
    // dx) with one A box of TW x (TH + 2) pixels (tensor map tma_a3) and the
    // three weight tiles of the row taps dy = 0..2; the A operand of tap (dy,
    // dx) is that box from row dy TW on. reuse = the number of such stages
    // that fit the shared memory (0: off), rsb its bytes, rab its A bytes.
    int reuse, rsb, rab;
    // Epilogue through TMA stores (output tensor map tma_c); else one
    // coalesced store per row.
    int tma_out;
};

template <int BN, int STAGES>
struct Smem {
    alignas(1024) __nv_bfloat16 a[STAGES][BM * BK];
    alignas(1024) __nv_bfloat16 b[STAGES][BN * BK];
    // Per epilogue warp: the staging block of its TMA stores (32 x 32
    // values, swizzled), or of its transposes.
    alignas(1024) unsigned char cst[8][4096];
    uint64_t full[STAGES], empty[STAGES], acc_full[4], acc_empty[4];
    uint32_t tmem;
};

constexpr int EPI_WARPS = NTHREADS / 32 - 2;
static_assert(EPI_WARPS == 8, "one staging block per epilogue warp");

// TMEM columns per accumulator: BN rounded up to a power of two (the
// allocation must be one), at least the 32 that one tcgen05.ld of the
// epilogue reads (the allocation granule).
template <int BN>
constexpr int acc_cols() { return BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256; }

// Tiles of at most 64 columns end after a few k-blocks, so that one
// epilogue per tile cannot keep up: the two epilogue warp groups (warps
// 2..5, 6..9) take alternate tiles whole, over four accumulators. Wider
// tiles: both groups on every tile (alternate 32-column chunks), two
// accumulators.
template <int BN>
constexpr bool split_epi() { return BN <= 64; }
template <int BN>
constexpr int n_acc() { return split_epi<BN>() ? 4 : 2; }

// Output tile t: first row (dense) or pixel origin (convolution) and first
// column.
struct Tile {
    int m0, n0, cx0, cy0;
};

template <int BN>
__device__ __forceinline__ Tile tile_of(const TcParams &p, int t, int tiles_m)
{
    const int mt = t % tiles_m;
    Tile r;
    r.m0 = mt * BM;
    r.n0 = (t / tiles_m) * BN;
    r.cx0 = p.conv ? (mt % p.tiles_x) * p.TW : 0;
    r.cy0 = p.conv ? (mt / p.tiles_x) * p.TH : 0;
    return r;
}

// First k-block of tile t: the tiles that share an A row block or a B
// column block start their K loops at different k-blocks, so that the
// CTAs running at one time do not all request the same operand tile from
// L2 at once. Only the order of the float32 sums changes.
__device__ __forceinline__ int k_rotation(int t, int tiles_m, int nk)
{
    const int mt = t % tiles_m, nt = t / tiles_m;
    return (int)(((unsigned)mt * 5u + (unsigned)nt * 3u) % (unsigned)nk);
}

// v[j] += R[j] for the j < n (at most 32) columns of a residual row.
__device__ __forceinline__ void add_row(float v[32], const float *R, int n)
{
    if (n >= 32 && ((uintptr_t)R & 15) == 0) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float4 x = __ldg((const float4 *)R + j);
            v[4 * j] += x.x;
            v[4 * j + 1] += x.y;
            v[4 * j + 2] += x.z;
            v[4 * j + 3] += x.w;
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < 32; j++)
        if (j < n)
            v[j] += R[j];
}

__device__ __forceinline__ void add_row(float v[32], const __nv_bfloat16 *R, int n)
{
    if (n >= 32 && ((uintptr_t)R & 15) == 0) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint4 x = __ldg((const uint4 *)R + j);
            const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                v[8 * j + 2 * k] += __uint_as_float(w[k] << 16);
                v[8 * j + 2 * k + 1] += __uint_as_float(w[k] & 0xffff0000u);
            }
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < 32; j++)
        if (j < n)
            v[j] += __bfloat162float(R[j]);
}

// Row l of a 32-column staging block in the layout of the output tensor
// map's box: float rows of 128 bytes, 16-byte chunk c at c ^ (l % 8)
// (128-byte swizzle); bfloat16 rows of 64 bytes, chunk c at c ^ ((l / 2) %
// 4) (64-byte swizzle).
__device__ __forceinline__ void stage_row(unsigned char *blk, int l, const float v[32], float *)
{
#pragma unroll
    for (int c = 0; c < 8; c++)
        *(float4 *)(blk + l * 128 + ((c ^ (l & 7)) << 4)) =
            make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
}

__device__ __forceinline__ void stage_row(unsigned char *blk, int l, const float v[32],
                                          __nv_bfloat16 *)
{
#pragma unroll
    for (int c = 0; c < 4; c++) {
        uint32_t w[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(v[8 * c + 2 * k], v[8 * c + 2 * k + 1]);
            w[k] = *(const uint32_t *)&h;
        }
        *(uint4 *)(blk + l * 64 + ((c ^ ((l >> 1) & 3)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// The activation (ACT, or -1 for the run-time one of p.act) and the output
// type are template parameters: a run-time switch would inline every
// activation's math into the unrolled epilogue loop, and that code size
// slows the epilogue down by several times.
template <int BN, int STAGES, int ACT, typename TC>
__global__ void __launch_bounds__(NTHREADS, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tma_a,
               const __grid_constant__ CUtensorMap tma_b,
               const __grid_constant__ CUtensorMap tma_c,
               const __grid_constant__ CUtensorMap tma_a3, TcParams p)
{
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    Smem<BN, STAGES> &s = *reinterpret_cast<Smem<BN, STAGES> *>(
        smem_raw + ((1024u - (su32(smem_raw) & 1023u)) & 1023u));
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int nk = (p.K + BK - 1) / BK;
    // Stages per tile and stage slots: k-blocks, or (chunk, dx) pairs with
    // tap reuse.
    const int nst = p.reuse ? 3 * (p.cC / BK) : nk;
    const int slots = p.reuse ? p.reuse : STAGES;
    unsigned char *const rbase = reinterpret_cast<unsigned char *>(s.a);
    const int tiles_m = p.conv ? p.tiles_x * p.tiles_y : (p.M + BM - 1) / BM;
    const int ntiles = tiles_m * ((p.N + BN - 1) / BN);

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        for (int i = 0; i < n_acc<BN>(); i++) {
            mbar_init(&s.acc_full[i], 1);
            mbar_init(&s.acc_empty[i], split_epi<BN>() ? 4 : EPI_WARPS);
        }
        mbar_fence_init();
    }
    if (warp == 1)
        tmem_alloc(&s.tmem, n_acc<BN>() * acc_cols<BN>());
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = s.tmem;

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t bytes =
                p.reuse ? (uint32_t)(p.rab + 3 * BN * BK * 2) : (uint32_t)((BM + BN) * BK * 2);
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const Tile tl = tile_of<BN>(p, t, tiles_m);
                const int k_off = k_rotation(t, tiles_m, nst);
                for (int kk = 0; kk < nst; kk++, it++) {
                    const int kb = kk + k_off < nst ? kk + k_off : kk + k_off - nst;
                    const int st = it % slots;
                    if (it >= slots && !mbar_wait(&s.empty[st], ((it / slots) - 1) & 1, 1)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&s.full[st], bytes);
                    if (p.reuse) {
                        // Stage kb = (chunk c, column tap dx): the A box one
                        // row above the tile, then the weights of taps (dy,
                        // dx), columns (dy 3 + dx) C + 64 c.
                        unsigned char *sa = rbase + (size_t)st * p.rsb;
                        const int c = kb / 3, dx = kb % 3;
                        tma_load_3d(sa, &tma_a3, &s.full[st], c * BK, tl.cx0 + dx - 1, tl.cy0 - 1);
                        for (int dy = 0; dy < 3; dy++)
                            tma_load_2d(sa + p.rab + dy * BN * BK * 2, &tma_b, &s.full[st],
                                        (dy * 3 + dx) * p.cC + c * BK, tl.n0);
                        continue;
                    }
                    if (p.conv) {
                        const int chunks = p.cC / BK, tap = kb / chunks;
                        const int c0 = (kb % chunks) * BK, pad = p.ksz / 2;
                        tma_load_3d(s.a[st], &tma_a, &s.full[st], c0,
                                    tl.cx0 + tap % p.ksz - pad, tl.cy0 + tap / p.ksz - pad);
                    }
                    else
                        tma_load_2d(s.a[st], &tma_a, &s.full[st], kb * BK, tl.m0);
                    tma_load_2d(s.b[st], &tma_b, &s.full[st], kb * BK, tl.n0);
                }
            }
        }
    }
    else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(BM, BN);
            int it = 0, lt = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, lt++) {
                const int buf = lt % n_acc<BN>(), use = lt / n_acc<BN>();
                // The epilogue has read this accumulator's previous tile.
                if (use > 0 && !mbar_wait(&s.acc_empty[buf], (use - 1) & 1, 4))
                    break;
                fence_after();
                const uint32_t acc = tmem + (uint32_t)(buf * acc_cols<BN>());
                for (int kk = 0; kk < nst; kk++, it++) {
                    const int st = it % slots;
                    // TMA completion through the mbarrier orders the tile
                    // for the tensor cores; no tcgen05 fence is needed here.
                    if (!mbar_wait(&s.full[st], (it / slots) & 1, 2)) {
                        ok = false;
                        break;
                    }
                    if (p.reuse) {
                        // Taps (dy, dx) for dy = 0..2: A from row dy TW of
                        // the box (a multiple of 8 rows: 1024-byte aligned).
                        const uint32_t sa = su32(rbase + (size_t)st * p.rsb);
                        for (int dy = 0; dy < 3; dy++) {
                            const uint64_t da = sw128_desc(sa + (uint32_t)(dy * p.TW * 128));
                            const uint64_t db =
                                sw128_desc(sa + (uint32_t)(p.rab + dy * BN * BK * 2));
#pragma unroll
                            for (int k = 0; k < BK / 16; k++)
                                mma_bf16(acc, da + 2 * k, db + 2 * k, idesc,
                                         (kk > 0 || dy > 0 || k > 0) ? 1u : 0u);
                        }
                        mma_commit(&s.empty[st]);
                        continue;
                    }
                    const uint64_t da = sw128_desc(su32(s.a[st]));
                    const uint64_t db = sw128_desc(su32(s.b[st]));
#pragma unroll
                    for (int k = 0; k < BK / 16; k++)
                        mma_bf16(acc, da + 2 * k, db + 2 * k, idesc,
                                 (kk > 0 || k > 0) ? 1u : 0u);
                    mma_commit(&s.empty[st]);
                }
                if (ok)
                    mma_commit(&s.acc_full[buf]);
            }
        }
    }
    else {
        // Epilogue: warp w owns TMEM lanes (rows) 32 (w % 4) ...; of wide
        // tiles it takes the 32-column chunks of parity (w - 2) / 4 (two
        // warps per lane quadrant, so that each scheduler interleaves two
        // epilogue warps), of narrow ones (split_epi) every column of the
        // tiles of parity (w - 2) / 4.
        const int q = warp % 4, half = (warp - 2) / 4;
        const int r = 32 * q + lane;
        unsigned char *cst = s.cst[warp - 2];
        float *stage = (float *)cst;
        TC *C = (TC *)p.C;
        const TC *R = (const TC *)p.R;
        int lt = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, lt++) {
            if (split_epi<BN>() && (lt & 1) != half)
                continue;
            const int buf = lt % n_acc<BN>(), use = lt / n_acc<BN>();
            const Tile tl = tile_of<BN>(p, t, tiles_m);
            int row = tl.m0 + r;
            if (p.conv) {
                const int px = tl.cx0 + r % p.TW, py = tl.cy0 + r / p.TW;
                row = px < p.cW && py < p.cH ? py * p.cW + px : p.M;
            }
            // Decided per warp: the TMEM loads below are warp-collective.
            if (!__all_sync(0xffffffffu, mbar_wait_backoff(&s.acc_full[buf], use & 1, 3)))
                break;
            fence_after();
            const uint32_t acc =
                tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(buf * acc_cols<BN>());
            const int cs = split_epi<BN>() ? 0 : 32 * half, cstep = split_epi<BN>() ? 32 : 64;
            for (int c0 = cs; c0 < BN && tl.n0 + c0 < p.N; c0 += cstep) {
                float v[32];
                tmem_ld32(acc + c0, v);
                if (p.tma_out) {
                    // Lane = row: bias, activation and residual on this
                    // row's 32 values, then one TMA store of the warp's 32 x
                    // 32 block (clipped at the matrix or map edges).
                    const int col0 = tl.n0 + c0;
                    const float br = p.bias_r && row < p.M ? __ldg(p.bias_r + row) : 0.0f;
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        const float b = p.bias && col0 + j < p.N ? __ldg(p.bias + col0 + j) : 0.0f;
                        v[j] = apply_act(p.alpha * v[j] + b + br, ACT >= 0 ? ACT : p.act,
                                         p.slope);
                    }
                    if (R && row < p.M)
                        add_row(v, R + (long)row * p.ldc + col0, p.N - col0);
                    // The previous store has read the staging block.
                    if (lane == 0)
                        bulk_wait_read<0>();
                    __syncwarp();
                    stage_row(cst, lane, v, (TC *)nullptr);
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        if (p.conv)
                            tma_store_3d(&tma_c, cst, col0, tl.cx0 + (32 * q) % p.TW,
                                         tl.cy0 + (32 * q) / p.TW);
                        else
                            tma_store_2d(&tma_c, cst, col0, tl.m0 + 32 * q);
                        bulk_commit();
                    }
                    continue;
                }
                // Transpose through the staging block (rotated rows: no bank
                // conflicts either way).
#pragma unroll
                for (int j = 0; j < 32; j++)
                    stage[lane * 32 + ((j + lane) & 31)] = v[j];
                __syncwarp();
                // Lane = column from here on.
                const int col = tl.n0 + c0 + lane;
                const bool cok = col < p.N && c0 + lane < BN;
                const float bias = cok && p.bias ? p.bias[col] : 0.0f;
#pragma unroll 4
                for (int rr = 0; rr < 32; rr++) {
                    const int grow = __shfl_sync(0xffffffffu, row, rr);
                    if (grow < p.M && cok) {
                        const long idx = (long)grow * p.ldc + col;
                        float x = p.alpha * stage[rr * 32 + ((lane + rr) & 31)] + bias;
                        if (p.bias_r)
                            x += p.bias_r[grow];
                        x = apply_act(x, ACT >= 0 ? ACT : p.act, p.slope);
                        if (R)
                            x += ldf(R + idx);
                        stf(C + idx, x);
                    }
                }
                __syncwarp();
            }
            // This warp's reads of the accumulator are complete (each
            // tcgen05.ld waited): hand it back to the MMA warp.
            fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&s.acc_empty[buf]);
        }
        // This warp's TMA stores have written global memory.
        if (lane == 0)
            bulk_wait_all();
    }
    fence_before();
    __syncthreads();
    if (warp == 1) {
        fence_after();
        tmem_dealloc(tmem, n_acc<BN>() * acc_cols<BN>());
    }
}

// ------------------------------------------------------------ 256 x 256
//
// Dense products with 256 x BN2 output tiles (BN2 256, 192 or 160): two M =
// 128 tcgen05.mma per k-step share each B tile (acc0 = rows 0..127 in TMEM
// columns 0.., acc1 = rows 128..255 from column 256). Per staged byte that
// is up to 1.5 times the tensor work of the 128 x 256 tile (64 KB feed 8
// MMAs instead of 48 KB feeding 4) and a third less L2 traffic per
// product, so that the three stages that fit the shared memory hold more
// work in flight; the width is chosen so that the tiles fill whole rounds
// of the SMs. The price: the accumulators take the tensor memory, so that
// a tile's epilogue overlaps only the TMA loads of the next. Same
// warp roles as tc_gemm_kernel: warp 0 TMA, warp 1 TMEM and MMA, warps
// 2..9 epilogue (warp w: TMEM lane quadrant w % 4 of accumulator (w - 2) /
// 4, all 256 columns in 32-column chunks, TMA stores).
constexpr int BM2 = 256, ST2 = 3;

template <int BN2>
struct Smem2 {
    alignas(1024) __nv_bfloat16 a[ST2][BM2 * BK];
    alignas(1024) __nv_bfloat16 b[ST2][BN2 * BK];
    alignas(1024) unsigned char cst[8][4096];
    uint64_t full[ST2], empty[ST2], acc_full, acc_empty;
    uint32_t tmem;
};

template <int BN2, int ACT, typename TC>
__global__ void __launch_bounds__(NTHREADS, 1)
tc_gemm2_kernel(const __grid_constant__ CUtensorMap tma_a,
                const __grid_constant__ CUtensorMap tma_b,
                const __grid_constant__ CUtensorMap tma_c, TcParams p)
{
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    Smem2<BN2> &s =
        *reinterpret_cast<Smem2<BN2> *>(smem_raw + ((1024u - (su32(smem_raw) & 1023u)) & 1023u));
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int nk = (p.K + BK - 1) / BK;
    const int tiles_m = (p.M + BM2 - 1) / BM2;
    const int ntiles = tiles_m * ((p.N + BN2 - 1) / BN2);

    if (threadIdx.x == 0) {
        for (int i = 0; i < ST2; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        mbar_init(&s.acc_full, 1);
        mbar_init(&s.acc_empty, EPI_WARPS);
        mbar_fence_init();
    }
    if (warp == 1)
        tmem_alloc(&s.tmem, 512);
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = s.tmem;

    if (warp == 0) {
        if (lane == 0) {
            constexpr uint32_t bytes = (uint32_t)(BM2 + BN2) * BK * 2;
            int it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x) {
                const int m0 = (t % tiles_m) * BM2, n0 = (t / tiles_m) * BN2;
                const int k_off = k_rotation(t, tiles_m, nk);
                for (int kk = 0; kk < nk; kk++, it++) {
                    const int kb = kk + k_off < nk ? kk + k_off : kk + k_off - nk;
                    const int st = it % ST2;
                    if (it >= ST2 && !mbar_wait(&s.empty[st], ((it / ST2) - 1) & 1, 31)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(&s.full[st], bytes);
                    tma_load_2d(s.a[st], &tma_a, &s.full[st], kb * BK, m0);
                    tma_load_2d(s.b[st], &tma_b, &s.full[st], kb * BK, n0);
                }
            }
        }
    }
    else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(128, BN2);
            int it = 0, lt = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < ntiles && ok; t += gridDim.x, lt++) {
                // The epilogue has read both accumulators of the previous tile.
                if (lt > 0 && !mbar_wait(&s.acc_empty, (lt - 1) & 1, 34))
                    break;
                fence_after();
                for (int kk = 0; kk < nk; kk++, it++) {
                    const int st = it % ST2;
                    if (!mbar_wait(&s.full[st], (it / ST2) & 1, 32)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sa = su32(s.a[st]);
                    const uint64_t da0 = sw128_desc(sa), da1 = sw128_desc(sa + 128 * 128);
                    const uint64_t db = sw128_desc(su32(s.b[st]));
#pragma unroll
                    for (int k = 0; k < BK / 16; k++) {
                        const uint32_t acc = (kk > 0 || k > 0) ? 1u : 0u;
                        mma_bf16(tmem, da0 + 2 * k, db + 2 * k, idesc, acc);
                        mma_bf16(tmem + 256, da1 + 2 * k, db + 2 * k, idesc, acc);
                    }
                    mma_commit(&s.empty[st]);
                }
                if (ok)
                    mma_commit(&s.acc_full);
            }
        }
    }
    else {
        const int q = warp % 4, half = (warp - 2) / 4;
        const int rr = 128 * half + 32 * q + lane;
        unsigned char *cst = s.cst[warp - 2];
        const TC *R = (const TC *)p.R;
        int lt = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, lt++) {
            const int m0 = (t % tiles_m) * BM2, n0 = (t / tiles_m) * BN2;
            const int row = m0 + rr;
            if (!__all_sync(0xffffffffu, mbar_wait_backoff(&s.acc_full, lt & 1, 33)))
                break;
            fence_after();
            const uint32_t acc = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(256 * half);
            const float br = p.bias_r && row < p.M ? __ldg(p.bias_r + row) : 0.0f;
            for (int c0 = 0; c0 < BN2 && n0 + c0 < p.N; c0 += 32) {
                float v[32];
                tmem_ld32(acc + c0, v);
                const int col0 = n0 + c0;
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    const float b = p.bias && col0 + j < p.N ? __ldg(p.bias + col0 + j) : 0.0f;
                    v[j] = apply_act(p.alpha * v[j] + b + br, ACT >= 0 ? ACT : p.act, p.slope);
                }
                if (R && row < p.M)
                    add_row(v, R + (long)row * p.ldc + col0, p.N - col0);
                if (lane == 0)
                    bulk_wait_read<0>();
                __syncwarp();
                stage_row(cst, lane, v, (TC *)nullptr);
                fence_async_smem();
                __syncwarp();
                if (lane == 0) {
                    tma_store_2d(&tma_c, cst, col0, m0 + 128 * half + 32 * q);
                    bulk_commit();
                }
            }
            fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&s.acc_empty);
        }
        if (lane == 0)
            bulk_wait_all();
    }
    fence_before();
    __syncthreads();
    if (warp == 1) {
        fence_after();
        tmem_dealloc(tmem, 512);
    }
}

template <int BN2, int ACT, typename TC>
bool run_tc2(cudaStream_t st, int grid, const CUtensorMap &ma, const CUtensorMap &mb,
             const CUtensorMap &mc, const TcParams &p)
{
    const size_t smem = sizeof(Smem2<BN2>) + 1024;
    static unsigned done = 0;
    if (!smem_opt_in((const void *)tc_gemm2_kernel<BN2, ACT, TC>, smem, &done))
        return false;
    tc_gemm2_kernel<BN2, ACT, TC><<<grid, NTHREADS, smem, st>>>(ma, mb, mc, p);
    return true;
}

// Tile width (pixels) of the convolution mode with the fewest wasted
// output positions for an H x W map.
int conv_tile_width(int H, int W)
{
    int best = 128;
    long best_w = -1;
    for (int tw = 128; tw >= 8; tw /= 2) {
        const int th = BM / tw;
        const long cells = (long)cdiv(W, tw) * tw * cdiv(H, th) * th;
        if (best_w < 0 || cells < best_w) {
            best_w = cells;
            best = tw;
        }
    }
    return best;
}

template <int BN, int STAGES, int ACT, typename TC>
bool run_tc(cudaStream_t st, int grid, const CUtensorMap &ma, const CUtensorMap &mb,
            const CUtensorMap &mc, const CUtensorMap &ma3, const TcParams &p)
{
    const size_t smem = sizeof(Smem<BN, STAGES>) + 1024;
    static unsigned done = 0;
    if (!smem_opt_in((const void *)tc_gemm_kernel<BN, STAGES, ACT, TC>, smem, &done))
        return false;
    tc_gemm_kernel<BN, STAGES, ACT, TC><<<grid, NTHREADS, smem, st>>>(ma, mb, mc, ma3, p);
    return true;
}

bool make_map_c(CUtensorMap *map, void *base, int es, const TcParams &p, long ldc);

template <int BN, int STAGES>
bool launch_tc(cudaStream_t st, const GemmArgs &g, int sm_count)
{
    CUtensorMap ma, mb, mc, ma3;
    TcParams p;
    memset(&p, 0, sizeof(p));
    memset(&ma3, 0, sizeof(ma3));
    long tiles_m = cdiv(g.M, BM);
    if (g.amode == 1) {
        p.conv = 1;
        p.ksz = g.cK ? g.cK : 3;
        p.cH = g.cH;
        p.cW = g.cW;
        p.cC = g.cC;
        p.TW = conv_tile_width(g.cH, g.cW);
        p.TH = BM / p.TW;
        p.tiles_x = cdiv(g.cW, p.TW);
        p.tiles_y = cdiv(g.cH, p.TH);
        tiles_m = (long)p.tiles_x * p.tiles_y;
        if (!make_map_conv(&ma, g.A, g.cH, g.cW, g.cC, p.TW, p.TH))
            return false;
        // Tap reuse where two of its stages fit the stage memory and the
        // shifted A operands stay 1024-byte aligned (TW a multiple of 8).
        const int rab = (p.TW * (p.TH + 2) * BK * 2 + 1023) / 1024 * 1024;
        const int rsb = rab + 3 * BN * BK * 2;
        const int total = STAGES * (BM + BN) * BK * 2;
        if (p.ksz == 3 && p.TW % 8 == 0 && p.TH + 2 <= 256 && total / rsb >= 2 &&
            make_map_conv(&ma3, g.A, g.cH, g.cW, g.cC, p.TW, p.TH + 2)) {
            p.reuse = total / rsb;
            p.rsb = rsb;
            p.rab = rab;
        }
    }
    else if (!make_map_2d(&ma, g.A, g.M, g.K, g.lda, BM))
        return false;
    if (!make_map_2d(&mb, g.B, g.N, g.K, g.ldb, BN))
        return false;
    p.M = g.M;
    p.N = g.N;
    p.K = g.K;
    p.C = g.C;
    p.ldc = g.ldc;
    p.bias = g.biasrow ? nullptr : g.bias;
    p.bias_r = g.biasrow ? g.bias : nullptr;
    p.R = g.R;
    p.alpha = g.alpha;
    p.act = g.act;
    p.slope = g.slope;
    p.c_bf16 = g.c == DT_BF16;
    const long ntiles = tiles_m * cdiv(g.N, BN);
    if (ntiles >= (1L << 31))
        return false;
    // TMA-store epilogue where the output allows a tensor map (tiles of at
    // least 32 columns, 16-byte aligned rows).
    memset(&mc, 0, sizeof(mc));
    p.tma_out = BN >= 32 && make_map_c(&mc, g.C, g.c == DT_BF16 ? 2 : 4, p, g.ldc);
    // Persistent: at most one CTA per SM (the shared memory allows one).
    const int grid = (int)(ntiles < sm_count ? ntiles : sm_count);
    if (p.c_bf16) {
        if (g.act == ACTF_NONE)
            return run_tc<BN, STAGES, ACTF_NONE, __nv_bfloat16>(st, grid, ma, mb, mc, ma3, p);
        if (g.act == ACTF_GELU)
            return run_tc<BN, STAGES, ACTF_GELU, __nv_bfloat16>(st, grid, ma, mb, mc, ma3, p);
        if (g.act == ACTF_RELU)
            return run_tc<BN, STAGES, ACTF_RELU, __nv_bfloat16>(st, grid, ma, mb, mc, ma3, p);
        return run_tc<BN, STAGES, -1, __nv_bfloat16>(st, grid, ma, mb, mc, ma3, p);
    }
    if (g.act == ACTF_NONE)
        return run_tc<BN, STAGES, ACTF_NONE, float>(st, grid, ma, mb, mc, ma3, p);
    return run_tc<BN, STAGES, -1, float>(st, grid, ma, mb, mc, ma3, p);
}

// 256 x BN2 tiles for a dense product without an activation (GemmArgs
// amode 0).
template <int BN2>
bool launch_tc2(cudaStream_t st, const GemmArgs &g, int sm_count)
{
    CUtensorMap ma, mb, mc;
    TcParams p;
    memset(&p, 0, sizeof(p));
    if (!make_map_2d(&ma, g.A, g.M, g.K, g.lda, BM2) || !make_map_2d(&mb, g.B, g.N, g.K, g.ldb, BN2))
        return false;
    p.M = g.M;
    p.N = g.N;
    p.K = g.K;
    p.C = g.C;
    p.ldc = g.ldc;
    p.bias = g.biasrow ? nullptr : g.bias;
    p.bias_r = g.biasrow ? g.bias : nullptr;
    p.R = g.R;
    p.alpha = g.alpha;
    p.act = g.act;
    p.slope = g.slope;
    p.c_bf16 = g.c == DT_BF16;
    memset(&mc, 0, sizeof(mc));
    if (!make_map_c(&mc, g.C, g.c == DT_BF16 ? 2 : 4, p, g.ldc))
        return false;
    const long ntiles = (long)cdiv(g.M, BM2) * cdiv(g.N, BN2);
    const int grid = (int)(ntiles < sm_count ? ntiles : sm_count);
    if (g.act != ACTF_NONE)
        return false;
    if (p.c_bf16)
        return run_tc2<BN2, ACTF_NONE, __nv_bfloat16>(st, grid, ma, mb, mc, p);
    return run_tc2<BN2, ACTF_NONE, float>(st, grid, ma, mb, mc, p);
}

typedef CUresult (*EncodeTiled)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                const cuuint32_t *, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion,
                                CUtensorMapFloatOOBfill);

EncodeTiled encoder()
{
    static EncodeTiled fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiled)p;
        else
            cudaGetLastError();
    });
    return fn;
}

// Tensor map of the GEMM output C for the epilogue's TMA stores: 2-D
// (N columns x M rows, row pitch ldc) or, in convolution mode, 3-D
// channels-last (N, cW, cH); box 32 columns x 32 rows (pixels), 128-byte
// (float) or 64-byte (bfloat16) swizzle. False when C's alignment or pitch
// does not allow one.
bool make_map_c(CUtensorMap *map, void *base, int es, const TcParams &p, long ldc)
{
    EncodeTiled enc = encoder();
    if (!enc || ((uintptr_t)base & 15) || (ldc * es) % 16)
        return false;
    const CUtensorMapDataType dt =
        es == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    const CUtensorMapSwizzle sw = es == 4 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    cuuint32_t estr[3] = {1, 1, 1};
    if (p.conv) {
        const int bw = p.TW < 32 ? p.TW : 32;
        cuuint64_t dims[3] = {(cuuint64_t)p.N, (cuuint64_t)p.cW, (cuuint64_t)p.cH};
        cuuint64_t strides[2] = {(cuuint64_t)ldc * es, (cuuint64_t)p.cW * ldc * es};
        cuuint32_t box[3] = {32, (cuuint32_t)bw, (cuuint32_t)(32 / bw)};
        return enc(map, dt, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    cuuint64_t dims[2] = {(cuuint64_t)p.N, (cuuint64_t)p.M};
    cuuint64_t strides[1] = {(cuuint64_t)ldc * es};
    cuuint32_t box[2] = {32, 32};
    return enc(map, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool make_map_2d(CUtensorMap *map, const void *base, long rows, long cols, long ld,
                 int box_rows)
{
    EncodeTiled enc = encoder();
    if (!enc)
        return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims,
               strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_map_conv(CUtensorMap *map, const void *base, int H, int W, int C, int TW,
                   int TH)
{
    EncodeTiled enc = encoder();
    if (!enc)
        return false;
    cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H};
    cuuint64_t strides[2] = {(cuuint64_t)C * 2, (cuuint64_t)W * C * 2};
    cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)TW, (cuuint32_t)TH};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void *>(base), dims,
               strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D bfloat16 tensor map of a channels-last (H, W, C) map for TMA
// stores (or loads) of box_c x box_w x box_h boxes, swizzle_bytes 0, 64 or
// 128.
bool make_map_hwc(CUtensorMap *map, void *base, int H, int W, int C, int box_c, int box_w,
                  int box_h, int swizzle_bytes)
{
    EncodeTiled enc = encoder();
    if (!enc)
        return false;
    cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)W, (cuuint64_t)H};
    cuuint64_t strides[2] = {(cuuint64_t)C * 2, (cuuint64_t)W * C * 2};
    cuuint32_t box[3] = {(cuuint32_t)box_c, (cuuint32_t)box_w, (cuuint32_t)box_h};
    cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapSwizzle sw = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                  : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                        : CU_TENSOR_MAP_SWIZZLE_NONE;
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, base, dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool smem_opt_in(const void *fn, size_t bytes, unsigned *done_mask)
{
    int dev = 0;
    cudaGetDevice(&dev);
    if (*done_mask >> (dev & 31) & 1)
        return true;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) !=
        cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    *done_mask |= 1u << (dev & 31);
    return true;
}

int gemm_status()
{
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_error, sizeof(int));
    if (v)
        cudaMemcpyToSymbol(g_error, &z, sizeof(int));
    return v;
}

}  // namespace tc

// Output tiles of 128 x bn for g.
static long tiles_for(const GemmArgs &g, int bn)
{
    long tm = cdiv(g.M, tc::BM);
    if (g.amode == 1) {
        const int tw = tc::conv_tile_width(g.cH, g.cW);
        tm = (long)cdiv(g.cW, tw) * cdiv(g.cH, tc::BM / tw);
    }
    return tm * cdiv(g.N, bn);
}

bool gemm_tc(cudaStream_t st, const GemmArgs &g, int sm_count)
{
    if (sm_count <= 0)
        sm_count = 148;
    if (g.ab != DT_BF16 || !g.transb || g.nb != 1)
        return false;
    const int ksz = g.cK ? g.cK : 3;
    if (g.amode == 2 ||
        (g.amode == 1 && ((ksz != 3 && ksz != 5) || g.cC % tc::BK || g.K != ksz * ksz * g.cC)))
        return false;
    if (g.M < 64 || g.N < 1 || g.K < 16)
        return false;
    if (((uintptr_t)g.A & 15) || ((uintptr_t)g.B & 15) ||
        (g.amode == 0 && (g.lda & 7)) || (g.ldb & 7))
        return false;
    // Large dense products without an activation: 256-row tiles, 256, 192
    // or 160 columns wide, whichever fills the rounds of tiles over the SMs
    // best, where that is at least 80 % (COREG_GEMM256=0 turns them off, for
    // comparison). With an activation the epilogue, which these tiles
    // cannot overlap with the next tile's products, costs more than the
    // wider tile saves (measured on the ViT's fc1).
    static const bool t256 = [] {
        const char *e = getenv("COREG_GEMM256");
        return !(e && e[0] == '0');
    }();
    if (t256 && g.amode == 0 && g.act == ACTF_NONE && g.N >= 512 && g.M >= 512 && g.K >= 256 &&
        ((uintptr_t)g.C & 15) == 0 && (g.ldc * (g.c == DT_BF16 ? 2 : 4)) % 16 == 0) {
        int best = 0;
        double best_u = 0.0;
        for (int bn : {256, 192, 160}) {
            const long tiles = (long)cdiv(g.M, 256) * cdiv(g.N, bn);
            const long rounds = (tiles + sm_count - 1) / sm_count;
            const double u = (double)tiles / (double)(rounds * sm_count);
            if (u > best_u + 1e-9) {
                best_u = u;
                best = bn;
            }
        }
        if (best_u >= 0.8) {
            if (best == 256 && tc::launch_tc2<256>(st, g, sm_count))
                return true;
            if (best == 192 && tc::launch_tc2<192>(st, g, sm_count))
                return true;
            if (best == 160 && tc::launch_tc2<160>(st, g, sm_count))
                return true;
        }
    }
    // Tile width by the rounds of tiles the persistent CTAs walk: a 128 x
    // 128 tile takes about half the time of a 128 x 256 one plus the
    // overhead of reading its operands twice as often (weighted 1.15).
    if (g.N >= 256) {
        const long r256 = (tiles_for(g, 256) + sm_count - 1) / sm_count;
        const long r128 = (tiles_for(g, 128) + sm_count - 1) / sm_count;
        if (r256 * 256 * 100 <= r128 * 128 * 115)
            return tc::launch_tc<256, 4>(st, g, sm_count);
    }
    // At most 16 columns: 32-wide tiles where the output takes the TMA-store
    // epilogue (16-byte aligned rows), else 16-wide ones.
    const int ces = g.c == DT_BF16 ? 2 : 4;
    if (g.N <= 16 && (((uintptr_t)g.C & 15) || (g.ldc * ces) % 16))
        return tc::launch_tc<16, 8>(st, g, sm_count);
    if (g.N <= 32)
        return tc::launch_tc<32, 8>(st, g, sm_count);
    if (g.N <= 64)
        return tc::launch_tc<64, 8>(st, g, sm_count);
    // 129 to 144 columns (DISK's last layer: 128 descriptor channels and
    // the heatmap) in one 144-wide tile rather than two of 128.
    if (g.N > 128 && g.N <= 144)
        return tc::launch_tc<144, 5>(st, g, sm_count);
    return tc::launch_tc<128, 6>(st, g, sm_count);
}

}  // namespace coreg
