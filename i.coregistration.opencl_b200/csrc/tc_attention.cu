// SPDX-License-Identifier: Unlicense
//
// Fused multi-head attention on tcgen05 tensor cores (sm_100a), never
// storing the score matrix: O = softmax(scale Q K^T) V per head for the
// transformer blocks of the models (the reference's attention(),
// roma.c:675-694, computes the full score matrices with two GEMMs and a
// row softmax). Operands come from the fused token-major qkv buffer
// (N x 3 Dm bfloat16: queries, keys, values, head h at columns h D of
// each), the output goes to the token-major (N x Dm) bfloat16 buffer.
//
// Head size 64 (DINOv2) runs tc_attn2_kernel below: two 128-query tiles
// per CTA with one softmax warpgroup each. Head size 128 (the RoMa decoder)
// runs tc_attn_kernel, one CTA per 128 queries of one head; keys in blocks
// of 128:
//   warp 0      TMA: Q once, K and V blocks into a ring of stages;
//   warp 1      tensor memory (512 columns: two 128-column score buffers
//               and the D-column output) and MMA issue: S(j) = Q K(j)^T
//               (K-major operands), O += P(j) V(j) (P from shared memory,
//               V as an MN-major operand), S computed two blocks ahead;
//   warps 2..17 softmax, four warps per query row: warp w takes the rows
//               of TMEM lane quadrant w % 4 and key quarter (w - 2) / 4 of
//               each block (32 keys) and the same quarter of O's columns.
//               S(j) from TMEM, masked keys, the row maximum of the four
//               quarters through shared memory (one barrier of the softmax
//               warps per block), online maximum (O and the row sum
//               rescaled in tensor memory only when the maximum grows by
//               more than 2^8, else the stale maximum is kept), P(j) = exp2
//               as bfloat16 into the 128-byte swizzled shared-memory tile
//               of the second MMA (two tiles when shared memory allows, so
//               that P(j) is written while the tensor cores read P(j - 1));
//               at the end
//               O / l to global memory. Four warps per scheduler, packed
//               float pairs and independent partial maxima and sums keep
//               the exponential unit busy.
// Every wait is bounded as in tc_gemm.cu.

#include <math.h>
#include <string.h>

#include "tc_common.cuh"

namespace coreg {
namespace tc {

namespace {

constexpr int BQ = 128, BKV = 128;
constexpr int SPLIT = 4;                       // softmax warps per query row
constexpr int SOFT_THREADS = 4 * SPLIT * 32;
constexpr int ATT_THREADS = 64 + SOFT_THREADS;  // TMA warp, MMA warp, softmax warps

template <int D>
struct AttnCfg {
    static constexpr int KA = D / 64;            // 64-wide atoms along D
    static constexpr int ST = D == 64 ? 3 : 2;   // K / V stages
    // P tiles: two for D 64, so that the softmax of block j writes P(j)
    // while the tensor cores still read P(j - 1); one for D 128 (shared
    // memory).
    static constexpr int PB = D == 64 ? 2 : 1;
};

template <int D>
struct AttnSmem {
    static constexpr int KA = AttnCfg<D>::KA, ST = AttnCfg<D>::ST, PB = AttnCfg<D>::PB;
    alignas(1024) __nv_bfloat16 q[KA][BQ * 64];
    alignas(1024) __nv_bfloat16 k[ST][KA][BKV * 64];
    alignas(1024) __nv_bfloat16 v[ST][KA][BKV * 64];
    alignas(1024) __nv_bfloat16 p[PB][2][BQ * 64];
    float red[2][SPLIT][BQ];  // per block parity and key quarter: row maxima, then sums
    // Softmax abort flags by block parity: a failed wait in block j sets
    // abort[j % 2] before the block's barrier, or abort[(j + 1) % 2] after
    // it; every softmax warp reads abort[j % 2] after barrier j.
    int abort[2];
    // p_full and pv_done per P tile: the softmax may finish block j + 1
    // before the MMA warp has seen block j, so one barrier for both would
    // run two phases ahead of its waiter.
    uint64_t q_full, kv_full[ST], kv_empty[ST], s_full[2], p_full[PB], pv_done[PB];
    uint32_t tmem;
};

struct AttnParams {
    int N, Dm;
    __nv_bfloat16 *out;
    long ldo, out_img;  // output row pitch; elements between images
    float scale_log2;
};

__device__ __forceinline__ uint32_t pack_bf16(float a, float b)
{
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

// Packed float32 pairs (sm_100a): one instruction for both values.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c)
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

__device__ __forceinline__ float2 fadd2(float2 a, float2 b)
{
    unsigned long long aa, bb, dd;
    asm("mov.b64 %0, {%1, %2};" : "=l"(aa) : "f"(a.x), "f"(a.y));
    asm("mov.b64 %0, {%1, %2};" : "=l"(bb) : "f"(b.x), "f"(b.y));
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(dd) : "l"(aa), "l"(bb));
    float2 d;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(dd));
    return d;
}

// The hardware base-2 exponential (results below 2^-126 flush to zero,
// negligible next to the row maximum's 1).
__device__ __forceinline__ float ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int D>
__global__ void __launch_bounds__(ATT_THREADS, 1)
tc_attn_kernel(const __grid_constant__ CUtensorMap map, AttnParams p)
{
    constexpr int KA = AttnCfg<D>::KA, ST = AttnCfg<D>::ST, PB = AttnCfg<D>::PB;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    AttnSmem<D> &s = *reinterpret_cast<AttnSmem<D> *>(
        (void *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023));
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int q0 = blockIdx.x * BQ, h = blockIdx.y, img = blockIdx.z;
    const int nblk = (p.N + BKV - 1) / BKV;

    if (threadIdx.x == 0) {
        mbar_init(&s.q_full, 1);
        for (int i = 0; i < ST; i++) {
            mbar_init(&s.kv_full[i], 1);
            mbar_init(&s.kv_empty[i], 1);
        }
        mbar_init(&s.s_full[0], 1);
        mbar_init(&s.s_full[1], 1);
        for (int i = 0; i < PB; i++)
            mbar_init(&s.p_full[i], SOFT_THREADS);
        for (int i = 0; i < PB; i++)
            mbar_init(&s.pv_done[i], 1);
        s.abort[0] = s.abort[1] = 0;
        mbar_fence_init();
    }
    if (warp == 1)
        tmem_alloc(&s.tmem, 512);
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = s.tmem;
    const uint32_t tO = tmem + 256;

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t tile = BQ * 64 * 2;
            mbar_expect_tx(&s.q_full, KA * tile);
            for (int a = 0; a < KA; a++)
                tma_load_3d(s.q[a], &map, &s.q_full, h * D + a * 64, q0, img);
            for (int j = 0; j < nblk; j++) {
                const int st = j % ST;
                if (j >= ST && !mbar_wait(&s.kv_empty[st], ((j / ST) - 1) & 1, 11))
                    break;
                mbar_expect_tx(&s.kv_full[st], 2 * KA * tile);
                for (int a = 0; a < KA; a++) {
                    tma_load_3d(s.k[st][a], &map, &s.kv_full[st], p.Dm + h * D + a * 64,
                                j * BKV, img);
                    tma_load_3d(s.v[st][a], &map, &s.kv_full[st], 2 * p.Dm + h * D + a * 64,
                                j * BKV, img);
                }
            }
        }
    }
    else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t id_s = idesc_bf16(BQ, BKV, 0);
            constexpr uint32_t id_o = idesc_bf16(BQ, D, 1);
            bool ok = mbar_wait(&s.q_full, 0, 12);
            auto issue_s = [&](int j) -> bool {
                const int st = j % ST;
                if (!mbar_wait(&s.kv_full[st], (j / ST) & 1, 13))
                    return false;
                fence_after();
                const uint32_t tS = tmem + (j & 1) * 128;
#pragma unroll
                for (int a = 0; a < KA; a++) {
                    const uint64_t dq = sw128_desc(su32(s.q[a]));
                    const uint64_t dk = sw128_desc(su32(s.k[st][a]));
#pragma unroll
                    for (int k = 0; k < 4; k++)
                        mma_bf16(tS, dq + 2 * k, dk + 2 * k, id_s, (a | k) ? 1u : 0u);
                }
                mma_commit(&s.s_full[j & 1]);
                return true;
            };
            if (ok)
                ok = issue_s(0) && (nblk < 2 || issue_s(1));
            for (int j = 0; j < nblk && ok; j++) {
                if (!mbar_wait(&s.p_full[j % PB], (j / PB) & 1, 14))
                    break;
                fence_after();
                const int st = j % ST;
                const uint32_t vbase = su32(s.v[st][0]);
#pragma unroll
                for (int a = 0; a < 2; a++) {
                    const uint64_t dp = sw128_desc(su32(s.p[j % PB][a]));
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        // 16 keys from key a 64 + 16 k: V rows of 128 bytes,
                        // 64-wide D groups BKV * 128 bytes apart.
                        const uint64_t dv =
                            sw128_desc(vbase + (uint32_t)(a * 64 + k * 16) * 128,
                                       BKV * 128, 1024);
                        mma_bf16(tO, dp + 2 * k, dv, id_o, (j | a | k) ? 1u : 0u);
                    }
                }
                mma_commit(&s.pv_done[j % PB]);
                mma_commit(&s.kv_empty[st]);
                if (j + 2 < nblk)
                    ok = issue_s(j + 2);
            }
        }
    }
    else {
        constexpr int KW = BKV / SPLIT, OW = D / SPLIT;  // keys and O columns per warp
        const int qd = warp % 4, part = (warp - 2) / 4, r = 32 * qd + lane;
        const uint32_t lane_off = (uint32_t)(32 * qd) << 16;
        float m_used = -INFINITY, l = 0.0f;
        bool ok = true;
        // O columns of this warp: load, store.
        auto o_ld = [&](float *o) {
            if (OW == 16)
                tmem_ld16(tO + lane_off + OW * part, o);
            else
                tmem_ld32(tO + lane_off + OW * part, o);
        };
        auto o_st = [&](const float *o) {
            if (OW == 16)
                tmem_st16(tO + lane_off + OW * part, o);
            else
                tmem_st32(tO + lane_off + OW * part, o);
        };
        for (int j = 0; j < nblk; j++) {
            // Waits decided per warp, so that the warp-collective TMEM
            // accesses below never see a partial warp.
            const bool sok = __all_sync(0xffffffffu, mbar_wait(&s.s_full[j & 1], (j >> 1) & 1, 15));
            if (!sok && lane == 0)
                s.abort[j & 1] = 1;
            float sv[KW];
            float mx = -INFINITY;
            if (sok) {
                fence_after();
                tmem_ld32(tmem + lane_off + (j & 1) * 128 + KW * part, sv);
                const int kvalid = p.N - j * BKV - KW * part;
                if (kvalid < KW) {
#pragma unroll
                    for (int i = 0; i < KW; i++)
                        if (i >= kvalid)
                            sv[i] = -INFINITY;
                }
                float m8[8];
#pragma unroll
                for (int t = 0; t < 8; t++)
                    m8[t] = sv[t];
#pragma unroll
                for (int i = 8; i < KW; i++)
                    m8[i & 7] = fmaxf(m8[i & 7], sv[i]);
#pragma unroll
                for (int t = 0; t < 4; t++)
                    m8[t] = fmaxf(m8[t], m8[t + 4]);
                mx = fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3]));
            }
            // The quarters' maxima (raw scores; the scale is positive).
            s.red[j & 1][part][r] = mx;
            named_bar(1, SOFT_THREADS);
            if (s.abort[j & 1]) {
                ok = false;
                break;
            }
#pragma unroll
            for (int o = 1; o < SPLIT; o++)
                mx = fmaxf(mx, s.red[j & 1][(part + o) % SPLIT][r]);
            mx *= p.scale_log2;
            // PV(i) has completed (pv_done[i % PB] phase i / PB).
            auto pv_wait = [&](int i) {
                return __all_sync(0xffffffffu, mbar_wait(&s.pv_done[i % PB], (i / PB) & 1, 16));
            };
            const float m_new = fmaxf(m_used, mx);
            // The tensor-memory loads and stores are warp-collective: the
            // whole warp rescales when one of its rows needs it, the other
            // rows by 1. The warps of a row decide alike.
            const bool need = j > 0 && m_new > m_used + 8.0f;
            const bool rescale = __any_sync(0xffffffffu, need);
            // O is final up to PV(j - 1) before a rescale; P(j)'s tiles are
            // free once PV(j - PB) has read them.
            if ((rescale && !pv_wait(j - 1)) || (j >= PB && !pv_wait(j - PB))) {
                ok = false;
                if (lane == 0)
                    s.abort[(j + 1) & 1] = 1;
                continue;
            }
            fence_after();
            if (j == 0)
                m_used = m_new;
            else if (rescale) {
                const float corr = need ? exp2f(m_used - m_new) : 1.0f;
                l *= corr;
                float o[OW];
                o_ld(o);
#pragma unroll
                for (int i = 0; i < OW; i++)
                    o[i] *= corr;
                o_st(o);
                if (need)
                    m_used = m_new;
            }
            float2 s4[4];
#pragma unroll
            for (int t = 0; t < 4; t++)
                s4[t] = make_float2(0.0f, 0.0f);
            const float2 sc = make_float2(p.scale_log2, p.scale_log2);
            const float2 mm = make_float2(-m_used, -m_used);
            // Keys KW part .. of the block: 64-key tile part / 2, 16-byte
            // chunks from 4 (part % 2).
            unsigned char *row = (unsigned char *)s.p[j % PB][part >> 1] + r * 128;
#pragma unroll
            for (int cc = 0; cc < KW / 8; cc++) {
                float e[8];
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const float2 a =
                        ffma2(make_float2(sv[cc * 8 + 2 * t], sv[cc * 8 + 2 * t + 1]), sc, mm);
                    e[2 * t] = ex2(a.x);
                    e[2 * t + 1] = ex2(a.y);
                    s4[t] = fadd2(s4[t], make_float2(e[2 * t], e[2 * t + 1]));
                }
                uint4 w;
                w.x = pack_bf16(e[0], e[1]);
                w.y = pack_bf16(e[2], e[3]);
                w.z = pack_bf16(e[4], e[5]);
                w.w = pack_bf16(e[6], e[7]);
                const int chunk = 4 * (part & 1) + cc;
                *reinterpret_cast<uint4 *>(row + ((chunk ^ (r & 7)) << 4)) = w;
            }
            const float2 s2 = fadd2(fadd2(s4[0], s4[1]), fadd2(s4[2], s4[3]));
            l += s2.x + s2.y;
            fence_async_smem();
            fence_before();
            mbar_arrive(&s.p_full[j % PB]);
        }
        if (ok && __all_sync(0xffffffffu, mbar_wait(&s.pv_done[(nblk - 1) % PB],
                                                    ((nblk - 1) / PB) & 1, 17)))
            fence_after();
        else
            ok = false;
        // Row sums of the quarters (added in one order by every warp of a
        // row); every softmax warp reaches this barrier.
        s.red[nblk & 1][part][r] = l;
        named_bar(1, SOFT_THREADS);
        if (__all_sync(0xffffffffu, ok)) {
            l = 0.0f;
#pragma unroll
            for (int o = 0; o < SPLIT; o++)
                l += s.red[nblk & 1][o][r];
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            const int q = q0 + r;
            float o[OW];
            o_ld(o);
            if (q < p.N) {
                uint4 *dst = reinterpret_cast<uint4 *>(p.out + img * p.out_img + (long)q * p.ldo +
                                                       h * D + OW * part);
#pragma unroll
                for (int t = 0; t < OW / 8; t++) {
                    uint4 w;
                    w.x = pack_bf16(o[8 * t] * inv, o[8 * t + 1] * inv);
                    w.y = pack_bf16(o[8 * t + 2] * inv, o[8 * t + 3] * inv);
                    w.z = pack_bf16(o[8 * t + 4] * inv, o[8 * t + 5] * inv);
                    w.w = pack_bf16(o[8 * t + 6] * inv, o[8 * t + 7] * inv);
                    dst[t] = w;
                }
            }
        }
    }
    fence_before();
    __syncthreads();
    if (warp == 1) {
        fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------- two tiles
//
// Head size 64: one CTA per 256 queries (two 128-query tiles t = 0, 1) of
// one head. Each tile has its own softmax warpgroup, one thread per query
// row with the block's 128 scores in registers, so that no warps exchange
// row maxima; the two groups drift half a block apart, and while one
// exponentiates (the exponential unit is the bound) the other loads and
// reduces its scores and the tensor cores work for both.
//   warp 0      TMA: both Q tiles once, K and V blocks into a ring;
//   warp 1      tensor memory (S_t: 128 columns at 128 t, O_t: 64 at
//               256 + 64 t) and MMA issue, per block j in the order the
//               groups get there: S_0(j + 1) once softmax 0 has read S_0(j)
//               (s_free), S_1(j + 1) likewise, PV_0(j) once P_0(j) is in
//               shared memory (p_full), PV_1(j);
//   warps 2..5  softmax of tile 0, warps 6..9 of tile 1: S_t(j) from
//               tensor memory, masked keys, online maximum (O_t and the row
//               sum rescaled in tensor memory only when the maximum grows
//               by more than 2^8), P_t(j) = exp2 as bfloat16 into the tile's
//               128-byte swizzled P buffer (free once PV_t(j - 1) is done);
//               at the end O_t / l to global memory.
constexpr int ATT2_THREADS = 320;

struct Attn2Smem {
    alignas(1024) __nv_bfloat16 q[2][BQ * 64];
    alignas(1024) __nv_bfloat16 k[3][BKV * 64];
    alignas(1024) __nv_bfloat16 v[3][BKV * 64];
    alignas(1024) __nv_bfloat16 p[2][2][BQ * 64];  // tile, 64-key half
    uint64_t q_full, kv_full[3], kv_empty[3], s_full[2], s_free[2], p_full[2], pv_done[2];
    uint32_t tmem;
};

__global__ void __launch_bounds__(ATT2_THREADS, 1)
tc_attn2_kernel(const __grid_constant__ CUtensorMap map, AttnParams p)
{
    constexpr int ST = 3;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    Attn2Smem &s = *reinterpret_cast<Attn2Smem *>(smem_raw +
                                                  ((1024u - (su32(smem_raw) & 1023u)) & 1023u));
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int q0 = blockIdx.x * 2 * BQ, h = blockIdx.y, img = blockIdx.z;
    const int nblk = (p.N + BKV - 1) / BKV;

    if (threadIdx.x == 0) {
        mbar_init(&s.q_full, 1);
        for (int i = 0; i < ST; i++) {
            mbar_init(&s.kv_full[i], 1);
            mbar_init(&s.kv_empty[i], 1);
        }
        for (int t = 0; t < 2; t++) {
            mbar_init(&s.s_full[t], 1);
            mbar_init(&s.s_free[t], 4);
            mbar_init(&s.p_full[t], 128);
            mbar_init(&s.pv_done[t], 1);
        }
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
            const uint32_t tile = BQ * 64 * 2;
            mbar_expect_tx(&s.q_full, 2 * tile);
            for (int t = 0; t < 2; t++)
                tma_load_3d(s.q[t], &map, &s.q_full, h * 64, q0 + t * BQ, img);
            for (int j = 0; j < nblk; j++) {
                const int st = j % ST;
                if (j >= ST && !mbar_wait(&s.kv_empty[st], ((j / ST) - 1) & 1, 11))
                    break;
                mbar_expect_tx(&s.kv_full[st], 2 * tile);
                tma_load_3d(s.k[st], &map, &s.kv_full[st], p.Dm + h * 64, j * BKV, img);
                tma_load_3d(s.v[st], &map, &s.kv_full[st], 2 * p.Dm + h * 64, j * BKV, img);
            }
        }
    }
    else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t id_s = idesc_bf16(BQ, BKV, 0);
            constexpr uint32_t id_o = idesc_bf16(BQ, 64, 1);
            bool ok = mbar_wait(&s.q_full, 0, 12);
            // S_t(j) = Q_t K(j)^T once softmax t has read S_t(j - 1).
            auto issue_s = [&](int t, int j) -> bool {
                const int st = j % ST;
                if (t == 0 && !mbar_wait(&s.kv_full[st], (j / ST) & 1, 13))
                    return false;
                if (j > 0 && !mbar_wait(&s.s_free[t], (j - 1) & 1, 18))
                    return false;
                fence_after();
                const uint64_t dq = sw128_desc(su32(s.q[t]));
                const uint64_t dk = sw128_desc(su32(s.k[st]));
#pragma unroll
                for (int k = 0; k < 4; k++)
                    mma_bf16(tmem + 128 * t, dq + 2 * k, dk + 2 * k, id_s, k ? 1u : 0u);
                mma_commit(&s.s_full[t]);
                return true;
            };
            // O_t += P_t(j) V(j) once P_t(j) is in shared memory.
            auto issue_pv = [&](int t, int j) -> bool {
                if (!mbar_wait(&s.p_full[t], j & 1, 14))
                    return false;
                fence_after();
                const uint32_t vbase = su32(s.v[j % ST]);
#pragma unroll
                for (int a = 0; a < 2; a++) {
                    const uint64_t dp = sw128_desc(su32(s.p[t][a]));
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        // 16 keys from key a 64 + 16 k: V rows of 128 bytes.
                        const uint64_t dv =
                            sw128_desc(vbase + (uint32_t)(a * 64 + k * 16) * 128, BKV * 128, 1024);
                        mma_bf16(tmem + 256 + 64 * t, dp + 2 * k, dv, id_o,
                                 (j | a | k) ? 1u : 0u);
                    }
                }
                mma_commit(&s.pv_done[t]);
                return true;
            };
            if (ok)
                ok = issue_s(0, 0) && issue_s(1, 0);
            for (int j = 0; j < nblk && ok; j++) {
                if (j + 1 < nblk)
                    ok = issue_s(0, j + 1) && issue_s(1, j + 1);
                ok = ok && issue_pv(0, j) && issue_pv(1, j);
                if (ok)
                    mma_commit(&s.kv_empty[j % ST]);
            }
        }
    }
    else {
        const int t = (warp - 2) / 4, qd = warp % 4, r = 32 * qd + lane;
        const uint32_t lane_off = (uint32_t)(32 * qd) << 16;
        const uint32_t tS = tmem + lane_off + 128 * t, tO = tmem + lane_off + 256 + 64 * t;
        float m_used = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int j = 0; j < nblk; j++) {
            // Waits decided per warp: the TMEM accesses are warp-collective.
            if (!__all_sync(0xffffffffu, mbar_wait(&s.s_full[t], j & 1, 15))) {
                ok = false;
                break;
            }
            fence_after();
            float sv[BKV];
#pragma unroll
            for (int c = 0; c < BKV / 32; c++)
                tmem_ld32(tS + 32 * c, sv + 32 * c);
            // S_t's columns are free for S_t(j + 1).
            fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(&s.s_free[t]);
            const int kvalid = p.N - j * BKV;
            if (kvalid < BKV) {
#pragma unroll
                for (int i = 0; i < BKV; i++)
                    if (i >= kvalid)
                        sv[i] = -INFINITY;
            }
            float m4[4];
#pragma unroll
            for (int i = 0; i < 4; i++)
                m4[i] = sv[i];
#pragma unroll
            for (int i = 4; i < BKV; i++)
                m4[i & 3] = fmaxf(m4[i & 3], sv[i]);
            const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * p.scale_log2;
            const float m_new = fmaxf(m_used, mx);
            const bool need = j > 0 && m_new > m_used + 8.0f;
            const bool rescale = __any_sync(0xffffffffu, need);
            // PV_t(j - 1) is done: O_t final up to block j - 1, the P
            // buffer free.
            if (j > 0 && !__all_sync(0xffffffffu, mbar_wait(&s.pv_done[t], (j - 1) & 1, 16))) {
                ok = false;
                break;
            }
            fence_after();
            if (j == 0)
                m_used = m_new;
            else if (rescale) {
                // The whole warp rescales (warp-collective TMEM access),
                // the rows that keep their maximum by 1.
                const float corr = need ? exp2f(m_used - m_new) : 1.0f;
                l *= corr;
#pragma unroll 1
                for (int c = 0; c < 4; c++) {
                    float o[16];
                    tmem_ld16(tO + 16 * c, o);
#pragma unroll
                    for (int i = 0; i < 16; i++)
                        o[i] *= corr;
                    tmem_st16(tO + 16 * c, o);
                }
                if (need)
                    m_used = m_new;
            }
            float2 s2 = make_float2(0.0f, 0.0f);
            const float2 sc = make_float2(p.scale_log2, p.scale_log2);
            const float2 mm = make_float2(-m_used, -m_used);
#pragma unroll
            for (int a = 0; a < 2; a++) {
                unsigned char *row = (unsigned char *)s.p[t][a] + r * 128;
#pragma unroll
                for (int cc = 0; cc < 8; cc++) {
                    float e[8];
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int i = a * 64 + cc * 8 + 2 * u;
                        const float2 x = ffma2(make_float2(sv[i], sv[i + 1]), sc, mm);
                        e[2 * u] = ex2(x.x);
                        e[2 * u + 1] = ex2(x.y);
                        s2 = fadd2(s2, make_float2(e[2 * u], e[2 * u + 1]));
                    }
                    uint4 w;
                    w.x = pack_bf16(e[0], e[1]);
                    w.y = pack_bf16(e[2], e[3]);
                    w.z = pack_bf16(e[4], e[5]);
                    w.w = pack_bf16(e[6], e[7]);
                    *reinterpret_cast<uint4 *>(row + ((cc ^ (r & 7)) << 4)) = w;
                }
            }
            l += s2.x + s2.y;
            fence_async_smem();
            fence_before();
            mbar_arrive(&s.p_full[t]);
        }
        if (ok && __all_sync(0xffffffffu, mbar_wait(&s.pv_done[t], (nblk - 1) & 1, 17))) {
            fence_after();
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            const int q = q0 + t * BQ + r;
#pragma unroll 1
            for (int c = 0; c < 4; c++) {
                float o[16];
                tmem_ld16(tO + 16 * c, o);
                if (q < p.N) {
                    uint4 *dst = reinterpret_cast<uint4 *>(p.out + img * p.out_img +
                                                           (long)q * p.ldo + h * 64 + 16 * c);
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        uint4 w;
                        w.x = pack_bf16(o[8 * u] * inv, o[8 * u + 1] * inv);
                        w.y = pack_bf16(o[8 * u + 2] * inv, o[8 * u + 3] * inv);
                        w.z = pack_bf16(o[8 * u + 4] * inv, o[8 * u + 5] * inv);
                        w.w = pack_bf16(o[8 * u + 6] * inv, o[8 * u + 7] * inv);
                        dst[u] = w;
                    }
                }
            }
        }
    }
    fence_before();
    __syncthreads();
    if (warp == 1) {
        fence_after();
        tmem_dealloc(tmem, 512);
    }
}

bool launch_attn2(cudaStream_t st, const void *qkv, int N, int Dm, int heads, void *out,
                  long ldo, float scale, int nimg)
{
    CUtensorMap map;
    if (!make_map_conv(&map, qkv, nimg, N, 3 * Dm, BQ, 1))
        return false;
    AttnParams p;
    p.N = N;
    p.Dm = Dm;
    p.out = (__nv_bfloat16 *)out;
    p.ldo = ldo;
    p.out_img = (long)N * ldo;
    p.scale_log2 = scale * 1.4426950408889634f;
    const size_t smem = sizeof(Attn2Smem) + 1024;
    static unsigned done = 0;
    if (!smem_opt_in((const void *)tc_attn2_kernel, smem, &done))
        return false;
    tc_attn2_kernel<<<dim3(cdiv(N, 2 * BQ), heads, nimg), ATT2_THREADS, smem, st>>>(map, p);
    return true;
}

template <int D>
bool launch_attn(cudaStream_t st, const void *qkv, int N, int Dm, int heads, void *out,
                 long ldo, float scale, int nimg)
{
    // (columns, rows, image) over nimg row blocks of N: boxes of 64
    // columns x BQ rows of one image, zeros past its last row.
    CUtensorMap map;
    if (!make_map_conv(&map, qkv, nimg, N, 3 * Dm, BQ, 1))
        return false;
    AttnParams p;
    p.N = N;
    p.Dm = Dm;
    p.out = (__nv_bfloat16 *)out;
    p.ldo = ldo;
    p.out_img = (long)N * ldo;
    p.scale_log2 = scale * 1.4426950408889634f;
    const size_t smem = sizeof(AttnSmem<D>) + 1024;
    static unsigned done = 0;
    if (!smem_opt_in((const void *)tc_attn_kernel<D>, smem, &done))
        return false;
    tc_attn_kernel<D><<<dim3(cdiv(N, BQ), heads, nimg), ATT_THREADS, smem, st>>>(map, p);
    return true;
}

int attn_status()
{
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_error, sizeof(int));
    if (v)
        cudaMemcpyToSymbol(g_error, &z, sizeof(int));
    return v;
}

}  // namespace

int gemm_status();
int dwpw_status();

}  // namespace tc

// Attention of the fused qkv buffer on tensor cores; false (nothing
// launched) when the head size or alignment is not supported.
bool attention_tc(cudaStream_t st, const void *qkv, int N, int Dm, int heads, void *out,
                  long ldo, float scale, int nimg)
{
    const int d = Dm / heads;
    if (N < 1 || nimg < 1 || nimg > 65535 || d * heads != Dm || ((uintptr_t)qkv & 15) || ((uintptr_t)out & 15) ||
        (ldo & 7) || (Dm & 63))
        return false;
    if (d == 64)
        return tc::launch_attn2(st, qkv, N, Dm, heads, out, ldo, scale, nimg);
    if (d == 128)
        return tc::launch_attn<128>(st, qkv, N, Dm, heads, out, ldo, scale, nimg);
    return false;
}

}  // namespace coreg

extern "C" int coreg_tc_status(void)
{
    const int a = coreg::tc::gemm_status();
    const int b = coreg::tc::attn_status();
    const int c = coreg::tc::dwpw_status();
    return a ? a : b ? b : c;
}
