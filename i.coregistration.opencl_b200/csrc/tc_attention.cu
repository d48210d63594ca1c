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
// One CTA per 128 queries of one head; keys in blocks of 128:
//   warp 0      TMA: Q once, K and V blocks into a ring of stages;
//   warp 1      tensor memory (512 columns: two 128-column score buffers
//               and the D-column output) and MMA issue: S(j) = Q K(j)^T
//               (K-major operands), O += P(j) V(j) (P from shared memory,
//               V as an MN-major operand), S computed two blocks ahead;
//   warps 2..5  softmax, one thread per query row: S(j) from TMEM, masked
//               keys, online maximum (O and the row sum rescaled in tensor
//               memory only when the maximum grows by more than 2^8, else
//               the stale maximum is kept), P(j) = exp2 as bfloat16 into
//               the 128-byte swizzled shared-memory tile of the second MMA;
//               at the end O / l to global memory.
// Every wait is bounded as in tc_gemm.cu.

#include <math.h>
#include <string.h>

#include "tc_common.cuh"

namespace coreg {
namespace tc {

namespace {

constexpr int BQ = 128, BKV = 128;

template <int D>
struct AttnCfg {
    static constexpr int KA = D / 64;            // 64-wide atoms along D
    static constexpr int ST = D == 64 ? 3 : 2;   // K / V stages
};

template <int D>
struct AttnSmem {
    static constexpr int KA = AttnCfg<D>::KA, ST = AttnCfg<D>::ST;
    alignas(1024) __nv_bfloat16 q[KA][BQ * 64];
    alignas(1024) __nv_bfloat16 k[ST][KA][BKV * 64];
    alignas(1024) __nv_bfloat16 v[ST][KA][BKV * 64];
    alignas(1024) __nv_bfloat16 p[2][BQ * 64];
    uint64_t q_full, kv_full[ST], kv_empty[ST], s_full[2], p_full, pv_done;
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

template <int D>
__global__ void __launch_bounds__(192, 1)
tc_attn_kernel(const __grid_constant__ CUtensorMap map, AttnParams p)
{
    constexpr int KA = AttnCfg<D>::KA, ST = AttnCfg<D>::ST;
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
        mbar_init(&s.p_full, 128);
        mbar_init(&s.pv_done, 1);
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
                if (!mbar_wait(&s.p_full, j & 1, 14))
                    break;
                fence_after();
                const int st = j % ST;
                const uint32_t vbase = su32(s.v[st][0]);
#pragma unroll
                for (int a = 0; a < 2; a++) {
                    const uint64_t dp = sw128_desc(su32(s.p[a]));
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
                mma_commit(&s.pv_done);
                mma_commit(&s.kv_empty[st]);
                if (j + 2 < nblk)
                    ok = issue_s(j + 2);
            }
        }
    }
    else {
        const int qd = warp % 4, r = 32 * qd + lane;
        const uint32_t lane_off = (uint32_t)(32 * qd) << 16;
        float m_used = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int j = 0; j < nblk; j++) {
            // Waits decided per warp, so that the warp-collective TMEM
            // accesses below never see a partial warp.
            if (!__all_sync(0xffffffffu, mbar_wait(&s.s_full[j & 1], (j >> 1) & 1, 15))) {
                ok = false;
                break;
            }
            fence_after();
            float sv[BKV];
#pragma unroll
            for (int c = 0; c < BKV / 32; c++)
                tmem_ld32(tmem + lane_off + (j & 1) * 128 + 32 * c, sv + 32 * c);
            const int kvalid = p.N - j * BKV;
            float mx = -INFINITY;
#pragma unroll
            for (int i = 0; i < BKV; i++) {
                sv[i] = i < kvalid ? sv[i] * p.scale_log2 : -INFINITY;
                mx = fmaxf(mx, sv[i]);
            }
            if (j > 0) {
                if (!__all_sync(0xffffffffu, mbar_wait(&s.pv_done, (j - 1) & 1, 16))) {
                    ok = false;
                    break;
                }
                fence_after();
            }
            const float m_new = fmaxf(m_used, mx);
            if (j == 0)
                m_used = m_new;
            else {
                // The tensor-memory loads and stores are warp-collective:
                // the whole warp rescales when one of its rows needs it,
                // the other rows by 1.
                const bool need = m_new > m_used + 8.0f;
                if (__any_sync(0xffffffffu, need)) {
                    const float corr = need ? exp2f(m_used - m_new) : 1.0f;
                    l *= corr;
#pragma unroll
                    for (int c = 0; c < D / 32; c++) {
                        float o[32];
                        tmem_ld32(tO + lane_off + 32 * c, o);
#pragma unroll
                        for (int i = 0; i < 32; i++)
                            o[i] *= corr;
                        tmem_st32(tO + lane_off + 32 * c, o);
                    }
                    if (need)
                        m_used = m_new;
                }
            }
            float sum = 0.0f;
#pragma unroll
            for (int a = 0; a < 2; a++) {
                unsigned char *row = (unsigned char *)s.p[a] + r * 128;
#pragma unroll
                for (int cc = 0; cc < 8; cc++) {
                    float e[8];
#pragma unroll
                    for (int t = 0; t < 8; t++) {
                        e[t] = exp2f(sv[a * 64 + cc * 8 + t] - m_used);
                        sum += e[t];
                    }
                    uint4 w;
                    w.x = pack_bf16(e[0], e[1]);
                    w.y = pack_bf16(e[2], e[3]);
                    w.z = pack_bf16(e[4], e[5]);
                    w.w = pack_bf16(e[6], e[7]);
                    *reinterpret_cast<uint4 *>(row + ((cc ^ (r & 7)) << 4)) = w;
                }
            }
            l += sum;
            fence_async_smem();
            fence_before();
            mbar_arrive(&s.p_full);
        }
        if (ok && __all_sync(0xffffffffu, mbar_wait(&s.pv_done, (nblk - 1) & 1, 17))) {
            fence_after();
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            const int q = q0 + r;
#pragma unroll
            for (int c = 0; c < D / 32; c++) {
                float o[32];
                tmem_ld32(tO + lane_off + 32 * c, o);
                if (q < p.N) {
                    uint4 *dst = reinterpret_cast<uint4 *>(p.out + img * p.out_img +
                                                           (long)q * p.ldo + h * D +
                                                           32 * c);
#pragma unroll
                    for (int t = 0; t < 4; t++) {
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
    }
    fence_before();
    __syncthreads();
    if (warp == 1) {
        fence_after();
        tmem_dealloc(tmem, 512);
    }
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
    tc_attn_kernel<D><<<dim3(cdiv(N, BQ), heads, nimg), 192, smem, st>>>(map, p);
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
        return tc::launch_attn<64>(st, qkv, N, Dm, heads, out, ldo, scale, nimg);
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
