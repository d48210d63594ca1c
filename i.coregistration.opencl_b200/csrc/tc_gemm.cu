// SPDX-License-Identifier: Unlicense
//
// tcgen05 tensor-core GEMM for sm_100a: C = act(alpha A B^T + bias) + R
// with A (M x K) and B (N x K) bfloat16, K-major (row-major with K
// contiguous), float32 accumulation in tensor memory, float32 or
// bfloat16 C. The GemmArgs contract of gemm.cuh (one product, column
// bias).
//
// One CTA per 128 x BN output tile, warp-specialized:
//   warp 0      TMA producer: A and B tiles of 64 K-elements per stage,
//               128-byte swizzled, into a ring of STAGES shared-memory
//               stages (mbarrier full[s], transaction bytes);
//   warp 1      tensor-memory allocator and MMA issuer: one elected thread
//               issues 4 tcgen05.mma (K = 16 each) per stage into a
//               128 x BN float32 accumulator in TMEM and commits each
//               stage to empty[s] (the producer's refill signal), the last
//               one to done;
//   warps 2..5  epilogue: wait on done, tcgen05.ld 32 columns at a time
//               (warp w reads TMEM lanes 32 (w % 4) ..), bias, activation,
//               residual, store.
// Every mbarrier wait is bounded (about two seconds of global time); a
// wait that runs out records an error code that gemm_tc_status reports,
// and the CTA leaves the loops, frees its tensor memory and returns.

#include <cuda.h>
#include <mutex>
#include <string.h>

#include "gemm.cuh"

namespace coreg {

namespace {

constexpr int BM = 128, BK = 64;
constexpr int NTHREADS = 192;

__device__ int g_tc_error = 0;

__device__ __forceinline__ uint32_t su32(const void *p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t gtime()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t *b, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(su32(b)), "r"(parity)
                 : "memory");
    return ok != 0;
}

// Bounded wait for the phase of the given parity to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, int code)
{
    if (mbar_try(b, parity))
        return true;
    const uint64_t t0 = gtime();
    while (!mbar_try(b, parity)) {
        if (gtime() - t0 > 2000000000ull) {
            atomicCAS(&g_tc_error, 0, code);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map,
                                            uint64_t *bar, int x, int y)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4}], [%2];" ::"r"(su32(dst)),
                 "l"((uint64_t)map), "r"(su32(bar)), "r"(x), "r"(y)
                 : "memory");
}

// 3-D box (innermost coordinate x first); coordinates outside the tensor
// (negative ones included) read zeros.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map,
                                            uint64_t *bar, int x, int y, int z)
{
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(su32(dst)),
                 "l"((uint64_t)map), "r"(su32(bar)), "r"(x), "r"(y), "r"(z)
                 : "memory");
}

// Shared-memory matrix descriptor of a K-major tile with 128-byte
// swizzling: rows of 128 bytes, 8-row groups 1024 bytes apart (SBO);
// version 1 (tcgen05), layout type 2 (SWIZZLE_128B).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr)
{
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFF) >> 4);
    d |= (uint64_t)(16 >> 4) << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor: kind::f16 with bfloat16 A and B, float32 D,
// both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem, uint64_t da, uint64_t db,
                                         uint32_t idesc, uint32_t accum)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
                 "l"(da), "l"(db), "r"(idesc), "r"(accum));
}

__device__ __forceinline__ void mma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     su32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float v[32])
{
    uint32_t r[32];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                   "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
                   "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                   "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]),
                   "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++)
        v[i] = __uint_as_float(r[i]);
}

struct TcParams {
    int M, N, K;
    void *C;
    long ldc;
    const float *bias;
    const void *R;
    float alpha;
    int act;
    float slope;
    int c_bf16;
    // Convolution mode (3 x 3, stride 1, padding 1, channels-last input of
    // cH x cW x cC, cC a multiple of 64): the tile is TW x TH output pixels
    // (TW TH = 128), k-block kb = (tap, 64-channel chunk).
    int conv, cH, cW, cC, TW, TH, tiles_x;
};

template <int BN, int STAGES>
struct Smem {
    alignas(1024) __nv_bfloat16 a[STAGES][BM * BK];
    alignas(1024) __nv_bfloat16 b[STAGES][BN * BK];
    uint64_t full[STAGES], empty[STAGES], done;
    uint32_t tmem;
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(NTHREADS, 1)
tc_gemm_kernel(const __grid_constant__ CUtensorMap tma_a,
               const __grid_constant__ CUtensorMap tma_b, TcParams p)
{
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // 1024-byte alignment of the swizzled stages.
    Smem<BN, STAGES> &s = *reinterpret_cast<Smem<BN, STAGES> *>(
        (void *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023));
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int nk = (p.K + BK - 1) / BK;
    // Convolution tile origin (pixels x0 .., rows y0 ..).
    const int cx0 = p.conv ? (blockIdx.y % p.tiles_x) * p.TW : 0;
    const int cy0 = p.conv ? (blockIdx.y / p.tiles_x) * p.TH : 0;

    if (threadIdx.x == 0) {
        for (int i = 0; i < STAGES; i++) {
            mbar_init(&s.full[i], 1);
            mbar_init(&s.empty[i], 1);
        }
        mbar_init(&s.done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         su32(&s.tmem)),
                     "r"(BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = s.tmem;

    if (warp == 0) {
        if (lane == 0) {
            const uint32_t bytes = (BM + BN) * BK * 2;
            for (int kb = 0; kb < nk; kb++) {
                const int st = kb % STAGES;
                if (kb >= STAGES &&
                    !mbar_wait(&s.empty[st], ((kb / STAGES) - 1) & 1, 1))
                    break;
                mbar_expect_tx(&s.full[st], bytes);
                if (p.conv) {
                    const int chunks = p.cC / BK, tap = kb / chunks;
                    const int c0 = (kb % chunks) * BK;
                    tma_load_3d(s.a[st], &tma_a, &s.full[st], c0, cx0 + tap % 3 - 1,
                                cy0 + tap / 3 - 1);
                }
                else
                    tma_load_2d(s.a[st], &tma_a, &s.full[st], kb * BK, m0);
                tma_load_2d(s.b[st], &tma_b, &s.full[st], kb * BK, n0);
            }
        }
    }
    else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16(BM, BN);
            bool ok = true;
            for (int kb = 0; kb < nk && ok; kb++) {
                const int st = kb % STAGES;
                if (!mbar_wait(&s.full[st], (kb / STAGES) & 1, 2)) {
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint64_t da = sw128_desc(su32(s.a[st]));
                const uint64_t db = sw128_desc(su32(s.b[st]));
#pragma unroll
                for (int k = 0; k < BK / 16; k++)
                    mma_bf16(tmem, da + 2 * k, db + 2 * k, idesc,
                             (kb > 0 || k > 0) ? 1u : 0u);
                mma_commit(&s.empty[st]);
            }
            mma_commit(&s.done);
        }
    }
    else {
        // Epilogue: warp w owns TMEM lanes (rows) 32 (w % 4) ...
        const int q = warp % 4;
        const int r = 32 * q + lane;
        int row = m0 + r;
        if (p.conv) {
            const int px = cx0 + r % p.TW, py = cy0 + r / p.TW;
            row = px < p.cW && py < p.cH ? py * p.cW + px : p.M;
        }
        if (mbar_wait(&s.done, 0, 3)) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            for (int c0 = 0; c0 < BN; c0 += 32) {
                float v[32];
                tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + c0, v);
                if (row >= p.M)
                    continue;
                const long base = (long)row * p.ldc;
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    const int col = n0 + c0 + j;
                    if (col >= p.N)
                        break;
                    float x = p.alpha * v[j];
                    if (p.bias)
                        x += p.bias[col];
                    x = apply_act(x, p.act, p.slope);
                    if (p.c_bf16) {
                        __nv_bfloat16 *C = (__nv_bfloat16 *)p.C + base + col;
                        if (p.R)
                            x += __bfloat162float(((const __nv_bfloat16 *)p.R)[base + col]);
                        *C = __float2bfloat16_rn(x);
                    }
                    else {
                        float *C = (float *)p.C + base + col;
                        if (p.R)
                            x += ((const float *)p.R)[base + col];
                        *C = x;
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(BN));
    }
}

// ------------------------------------------------------------- host side

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

// 2-D bfloat16 tensor map of a rows x cols row-major matrix (leading
// dimension ld elements), box of box_rows x 64, 128-byte swizzle, zero
// fill outside.
bool make_map(CUtensorMap *map, const void *base, long rows, long cols, long ld,
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

// 3-D bfloat16 tensor map of a channels-last (H, W, C) image, box of TH
// rows x TW pixels x 64 channels, 128-byte swizzle, zero fill outside.
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

template <int BN, int STAGES>
bool launch_tc(cudaStream_t st, const GemmArgs &g)
{
    CUtensorMap ma, mb;
    TcParams p;
    memset(&p, 0, sizeof(p));
    int grid_y = cdiv(g.M, BM);
    if (g.amode == 1) {
        p.conv = 1;
        p.cH = g.cH;
        p.cW = g.cW;
        p.cC = g.cC;
        p.TW = conv_tile_width(g.cH, g.cW);
        p.TH = BM / p.TW;
        p.tiles_x = cdiv(g.cW, p.TW);
        grid_y = p.tiles_x * cdiv(g.cH, p.TH);
        if (!make_map_conv(&ma, g.A, g.cH, g.cW, g.cC, p.TW, p.TH))
            return false;
    }
    else if (!make_map(&ma, g.A, g.M, g.K, g.lda, BM))
        return false;
    if (!make_map(&mb, g.B, g.N, g.K, g.ldb, BN))
        return false;
    p.M = g.M;
    p.N = g.N;
    p.K = g.K;
    p.C = g.C;
    p.ldc = g.ldc;
    p.bias = g.biasrow ? nullptr : g.bias;
    p.R = g.R;
    p.alpha = g.alpha;
    p.act = g.act;
    p.slope = g.slope;
    p.c_bf16 = g.c == DT_BF16;
    const size_t smem = sizeof(Smem<BN, STAGES>) + 1024;
    // The shared-memory opt-in is per device.
    static unsigned attr_done = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_done >> (dev & 31) & 1)) {
        if (cudaFuncSetAttribute(tc_gemm_kernel<BN, STAGES>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        attr_done |= 1u << (dev & 31);
    }
    dim3 grid(cdiv(g.N, BN), grid_y);
    tc_gemm_kernel<BN, STAGES><<<grid, NTHREADS, smem, st>>>(ma, mb, p);
    return true;
}

}  // namespace

bool gemm_tc(cudaStream_t st, const GemmArgs &g, int sm_count)
{
    (void)sm_count;
    if (g.ab != DT_BF16 || !g.transb || g.nb != 1)
        return false;
    if (g.amode == 2 || (g.amode == 1 && (g.cC % BK || g.K != 9 * g.cC)))
        return false;
    if (g.biasrow && g.bias)
        return false;
    if (g.M < 64 || g.N < 64 || g.K < 16)
        return false;
    if (((uintptr_t)g.A & 15) || ((uintptr_t)g.B & 15) ||
        (g.amode == 0 && (g.lda & 7)) || (g.ldb & 7))
        return false;
    if (g.N >= 256)
        return launch_tc<256, 4>(st, g);
    return launch_tc<128, 6>(st, g);
}

// Error code of a bounded wait that ran out in a tensor-core kernel since
// the last call (0: none); clears it.
int gemm_tc_status()
{
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int));
    if (v)
        cudaMemcpyToSymbol(g_tc_error, &z, sizeof(int));
    return v;
}

}  // namespace coreg

// Test hook (no reference counterpart): 0 when no tensor-core wait ran out.
extern "C" int coreg_tc_status(void) { return coreg::gemm_tc_status(); }
