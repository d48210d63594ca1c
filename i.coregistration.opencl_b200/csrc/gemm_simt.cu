// SPDX-License-Identifier: Unlicense
//
// Float32 FMA GEMM (the accurate path of ops_gemm and of the models),
// with the contract of the reference's gemm / gemm_big kernels
// (ops.cl:39-284; see gemm.cuh). Tiles of BM x BN outputs per block of
// 256 threads, TM x TN outputs per thread, BK = 8 deep, double-buffered
// through shared memory with the next tile prefetched into registers.
// Bounds are checked per element, so any shape, stride and offset works.

#include "gemm.cuh"

namespace coreg {

template <typename T>
__device__ __forceinline__ float gld(const T *p) { return ldf(p); }

// Element (m, k) of the A operand in its mode (see GemmArgs::amode).
template <typename T>
__device__ __forceinline__ float a_elem(const GemmArgs &g, const T *A, int m,
                                        int k)
{
    if (g.amode == 1) {
        const int C = g.cC, x = m % g.cW, y = m / g.cW;
        const int c = k % C, kx = (k / C) % 3, ky = k / (3 * C);
        const int yy = y + ky - 1, xx = x + kx - 1;
        if (yy < 0 || yy >= g.cH || xx < 0 || xx >= g.cW)
            return 0.0f;
        return gld(A + ((long)yy * g.cW + xx) * C + c);
    }
    if (g.amode == 2) {
        const int P = g.cP, pw = g.cW / P;
        const int px = m % pw, py = m / pw;
        const int kx = k % P, ky = (k / P) % P, c = k / (P * P);
        return gld(A + ((long)(py * P + ky) * g.cW + px * P + kx) * g.cC + c);
    }
    return gld(A + (long)m * g.lda + k);
}

template <typename TA, typename TC, int BM, int BN, int TM, int TN>
__global__ void __launch_bounds__(256)
gemm_simt_kernel(GemmArgs g)
{
    constexpr int BK = 8;
    constexpr int NA = BM * BK / 256; // A elements per thread and tile
    constexpr int NB = BN * BK / 256;
    __shared__ float As[2][BK][BM + 4];
    __shared__ float Bs[2][BK][BN + 4];
    const int tid = threadIdx.x;
    const int tx = tid % (BN / TN), ty = tid / (BN / TN);
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const long b = blockIdx.z, b0 = b / g.nb1, b1 = b % g.nb1;
    const TA *A = (const TA *)g.A + b0 * g.sa0 + b1 * g.sa1;
    const TA *B = (const TA *)g.B + b0 * g.sb0 + b1 * g.sb1;
    TC *C = (TC *)g.C + b0 * g.sc0 + b1 * g.sc1;
    const TC *R = g.R ? (const TC *)g.R + b0 * g.sc0 + b1 * g.sc1 : nullptr;
    const int M = g.M, N = g.N, K = g.K;
    float acc[TM][TN];
    float ra[NA], rb[NB];

#pragma unroll
    for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++)
            acc[i][j] = 0.0f;

    // A: element e = tid + 256 i of the BM x BK tile, row e / BK, k e % BK.
    auto load_a = [&](int k0) {
#pragma unroll
        for (int i = 0; i < NA; i++) {
            const int e = tid + 256 * i, r = e / BK, c = e % BK;
            const int gm = m0 + r, gk = k0 + c;
            ra[i] = gm < M && gk < K ? a_elem(g, A, gm, gk) : 0.0f;
        }
    };
    auto load_b = [&](int k0) {
#pragma unroll
        for (int i = 0; i < NB; i++) {
            const int e = tid + 256 * i;
            int n, k;
            if (g.transb) {
                n = e / BK;
                k = e % BK;
            }
            else {
                k = e / BN;
                n = e % BN;
            }
            const int gn = n0 + n, gk = k0 + k;
            float v = 0.0f;
            if (gn < N && gk < K)
                v = g.transb ? gld(B + (long)gn * g.ldb + gk)
                             : gld(B + (long)gk * g.ldb + gn);
            rb[i] = v;
        }
    };
    auto store = [&](int buf) {
#pragma unroll
        for (int i = 0; i < NA; i++) {
            const int e = tid + 256 * i;
            As[buf][e % BK][e / BK] = ra[i];
        }
#pragma unroll
        for (int i = 0; i < NB; i++) {
            const int e = tid + 256 * i;
            if (g.transb)
                Bs[buf][e % BK][e / BK] = rb[i];
            else
                Bs[buf][e / BN][e % BN] = rb[i];
        }
    };

    load_a(0);
    load_b(0);
    store(0);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < K; k0 += BK) {
        const bool more = k0 + BK < K;
        if (more) {
            load_a(k0 + BK);
            load_b(k0 + BK);
        }
#pragma unroll
        for (int k = 0; k < BK; k++) {
            float a[TM], bb[TN];
            // Thread rows ty * TM/2 .. and BM/2 + ty * TM/2 .. (halves
            // apart, so that the shared-memory reads are conflict free).
#pragma unroll
            for (int i = 0; i < TM / 2; i++) {
                a[i] = As[buf][k][ty * (TM / 2) + i];
                a[TM / 2 + i] = As[buf][k][BM / 2 + ty * (TM / 2) + i];
            }
#pragma unroll
            for (int j = 0; j < TN / 2; j++) {
                bb[j] = Bs[buf][k][tx * (TN / 2) + j];
                bb[TN / 2 + j] = Bs[buf][k][BN / 2 + tx * (TN / 2) + j];
            }
#pragma unroll
            for (int i = 0; i < TM; i++)
#pragma unroll
                for (int j = 0; j < TN; j++)
                    acc[i][j] = fmaf(a[i], bb[j], acc[i][j]);
        }
        if (more) {
            store(buf ^ 1);
            __syncthreads();
            buf ^= 1;
        }
    }

#pragma unroll
    for (int i = 0; i < TM; i++) {
        const int m = m0 + (i < TM / 2 ? ty * (TM / 2) + i
                                       : BM / 2 + ty * (TM / 2) + i - TM / 2);
        if (m >= M)
            continue;
#pragma unroll
        for (int j = 0; j < TN; j++) {
            const int n = n0 + (j < TN / 2 ? tx * (TN / 2) + j
                                           : BN / 2 + tx * (TN / 2) + j - TN / 2);
            if (n >= N)
                continue;
            float v = g.alpha * acc[i][j];
            if (g.bias)
                v += g.bias[g.biasrow ? m : n];
            v = apply_act(v, g.act, g.slope);
            const long idx = (long)m * g.ldc + n;
            if (R)
                v += ldf(R + idx);
            stf(C + idx, v);
        }
    }
}

template <typename TA, typename TC>
static void launch(cudaStream_t st, const GemmArgs &g)
{
    const long tiles128 = (long)cdiv(g.M, 128) * cdiv(g.N, 128) * g.nb;

    if (tiles128 >= 148 && g.M >= 64 && g.N >= 64) {
        dim3 grid(cdiv(g.N, 128), cdiv(g.M, 128), g.nb);
        gemm_simt_kernel<TA, TC, 128, 128, 8, 8><<<grid, 256, 0, st>>>(g);
    }
    else {
        dim3 grid(cdiv(g.N, 64), cdiv(g.M, 64), g.nb);
        gemm_simt_kernel<TA, TC, 64, 64, 4, 4><<<grid, 256, 0, st>>>(g);
    }
}

void gemm_simt(cudaStream_t st, const GemmArgs &g)
{
    if (g.M <= 0 || g.N <= 0 || g.nb <= 0)
        return;
    if (g.nb > 65535) {
        fail("GEMM batch of %d products exceeds 65535", g.nb);
        return;
    }
    if (g.ab == DT_F32 && g.c == DT_F32)
        launch<float, float>(st, g);
    else if (g.ab == DT_F32 && g.c == DT_BF16)
        launch<float, __nv_bfloat16>(st, g);
    else if (g.ab == DT_BF16 && g.c == DT_F32)
        launch<__nv_bfloat16, float>(st, g);
    else
        launch<__nv_bfloat16, __nv_bfloat16>(st, g);
    launch_ok("gemm_simt");
}

void gemm_run(const struct ocl_backend *ocl, const GemmArgs &g,
              const char *what)
{
    Prof p(ocl, what);

    if (pending())
        return;
    if (g.ab == DT_BF16 && g.transb && gemm_tc(stream_of(ocl), g, ocl->sm_count))
        return;
    gemm_simt(stream_of(ocl), g);
}

}  // namespace coreg
