// SPDX-License-Identifier: Unlicense
//
// The Gaussian-process solve of RoMa on the device, in double precision:
// X = (K + noise I)^-1 F for the n x n kernel matrix K (float, symmetric)
// and the n x d basis F, by a blocked right-looking Cholesky factorization
// and two blocked triangular solves. Replaces the reference's host
// gp_solve (roma.c:772-836: Cholesky in double, L Z = F then L^T X = Z),
// whose device round trip (roma.c:885-888) disappears.
//
// Blocks of NB = 64. One CTA factors each diagonal block in shared memory
// and also inverts it (Linv); with the inverses every other step is a
// double-precision GEMM:
//   panel      L21 = A21 Linv^T
//   trailing   A22 -= L21 L21^T (lower triangle)
//   forward    Z_j = Linv_j F'_j, then F'_below -= L_below,j Z_j
//   backward   X_j = Linv_j^T Z'_j, then Z'_above -= L_j,above^T X_j
// A non-positive pivot sets *flag (the reference stops with "kernel not
// positive definite"); the host reads it after the tile.

#include "common.cuh"

namespace coreg {

#define GP_NB 64

// A = K + noise I in double (lower triangle used).
__global__ void gp_init_k(const float *K, int n, double noise, double *A)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= (long)n * n)
        return;
    const long i = e / n, j = e % n;
    A[e] = (double)K[e] + (i == j ? noise : 0.0);
}

// Factor the b x b diagonal block at (j0, j0) in place and write its
// inverse into Linv (GP_NB x GP_NB, zero padded beyond b). 256 threads
// stage the block through shared memory with coalesced accesses (identity
// beyond b); threads i < 64 then hold row i in registers. Per column
// k the pivot's owner publishes sqrt(L[k][k]) and its reciprocal, the rows
// below scale their entry k and publish it, and every row updates its own
// entries k < j <= i: two block barriers per column. The inverse is
// computed column by column (thread c solves L x = e_c) in axpy order, so
// that each step's multiply-adds are independent.
constexpr int GP_POTRF_THREADS = 256;

__global__ void __launch_bounds__(GP_POTRF_THREADS)
gp_potrf_inv_k(double *A, int n, int j0, int b, double *Linv, int *flag)
{
    __shared__ double Ls[GP_NB][GP_NB + 1];
    __shared__ double colk[GP_NB], rdiag[GP_NB];
    __shared__ double piv_r;
    const int t = threadIdx.x, i = t % GP_NB, rq = t / GP_NB;
    constexpr int RSTEP = GP_POTRF_THREADS / GP_NB;
#pragma unroll
    for (int row = rq; row < GP_NB; row += RSTEP)
        Ls[row][i] = row < b && i < b ? A[(long)(j0 + row) * n + j0 + i] : (row == i ? 1.0 : 0.0);
    __syncthreads();
    const bool own = t < GP_NB;
    double r[GP_NB];
#pragma unroll
    for (int j = 0; j < GP_NB; j++)
        r[j] = Ls[i][j];
#pragma unroll
    for (int k = 0; k < GP_NB; k++) {
        if (own && i == k) {
            double d = r[k];
            if (!(d > 0.0)) {
                *flag = 1;
                d = 1.0;
            }
            const double rc = rsqrt(d);
            r[k] = d * rc;
            piv_r = rc;
            rdiag[k] = rc;
        }
        __syncthreads();
        if (own && i > k) {
            r[k] *= piv_r;
            colk[i] = r[k];
        }
        __syncthreads();
        if (own && i > k) {
            const double lik = r[k];
#pragma unroll
            for (int j = k + 1; j < GP_NB; j++)
                if (j <= i)
                    r[j] = fma(-lik, colk[j], r[j]);
        }
    }
    if (own) {
#pragma unroll
        for (int j = 0; j < GP_NB; j++)
            Ls[i][j] = j <= i ? r[j] : 0.0;
    }
    __syncthreads();
#pragma unroll
    for (int row = rq; row < GP_NB; row += RSTEP)
        if (row < b && i < b)
            A[(long)(j0 + row) * n + j0 + i] = Ls[row][i];
    if (!own)
        return;
    // Column c of the inverse: x = e_c; for k = c, c + 1, ...: x_k /= L_kk,
    // then x_m -= L_mk x_k for m > k.
    const int c = i;
    double x[GP_NB];
#pragma unroll
    for (int m = 0; m < GP_NB; m++)
        x[m] = m == c ? 1.0 : 0.0;
#pragma unroll
    for (int k = 0; k < GP_NB; k++) {
        if (k >= c) {
            x[k] *= rdiag[k];
            const double xk = x[k];
#pragma unroll
            for (int m = k + 1; m < GP_NB; m++)
                x[m] = fma(-Ls[m][k], xk, x[m]);
        }
    }
    double *li = Linv + c;
#pragma unroll
    for (int m = 0; m < GP_NB; m++)
        li[(long)m * GP_NB] = x[m];
}

// C (M x N, ldc) = A B (sub 0) or C -= A B (sub 1), A(m, k) = A[m sam + k
// sak], B(k, n) = B[k sbk + n sbn]; 64 x 64 tiles, 4 x 4 per thread. Each
// CTA stages 64-deep K panels of both operands (dynamic shared memory,
// loads along each operand's unit-stride dimension) and runs the panel
// with no barrier inside; the blocked Cholesky's products have K <= 64, so
// one panel and two barriers per tile. lower_only skips tiles and elements
// above the diagonal.
constexpr int DG_T = 64, DG_K = 64;
constexpr size_t DG_SMEM = 2 * DG_K * (DG_T + 1) * sizeof(double);

__global__ void __launch_bounds__(256)
dgemm_k(int M, int N, int K, const double *A, long sam, long sak, const double *B,
        long sbk, long sbn, double *C, long ldc, int sub, int lower_only)
{
    extern __shared__ double dg_smem[];
    double(*As)[DG_T + 1] = reinterpret_cast<double(*)[DG_T + 1]>(dg_smem);
    double(*Bs)[DG_T + 1] = reinterpret_cast<double(*)[DG_T + 1]>(dg_smem + DG_K * (DG_T + 1));
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int m0 = blockIdx.y * DG_T, n0 = blockIdx.x * DG_T;
    if (lower_only && n0 > m0 + DG_T - 1)
        return;
    double acc[4][4] = {};
    const bool a_k = sak == 1, b_n = sbn == 1;
    for (int k0 = 0; k0 < K; k0 += DG_K) {
#pragma unroll 4
        for (int e = threadIdx.x; e < DG_T * DG_K; e += 256) {
            int r = a_k ? e / DG_K : e % DG_T, k = a_k ? e % DG_K : e / DG_T;
            int m = m0 + r, kk = k0 + k;
            As[k][r] = m < M && kk < K ? A[m * sam + kk * sak] : 0.0;
            r = b_n ? e % DG_T : e / DG_K;
            k = b_n ? e / DG_T : e % DG_K;
            const int nn = n0 + r;
            kk = k0 + k;
            Bs[k][r] = nn < N && kk < K ? B[kk * sbk + nn * sbn] : 0.0;
        }
        __syncthreads();
        const int kc = K - k0 < DG_K ? K - k0 : DG_K;
#pragma unroll 8
        for (int k = 0; k < kc; k++) {
            double a[4], bb[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                a[i] = As[k][ty + 16 * i];
                bb[i] = Bs[k][tx + 16 * i];
            }
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++)
                    acc[i][j] = fma(a[i], bb[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int m = m0 + ty + 16 * i;
        if (m >= M)
            continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int nn = n0 + tx + 16 * j;
            if (nn < N && (!lower_only || nn <= m)) {
                double *c = C + (long)m * ldc + nn;
                *c = sub ? *c - acc[i][j] : acc[i][j];
            }
        }
    }
}

static void dgemm(cudaStream_t st, int M, int N, int K, const double *A, long sam, long sak,
                  const double *B, long sbk, long sbn, double *C, long ldc, int sub,
                  int lower_only)
{
    if (M <= 0 || N <= 0 || K <= 0)
        return;
    dgemm_k<<<dim3(cdiv(N, DG_T), cdiv(M, DG_T)), 256, DG_SMEM, st>>>(
        M, N, K, A, sam, sak, B, sbk, sbn, C, ldc, sub, lower_only);
}

__global__ void gp_load_rhs_k(const float *F, long e_n, double *Z)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < e_n)
        Z[e] = F[e];
}

__global__ void gp_store_k(const double *Z, long e_n, float *X)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < e_n)
        X[e] = (float)Z[e];
}

// Work: n n + n d doubles (A, Z), cdiv(n, 64) 64 x 64 doubles (inverses)
// and 64 max(n, d) doubles (the panel or right-hand-side block copy).
size_t gp_work_doubles(int n, int d)
{
    const size_t nb = (size_t)cdiv(n, GP_NB);
    const size_t w = (size_t)(n > d ? n : d);
    return (size_t)n * n + (size_t)n * d + nb * GP_NB * GP_NB + GP_NB * w;
}

void gp_solve_dev(cudaStream_t st, const float *K, int n, const float *F, int d,
                  double noise, float *X, double *work, int *flag)
{
    const int nb = cdiv(n, GP_NB);
    double *A = work, *Z = A + (size_t)n * n;
    double *Linv = Z + (size_t)n * d;
    double *T = Linv + (size_t)nb * GP_NB * GP_NB;
    const long nn = (long)n * n, nd = (long)n * d;

    static unsigned opted = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(opted >> (dev & 31) & 1)) {
        if (!cuda_ok(cudaFuncSetAttribute(dgemm_k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)DG_SMEM),
                     "dgemm_k"))
            return;
        opted |= 1u << (dev & 31);
    }
    gp_init_k<<<cdiv(nn, 256), 256, 0, st>>>(K, n, noise, A);
    for (int j = 0; j < nb; j++) {
        const int j0 = j * GP_NB, b = n - j0 < GP_NB ? n - j0 : GP_NB;
        const int rest = n - j0 - b;
        double *Li = Linv + (size_t)j * GP_NB * GP_NB;
        gp_potrf_inv_k<<<1, GP_POTRF_THREADS, 0, st>>>(A, n, j0, b, Li, flag);
        if (rest > 0) {
            double *P = A + (long)(j0 + b) * n + j0;
            // Panel: L21 = A21 Linv^T, through a copy of A21.
            cudaMemcpy2DAsync(T, GP_NB * sizeof(double), P, n * sizeof(double),
                              b * sizeof(double), rest, cudaMemcpyDeviceToDevice, st);
            dgemm(st, rest, b, b, T, GP_NB, 1, Li, 1, GP_NB, P, n, 0, 0);
            // Trailing lower triangle -= L21 L21^T.
            dgemm(st, rest, rest, b, P, n, 1, P, 1, n, A + (long)(j0 + b) * n + j0 + b, n, 1,
                  1);
        }
    }
    gp_load_rhs_k<<<cdiv(nd, 256), 256, 0, st>>>(F, nd, Z);
    // L Z = F: Z_j = Linv_j F'_j, then the rows below.
    for (int j = 0; j < nb; j++) {
        const int j0 = j * GP_NB, b = n - j0 < GP_NB ? n - j0 : GP_NB;
        const int rest = n - j0 - b;
        const double *Li = Linv + (size_t)j * GP_NB * GP_NB;
        cudaMemcpyAsync(T, Z + (long)j0 * d, (size_t)b * d * sizeof(double),
                        cudaMemcpyDeviceToDevice, st);
        dgemm(st, b, d, b, Li, GP_NB, 1, T, d, 1, Z + (long)j0 * d, d, 0, 0);
        if (rest > 0)
            dgemm(st, rest, d, b, A + (long)(j0 + b) * n + j0, n, 1, Z + (long)j0 * d, d, 1,
                  Z + (long)(j0 + b) * d, d, 1, 0);
    }
    // L^T X = Z: X_j = Linv_j^T Z'_j from the last block up, then
    // Z'_above -= L_j,above^T X_j.
    for (int j = nb - 1; j >= 0; j--) {
        const int j0 = j * GP_NB, b = n - j0 < GP_NB ? n - j0 : GP_NB;
        const double *Li = Linv + (size_t)j * GP_NB * GP_NB;
        cudaMemcpyAsync(T, Z + (long)j0 * d, (size_t)b * d * sizeof(double),
                        cudaMemcpyDeviceToDevice, st);
        dgemm(st, b, d, b, Li, 1, GP_NB, T, d, 1, Z + (long)j0 * d, d, 0, 0);
        if (j0 > 0)
            dgemm(st, j0, d, b, A + (long)j0 * n, 1, n, Z + (long)j0 * d, d, 1, Z, d, 1, 0);
    }
    gp_store_k<<<cdiv(nd, 256), 256, 0, st>>>(Z, nd, X);
}

}  // namespace coreg
