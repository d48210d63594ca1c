// SPDX-License-Identifier: Unlicense
//
// The Gaussian-process solve of RoMa on the device, in double precision:
// X = (K + noise I)^-1 F for the n x n kernel matrix K (float, symmetric)
// and the n x d basis F, by a blocked right-looking Cholesky factorization
// and two blocked triangular solves. Replaces the reference's host
// gp_solve (roma.c:772-836: Cholesky in double, L Z = F then L^T X = Z),
// whose device round trip (roma.c:885-888) disappears.
//
// Blocks of NB = 64: the diagonal block is factored (or solved) by one
// thread block in shared memory, the panels and trailing updates are
// double-precision GEMMs. A non-positive pivot sets *flag (the reference
// stops with "kernel not positive definite"); the host reads it after
// the tile.

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

// Factor the b x b diagonal block at (j0, j0) in place: column by column
// (left-looking within the block, as the reference's loop).
__global__ void __launch_bounds__(256)
gp_potrf_k(double *A, int n, int j0, int b, int *flag)
{
    __shared__ double L[GP_NB][GP_NB + 1];
    const int t = threadIdx.x;
    for (int e = t; e < b * b; e += blockDim.x) {
        const int i = e / b, j = e % b;
        L[i][j] = A[(long)(j0 + i) * n + j0 + j];
    }
    __syncthreads();
    for (int j = 0; j < b; j++) {
        __shared__ double diag;
        if (t == 0) {
            double s = L[j][j];
            for (int k = 0; k < j; k++)
                s -= L[j][k] * L[j][k];
            if (!(s > 0)) {
                *flag = 1;
                s = 1.0;
            }
            diag = sqrt(s);
            L[j][j] = diag;
        }
        __syncthreads();
        for (int i = j + 1 + t; i < b; i += blockDim.x) {
            double s = L[i][j];
            for (int k = 0; k < j; k++)
                s -= L[i][k] * L[j][k];
            L[i][j] = s / diag;
        }
        __syncthreads();
    }
    for (int e = t; e < b * b; e += blockDim.x) {
        const int i = e / b, j = e % b;
        A[(long)(j0 + i) * n + j0 + j] = j <= i ? L[i][j] : 0.0;
    }
}

// Panel: rows i >= j0 + b of the block column: x L_d^T = a, one row per
// thread (forward substitution against the factored diagonal block).
__global__ void gp_trsm_panel_k(double *A, int n, int j0, int b)
{
    __shared__ double L[GP_NB][GP_NB + 1];
    for (int e = threadIdx.x; e < b * b; e += blockDim.x) {
        const int i = e / b, j = e % b;
        L[i][j] = A[(long)(j0 + i) * n + j0 + j];
    }
    __syncthreads();
    const int i = j0 + b + blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n)
        return;
    double x[GP_NB];
    double *row = A + (long)i * n + j0;
    for (int k = 0; k < b; k++) {
        double s = row[k];
        for (int q = 0; q < k; q++)
            s -= x[q] * L[k][q];
        x[k] = s / L[k][k];
    }
    for (int k = 0; k < b; k++)
        row[k] = x[k];
}

// C (M x N, ldc) -= A B with A(m, k) = A[m sam + k sak], B(k, n) =
// B[k sbk + n sbn]; 64 x 64 tiles, 16 k per step, 4 x 4 per thread.
__global__ void __launch_bounds__(256)
dgemm_sub_k(int M, int N, int K, const double *A, long sam, long sak,
            const double *B, long sbk, long sbn, double *C, long ldc,
            int lower_only)
{
    __shared__ double As[16][64 + 1];
    __shared__ double Bs[16][64 + 1];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    if (lower_only && n0 > m0 + 63)
        return;
    double acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 16) {
        for (int e = threadIdx.x; e < 64 * 16; e += 256) {
            const int r = e / 16, k = e % 16;
            const int m = m0 + r, kk = k0 + k;
            As[k][r] = m < M && kk < K ? A[m * sam + kk * sak] : 0.0;
            const int nn = n0 + r;
            Bs[k][r] = nn < N && kk < K ? B[kk * sbk + nn * sbn] : 0.0;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 16; k++) {
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
            if (nn < N && (!lower_only || nn <= m))
                C[(long)m * ldc + nn] -= acc[i][j];
        }
    }
}

static void dgemm_sub(cudaStream_t st, int M, int N, int K, const double *A,
                      long sam, long sak, const double *B, long sbk, long sbn,
                      double *C, long ldc, int lower_only)
{
    if (M <= 0 || N <= 0 || K <= 0)
        return;
    dgemm_sub_k<<<dim3(cdiv(N, 64), cdiv(M, 64)), 256, 0, st>>>(
        M, N, K, A, sam, sak, B, sbk, sbn, C, ldc, lower_only);
}

// Z (n x d) from F (float), for the solves.
__global__ void gp_load_rhs_k(const float *F, long e_n, double *Z)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < e_n)
        Z[e] = F[e];
}

// Diagonal-block triangular solve for every column of Z rows j0 .. j0+b:
// forward (L_d z = f) or backward (L_d^T x = z); one thread per column.
__global__ void gp_trsv_block_k(const double *A, int n, int j0, int b,
                                double *Z, int d, int backward)
{
    __shared__ double L[GP_NB][GP_NB + 1];
    for (int e = threadIdx.x; e < b * b; e += blockDim.x) {
        const int i = e / b, j = e % b;
        L[i][j] = A[(long)(j0 + i) * n + j0 + j];
    }
    __syncthreads();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= d)
        return;
    double z[GP_NB];
    for (int k = 0; k < b; k++)
        z[k] = Z[(long)(j0 + k) * d + c];
    if (!backward) {
        for (int k = 0; k < b; k++) {
            double s = z[k];
            for (int q = 0; q < k; q++)
                s -= L[k][q] * z[q];
            z[k] = s / L[k][k];
        }
    }
    else {
        for (int k = b - 1; k >= 0; k--) {
            double s = z[k];
            for (int q = k + 1; q < b; q++)
                s -= L[q][k] * z[q];
            z[k] = s / L[k][k];
        }
    }
    for (int k = 0; k < b; k++)
        Z[(long)(j0 + k) * d + c] = z[k];
}

__global__ void gp_store_k(const double *Z, long e_n, float *X)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < e_n)
        X[e] = (float)Z[e];
}

// Work: n * n + n * d doubles.
void gp_solve_dev(cudaStream_t st, const float *K, int n, const float *F, int d,
                  double noise, float *X, double *work, int *flag)
{
    double *A = work, *Z = work + (size_t)n * n;
    const long nn = (long)n * n, nd = (long)n * d;

    gp_init_k<<<cdiv(nn, 256), 256, 0, st>>>(K, n, noise, A);
    for (int j0 = 0; j0 < n; j0 += GP_NB) {
        const int b = n - j0 < GP_NB ? n - j0 : GP_NB;
        const int rest = n - j0 - b;
        gp_potrf_k<<<1, 256, 0, st>>>(A, n, j0, b, flag);
        if (rest > 0) {
            gp_trsm_panel_k<<<cdiv(rest, 64), 64, 0, st>>>(A, n, j0, b);
            // Trailing lower triangle -= panel panel^T.
            const double *P = A + (long)(j0 + b) * n + j0;
            dgemm_sub(st, rest, rest, b, P, n, 1, P, 1, n,
                      A + (long)(j0 + b) * n + j0 + b, n, 1);
        }
    }
    gp_load_rhs_k<<<cdiv(nd, 256), 256, 0, st>>>(F, nd, Z);
    // L Z = F: solve block j, then update the rows below.
    for (int j0 = 0; j0 < n; j0 += GP_NB) {
        const int b = n - j0 < GP_NB ? n - j0 : GP_NB;
        const int rest = n - j0 - b;
        gp_trsv_block_k<<<cdiv(d, 64), 64, 0, st>>>(A, n, j0, b, Z, d, 0);
        if (rest > 0)
            dgemm_sub(st, rest, d, b, A + (long)(j0 + b) * n + j0, n, 1,
                      Z + (long)j0 * d, d, 1, Z + (long)(j0 + b) * d, d, 0);
    }
    // L^T X = Z: from the last block up; the rows above get
    // Z[0:j0] -= L[j0:j0+b, 0:j0]^T X[j0:j0+b].
    int last = ((n - 1) / GP_NB) * GP_NB;
    for (int j0 = last; j0 >= 0; j0 -= GP_NB) {
        const int b = n - j0 < GP_NB ? n - j0 : GP_NB;
        gp_trsv_block_k<<<cdiv(d, 64), 64, 0, st>>>(A, n, j0, b, Z, d, 1);
        if (j0 > 0)
            dgemm_sub(st, j0, d, b, A + (long)j0 * n, 1, n, Z + (long)j0 * d, d,
                      1, Z, d, 0);
    }
    gp_store_k<<<cdiv(nd, 256), 256, 0, st>>>(Z, nd, X);
}

}  // namespace coreg
