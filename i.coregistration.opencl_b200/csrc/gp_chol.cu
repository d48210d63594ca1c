// SPDX-License-Identifier: Unlicense
//
// The Gaussian-process solve of RoMa on the device, in double precision:
// X = (K + noise I)^-1 F for the n x n kernel matrix K (float, symmetric)
// and the n x d basis F, by a blocked right-looking Cholesky factorization
// L L^T = K + noise I and the two triangular solves L Z = F, L^T X = Z.
// Replaces the reference's host gp_solve (roma.c:772-836: Cholesky in
// double, then the two substitutions), whose device round trip
// (roma.c:885-888) disappears.
//
// Blocks of NB = 64. One CTA of 256 threads factors each diagonal block
// and inverts it (Linv_j), so that every other step is a double-precision
// GEMM. The
// working matrix A, the factor L and the right-hand sides F, Z, X live in
// separate buffers, so no step multiplies in place:
//   step j     L_jj, Linv_j           from A_jj
//              L_below = A_below Linv_j^T,  Z_j = Linv_j F_j     (one launch)
//              A_trail -= L_below L_below^T (lower),
//              F_below -= L_below Z_j                            (one launch)
//   backward   X_j = Linv_j^T Z_j,  then Z_above -= L_j,above^T X_j
// A non-positive pivot sets *flag (the reference stops with "kernel not
// positive definite"); the host reads it after the tile.

#include <initializer_list>

#include "common.cuh"

namespace coreg {

#define GP_NB 64

// A = K + noise I in double.
__global__ void gp_init_k(const float *K, int n, double noise, double *A)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= (long)n * n)
        return;
    const long i = e / n, j = e % n;
    A[e] = (double)K[e] + (i == j ? noise : 0.0);
}

constexpr int GP_P = GP_NB + 1;  // shared-memory pitch (doubles)
// Elements of the 64 x 64 lower triangle each of the 256 threads owns.
constexpr int GP_OWN = (GP_NB * (GP_NB + 1) / 2 + 255) / 256;

// Factor the b x b diagonal block of A at (j0, j0) (b <= 64; identity beyond
// b) with all 256 threads: a right-looking unblocked Cholesky in shared
// memory, one barrier per column (thread t owns the lower-triangle elements
// t, t + 256, ...: at column k it updates those right of k with the scaled
// column, l_i = a_ik / sqrt(a_kk), a_ij -= l_i l_j, while the threads of
// rows i > k write l_i into the factor), then the inverse of the factor,
// four threads per column (each column of L^-1 by forward substitution,
// the sums split four ways and joined by shuffles). Writes the lower
// factor into L (pitch n) and the 64 x 64 inverse into Linv. A
// non-positive pivot sets *flag (the factor is then meaningless, as the
// reference's stop says).
__global__ void __launch_bounds__(256)
gp_potrf_inv_k(const double *A, double *L, int n, int j0, int b, double *Linv, int *flag)
{
    extern __shared__ double gp_smem[];
    double *M = gp_smem;                  // 64 x GP_P: the block, updated
    double *F = gp_smem + GP_NB * GP_P;   // 64 x GP_P: the factor
    double *X = F + GP_NB * GP_P;         // 64 x GP_P: the inverse
    const int t = threadIdx.x;
#pragma unroll
    for (int e = t; e < GP_NB * GP_NB; e += 256) {
        const int i = e / GP_NB, j = e % GP_NB;
        M[i * GP_P + j] = i < b && j < b ? A[(long)(j0 + i) * n + j0 + j] : (i == j ? 1.0 : 0.0);
        F[i * GP_P + j] = 0.0;
    }
    // This thread's lower-triangle elements (row-major order of the
    // triangle: element e lies in row i with i (i + 1) / 2 <= e).
    int oi[GP_OWN], oj[GP_OWN];
#pragma unroll
    for (int r = 0; r < GP_OWN; r++) {
        const int e = t + 256 * r;
        int i = (int)((sqrt(8.0 * e + 1.0) - 1.0) * 0.5);
        while ((i + 1) * (i + 2) / 2 <= e)
            i++;
        while (i * (i + 1) / 2 > e)
            i--;
        oi[r] = e < GP_NB * (GP_NB + 1) / 2 ? i : -1;
        oj[r] = e - i * (i + 1) / 2;
    }
    __syncthreads();
    for (int k = 0; k < GP_NB; k++) {
        double d = M[k * GP_P + k];
        if (!(d > 0.0)) {
            if (t == 0)
                *flag = 1;
            d = 1.0;
        }
        const double piv = sqrt(d), rinv = 1.0 / piv;
        if (t == k)
            F[k * GP_P + k] = piv;
        else if (t > k && t < GP_NB)
            F[t * GP_P + k] = M[t * GP_P + k] * rinv;
#pragma unroll
        for (int r = 0; r < GP_OWN; r++) {
            const int i = oi[r], j = oj[r];
            if (i >= 0 && j > k) {
                const double li = M[i * GP_P + k] * rinv, lj = M[j * GP_P + k] * rinv;
                M[i * GP_P + j] = fma(-li, lj, M[i * GP_P + j]);
            }
        }
        __syncthreads();
    }
    // The inverse: column c by threads 4 c .. 4 c + 3; x_i = (delta_ic -
    // sum_{c <= m < i} F_im x_m) / F_ii for i >= c, zero above.
    {
        // Every lane takes part in every shuffle (rows above a column's
        // diagonal sum nothing and store zero).
        const int c = t / 4, q = t % 4;
        for (int i = 0; i < GP_NB; i++) {
            double acc = 0.0;
            for (int m = c + q; m < i; m += 4)
                acc = fma(F[i * GP_P + m], X[m * GP_P + c], acc);
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            if (q == 0)
                X[i * GP_P + c] =
                    i < c ? 0.0 : ((i == c ? 1.0 : 0.0) - acc) / F[i * GP_P + i];
            __syncwarp();
        }
    }
    __syncthreads();
#pragma unroll
    for (int e = t; e < GP_NB * GP_NB; e += 256) {
        const int i = e / GP_NB, j = e % GP_NB;
        Linv[e] = X[i * GP_P + j];
        if (i < b && j < b)
            L[(long)(j0 + i) * n + j0 + j] = F[i * GP_P + j];
    }
}

constexpr size_t GP_POTRF_SMEM = 3 * GP_NB * GP_P * sizeof(double);

// C (M x N, ldc) = A B (sub 0) or C -= A B (sub 1), A(m, k) = A[m sam + k
// sak], B(k, n) = B[k sbk + n sbn]; lower_only skips tiles and elements
// above the diagonal.
struct DgProb {
    int M, N, K;
    const double *A;
    long sam, sak;
    const double *B;
    long sbk, sbn;
    double *C;
    long ldc;
    int sub, lower_only;
};

// Up to two independent products per launch (blockIdx.z).
struct DgBatch {
    DgProb p[2];
};

// 64 x 64 tiles, 4 x 4 per thread. Each CTA stages 64-deep K panels of
// both operands (dynamic shared memory, loads along each operand's
// unit-stride dimension) and runs the panel with no barrier inside; the
// blocked Cholesky's products have K <= 64, so one panel and two barriers
// per tile.
constexpr int DG_T = 64, DG_K = 64;
constexpr size_t DG_SMEM = 2 * DG_K * (DG_T + 1) * sizeof(double);

__device__ __forceinline__ void cp_async8(double *dst, const double *src, bool in)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(
                     (unsigned)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(in ? 8 : 0)
                 : "memory");
}

__global__ void __launch_bounds__(256) dgemm_k(DgBatch batch)
{
    extern __shared__ double dg_smem[];
    const DgProb &q = batch.p[blockIdx.z];
    double(*As)[DG_T + 1] = reinterpret_cast<double(*)[DG_T + 1]>(dg_smem);
    double(*Bs)[DG_T + 1] = reinterpret_cast<double(*)[DG_T + 1]>(dg_smem + DG_K * (DG_T + 1));
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int m0 = blockIdx.y * DG_T, n0 = blockIdx.x * DG_T;
    const int M = q.M, N = q.N, K = q.K;
    if (m0 >= M || n0 >= N || (q.lower_only && n0 > m0 + DG_T - 1))
        return;
    double acc[4][4] = {};
    const bool a_k = q.sak == 1, b_n = q.sbn == 1;
    for (int k0 = 0; k0 < K; k0 += DG_K) {
        // Element-wise asynchronous copies (8 bytes, zero fill outside the
        // operands): every load of the panel in flight at once, no register
        // staging.
#pragma unroll 4
        for (int e = threadIdx.x; e < DG_T * DG_K; e += 256) {
            int r = a_k ? e / DG_K : e % DG_T, k = a_k ? e % DG_K : e / DG_T;
            int m = m0 + r, kk = k0 + k;
            bool in = m < M && kk < K;
            cp_async8(&As[k][r], in ? q.A + (long)m * q.sam + (long)kk * q.sak : q.A, in);
            r = b_n ? e % DG_T : e / DG_K;
            k = b_n ? e / DG_T : e % DG_K;
            const int nn = n0 + r;
            kk = k0 + k;
            in = nn < N && kk < K;
            cp_async8(&Bs[k][r], in ? q.B + (long)kk * q.sbk + (long)nn * q.sbn : q.B, in);
        }
        asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
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
            if (nn < N && (!q.lower_only || nn <= m)) {
                double *c = q.C + (long)m * q.ldc + nn;
                *c = q.sub ? *c - acc[i][j] : acc[i][j];
            }
        }
    }
}

static DgProb prob(int M, int N, int K, const double *A, long sam, long sak, const double *B,
                   long sbk, long sbn, double *C, long ldc, int sub, int lower_only)
{
    DgProb p = {M, N, K, A, sam, sak, B, sbk, sbn, C, ldc, sub, lower_only};
    return p;
}

// One launch for the non-empty products among p0 and p1 (either may be
// NULL).
static void dgemm2(cudaStream_t st, const DgProb *p0, const DgProb *p1)
{
    DgBatch b;
    int count = 0, gx = 0, gy = 0;
    for (const DgProb *p : {p0, p1})
        if (p && p->M > 0 && p->N > 0 && p->K > 0) {
            b.p[count++] = *p;
            gx = max(gx, (int)cdiv(p->N, DG_T));
            gy = max(gy, (int)cdiv(p->M, DG_T));
        }
    if (count)
        dgemm_k<<<dim3(gx, gy, count), 256, DG_SMEM, st>>>(b);
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

// Work: A and L (n x n each), F, Z, X (n x d each) and cdiv(n, 64) 64 x 64
// inverses, in doubles.
size_t gp_work_doubles(int n, int d)
{
    const size_t nb = (size_t)cdiv(n, GP_NB);
    return 2 * (size_t)n * n + 3 * (size_t)n * d + nb * GP_NB * GP_NB;
}

static bool opt_in(const void *fn, size_t bytes, unsigned *mask)
{
    int dev = 0;
    cudaGetDevice(&dev);
    if (*mask >> (dev & 31) & 1)
        return true;
    if (!cuda_ok(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)bytes),
                 "gp kernels"))
        return false;
    *mask |= 1u << (dev & 31);
    return true;
}

void gp_solve_dev(cudaStream_t st, const float *K, int n, const float *F_in, int d,
                  double noise, float *X_out, double *work, int *flag)
{
    const int nb = cdiv(n, GP_NB);
    double *A = work, *L = A + (size_t)n * n;
    double *F = L + (size_t)n * n, *Z = F + (size_t)n * d, *X = Z + (size_t)n * d;
    double *Linv = X + (size_t)n * d;
    const long nn = (long)n * n, nd = (long)n * d;
    static unsigned opted_g = 0, opted_p = 0;
    if (!opt_in((const void *)dgemm_k, DG_SMEM, &opted_g) ||
        !opt_in((const void *)gp_potrf_inv_k, GP_POTRF_SMEM, &opted_p))
        return;

    gp_init_k<<<cdiv(nn, 256), 256, 0, st>>>(K, n, noise, A);
    gp_load_rhs_k<<<cdiv(nd, 256), 256, 0, st>>>(F_in, nd, F);
    for (int j = 0; j < nb; j++) {
        const int j0 = j * GP_NB, b = n - j0 < GP_NB ? n - j0 : GP_NB;
        const int rest = n - j0 - b;
        double *Li = Linv + (size_t)j * GP_NB * GP_NB;
        gp_potrf_inv_k<<<1, 256, GP_POTRF_SMEM, st>>>(A, L, n, j0, b, Li, flag);
        const long below = (long)(j0 + b) * n + j0;
        // L_below = A_below Linv^T;  Z_j = Linv F_j.
        const DgProb panel = prob(rest, b, b, A + below, n, 1, Li, 1, GP_NB, L + below, n, 0, 0);
        const DgProb zj = prob(b, d, b, Li, GP_NB, 1, F + (long)j0 * d, d, 1, Z + (long)j0 * d,
                               d, 0, 0);
        dgemm2(st, &panel, &zj);
        // A_trail -= L_below L_below^T (lower);  F_below -= L_below Z_j.
        const DgProb trail = prob(rest, rest, b, L + below, n, 1, L + below, 1, n,
                                  A + (long)(j0 + b) * n + j0 + b, n, 1, 1);
        const DgProb fb = prob(rest, d, b, L + below, n, 1, Z + (long)j0 * d, d, 1,
                               F + (long)(j0 + b) * d, d, 1, 0);
        dgemm2(st, &trail, &fb);
    }
    // L^T X = Z from the last block up.
    for (int j = nb - 1; j >= 0; j--) {
        const int j0 = j * GP_NB, b = n - j0 < GP_NB ? n - j0 : GP_NB;
        const double *Li = Linv + (size_t)j * GP_NB * GP_NB;
        const DgProb xj = prob(b, d, b, Li, 1, GP_NB, Z + (long)j0 * d, d, 1, X + (long)j0 * d,
                               d, 0, 0);
        dgemm2(st, &xj, nullptr);
        const DgProb up =
            prob(j0, d, b, L + (long)j0 * n, 1, n, X + (long)j0 * d, d, 1, Z, d, 1, 0);
        dgemm2(st, &up, nullptr);
    }
    gp_store_k<<<cdiv(nd, 256), 256, 0, st>>>(X, nd, X_out);
}

}  // namespace coreg
