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
// Blocks of 64 rows. The factor overwrites the lower triangle of the
// working matrix A in place; the right-hand sides F become Z, then X, in
// place in R. Three kernels, every CTA one 64 x 64 block of work:
//   gp_factor_k (j)  CTA 0: the diagonal block j receives the update of
//                    block column j - 1 and is factored (L_jj and the
//                    reciprocals 1 / L_kk); the other CTAs apply the same
//                    update to the rest of the trailing matrix (lower
//                    blocks) and to the right-hand sides below block j-1;
//   gp_panel_k (j)   the blocks below the diagonal, L_ij = A_ij L_jj^-T, and
//                    Z_j = L_jj^-1 F_j, by forward substitution;
//   gp_back_k (j)    from the last block up: Z_j receives the update of
//                    X_{j+1} and is solved against L_jj^T (X_j, also
//                    rounded to float into the output), while the other
//                    CTAs apply X_{j+1}'s update to Z_i, i < j.
// Each 64-vector of a substitution is held by four threads of a warp (16
// entries each); the entry solved at a step is passed to the other three
// by a shuffle, so the 64 steps need no barrier and, with the staged
// factor zero on and above its diagonal, no branch. The diagonal block is
// factored 16 columns at a time, each panel by one warp in registers.
// Operands are staged in shared memory by asynchronous copies. Every
// chain here is latency-bound (one pivot after another), so the kernels
// are written for short dependency chains and few instructions per step.
// A non-positive pivot sets *flag (the reference stops with "kernel not
// positive definite"); the host reads it after the tile.

#include "common.cuh"

namespace coreg {

#define GP_NB 64

namespace {

constexpr int GP_T = 256;         // threads per CTA
constexpr int GP_SP = GP_NB + 1;  // pitch of the staged product operands and of the block
// A staged triangular factor: row k holds four quarters of 16 entries,
// each padded to 18 doubles, so that the four quarters a warp reads at
// one step (16-byte loads) fall in different banks.
constexpr int GP_QP = 18, GP_LP = 4 * GP_QP;
constexpr size_t GP_SMEM = 2 * GP_NB * GP_SP * sizeof(double);
static_assert((size_t)GP_NB * GP_LP * sizeof(double) + GP_NB * sizeof(double) <= GP_SMEM,
              "the staged factor fits the operand staging");

struct Gp {
    double *A;   // n x n, pitch n: K + noise I (lower triangle), then L
    double *R;   // n x d: F, then Z, then X
    double *rd;  // n: 1 / L_kk
    float *X;    // n x d: X rounded to float
    int n, d, nb, db;
    int *flag;
};

__device__ __forceinline__ int block_rows(int n, int i)
{
    return min(GP_NB, n - i * GP_NB);
}

// Asynchronous 8-byte copy global -> shared; zeros when !in (no bytes
// read).
__device__ __forceinline__ void cp8(double *dst, const double *src, bool in)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(
                     (unsigned)__cvta_generic_to_shared(dst)),
                 "l"(src), "r"(in ? 8 : 0)
                 : "memory");
}

__device__ __forceinline__ void cp_wait_all()
{
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// C (rows x cols, pitch ldc) -= P Q over kd terms, P(r, k) = P[r psr + k
// psk], Q(k, c) = Q[k qsk + c qsc]; operand entries beyond rows, cols or kd
// read as zero. Both operands are staged k-major in shared memory by
// asynchronous copies (all 32 of a thread in flight at once, each operand
// read along its unit-stride dimension); the thread's 16 elements of C are
// read while they land; every thread accumulates a 4 x 4 block of C.
__device__ void tile_sub(double *C, long ldc, int rows, int cols, int kd, const double *P,
                         long psr, long psk, const double *Q, long qsk, long qsc, double *sm)
{
    double(*Ps)[GP_SP] = reinterpret_cast<double(*)[GP_SP]>(sm);
    double(*Qs)[GP_SP] = reinterpret_cast<double(*)[GP_SP]>(sm + GP_NB * GP_SP);
    const int t = threadIdx.x;
    const bool pk = psk == 1, qk = qsk == 1;
#pragma unroll
    for (int u = 0; u < 16; u++) {
        const int e = t + GP_T * u, hi = e / GP_NB, lo = e % GP_NB;
        int r = pk ? hi : lo, k = pk ? lo : hi;
        bool in = r < rows && k < kd;
        cp8(&Ps[k][r], in ? P + r * psr + k * psk : P, in);
        r = qk ? hi : lo;
        k = qk ? lo : hi;
        in = r < cols && k < kd;
        cp8(&Qs[k][r], in ? Q + k * qsk + r * qsc : Q, in);
    }
    const int tx = t % 16, ty = t / 16;
    double c0[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int r = ty + 16 * i, cc = tx + 16 * c;
            c0[i][c] = r < rows && cc < cols ? C[r * ldc + cc] : 0.0;
        }
    cp_wait_all();
    __syncthreads();
#pragma unroll 8
    for (int k = 0; k < GP_NB; k++) {
        double a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            a[i] = Ps[k][ty + 16 * i];
            b[i] = Qs[k][tx + 16 * i];
        }
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int c = 0; c < 4; c++)
                c0[i][c] = fma(-a[i], b[c], c0[i][c]);
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = ty + 16 * i;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const int cc = tx + 16 * c;
            if (r < rows && cc < cols)
                C[r * ldc + cc] = c0[i][c];
        }
    }
    // The staging may be reused, and C's new values are visible to the
    // whole CTA.
    __syncthreads();
}

// Position of entry m of row k in a staged triangular factor.
__device__ __forceinline__ int lpos(int k, int m)
{
    return k * GP_LP + (m >> 4) * GP_QP + (m & 15);
}

// Stages the strictly lower part of the factor L_jj (A's block (j, j);
// zeros on and above the diagonal and beyond the block's b rows) into sm:
// transposed (row k = column k of L) for the forward substitution, as is
// for the backward one; then the reciprocals 1 / L_kk (1 beyond b) at sm +
// 64 GP_LP.
template <bool FWD>
__device__ void stage_factor(const Gp &g, int j, double *sm)
{
    const int j0 = j * GP_NB, b = block_rows(g.n, j);
    const double *Ab = g.A + (long)j0 * g.n + j0;
#pragma unroll
    for (int u = 0; u < GP_NB * GP_NB / GP_T; u++) {
        const int e = threadIdx.x + GP_T * u, r = e / GP_NB, c = e % GP_NB;
        const bool in = c < r && r < b;
        cp8(sm + (FWD ? lpos(c, r) : lpos(r, c)), in ? Ab + (long)r * g.n + c : Ab, in);
    }
    if (threadIdx.x < GP_NB)
        sm[GP_NB * GP_LP + threadIdx.x] = threadIdx.x < b ? g.rd[j0 + threadIdx.x] : 1.0;
    cp_wait_all();
    __syncthreads();
}

// Solves L y = v (FWD) or L^T y = v in place for the 64-vector v held by
// the four threads (lane & ~3) + 0..3 of a warp, quarter q holding entries
// 16 q .. 16 q + 15. Ls is the staged strictly lower factor (transposed for
// FWD: row k holds L_mk; else row k holds L_km; zero elsewhere), rd the
// reciprocals of its diagonal. Step k: the quarter that holds entry k
// scales it by 1 / L_kk, the shuffle hands the result to the other three,
// and every thread subtracts its multiples from all its entries: the zeros
// of the staged factor leave the entries already solved (and entry k)
// unchanged, so that the 64 steps carry no branch.
template <bool FWD>
__device__ __forceinline__ void tri_solve(double v[16], int q, const double *Ls, const double *rd)
{
    const int base = (int)(threadIdx.x & 31) & ~3;
    const double *lq = Ls + q * GP_QP;
#pragma unroll
    for (int s = 0; s < GP_NB; s++) {
        const int k = FWD ? s : GP_NB - 1 - s;
        const int qk = k >> 4, ik = k & 15;
        double y = v[ik] * rd[k];
        y = __shfl_sync(0xffffffffu, y, base | qk);
        v[ik] = q == qk ? y : v[ik];
        const double *lk = lq + k * GP_LP;
#pragma unroll
        for (int u = 0; u < 16; u += 2) {
            const double2 l = *reinterpret_cast<const double2 *>(lk + u);
            v[u] = fma(-l.x, y, v[u]);
            v[u + 1] = fma(-l.y, y, v[u + 1]);
        }
    }
}

// The diagonal block j: the update of block column j - 1 (j > 0), then its
// factorization in shared memory, 16 columns at a time. Warp 0 factors the
// 16-column panel (rows c0 .. 63) in registers, lane l holding rows c0 + l
// and c0 + 32 + l: at step k the pivot comes from lane k by a shuffle, the
// column is scaled by the pivot's inverse square root, and the entries
// L_c,k of the panel's own rows reach every lane by shuffles, so that the
// 16 steps need no barrier. Then all warps subtract the panel's product
// from the trailing lower triangle. Finally L into A's block and 1 / L_kk
// into rd. The staged upper triangle is zero, so that the lanes' updates
// of entries above the diagonal stay finite (they are never read).
__device__ void diag_factor(const Gp &g, int j, double *sm)
{
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int j0 = j * GP_NB, b = block_rows(g.n, j);
    double *Ab = g.A + (long)j0 * g.n + j0;
    if (j > 0)
        tile_sub(Ab, g.n, b, b, GP_NB, Ab - GP_NB, g.n, 1, Ab - GP_NB, 1, g.n, sm);
    double(*S)[GP_SP] = reinterpret_cast<double(*)[GP_SP]>(sm);
    double *rs = sm + GP_NB * GP_SP;  // 1 / L_kk
#pragma unroll
    for (int u = 0; u < GP_NB * GP_NB / GP_T; u++) {
        const int e = t + GP_T * u, r = e / GP_NB, c = e % GP_NB;
        const bool in = c <= r && r < b;
        cp8(&S[r][c], in ? Ab + (long)r * g.n + c : Ab, in);
    }
    cp_wait_all();
    // Identity beyond the block's rows.
    if (t >= b && t < GP_NB)
        S[t][t] = 1.0;
    __syncthreads();
    for (int p = 0; p < GP_NB / 16; p++) {
        const int c0 = 16 * p;
        if (warp == 0) {
            const int r0 = c0 + lane, r1 = c0 + 32 + lane;
            double a0[16], a1[16];
#pragma unroll
            for (int c = 0; c < 16; c++) {
                a0[c] = r0 < GP_NB ? S[r0][c0 + c] : 0.0;
                a1[c] = r1 < GP_NB ? S[r1][c0 + c] : 0.0;
            }
#pragma unroll
            for (int k = 0; k < 16; k++) {
                double d = __shfl_sync(0xffffffffu, a0[k], k);
                if (!(d > 0.0)) {
                    if (lane == 0 && c0 + k < b)
                        *g.flag = 1;
                    d = 1.0;
                }
                const double r = rsqrt(d);
                a0[k] *= r;
                a1[k] *= r;
                if (lane == 0)
                    rs[c0 + k] = r;
#pragma unroll
                for (int c = k + 1; c < 16; c++) {
                    const double lc = __shfl_sync(0xffffffffu, a0[k], c);
                    a0[c] = fma(-a0[k], lc, a0[c]);
                    a1[c] = fma(-a1[k], lc, a1[c]);
                }
            }
#pragma unroll
            for (int c = 0; c < 16; c++) {
                if (r0 < GP_NB)
                    S[r0][c0 + c] = a0[c];
                if (r1 < GP_NB)
                    S[r1][c0 + c] = a1[c];
            }
        }
        __syncthreads();
        // Trailing lower triangle: S_im -= sum_k L_i,k L_m,k over the panel.
        const int t0 = c0 + 16, R = GP_NB - t0;
        for (int e = t; e < R * R; e += GP_T) {
            const int i = t0 + e / R, m = t0 + e % R;
            if (m <= i) {
                double acc = S[i][m];
#pragma unroll
                for (int k = 0; k < 16; k++)
                    acc = fma(-S[i][c0 + k], S[m][c0 + k], acc);
                S[i][m] = acc;
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int u = 0; u < GP_NB * GP_NB / GP_T; u++) {
        const int e = t + GP_T * u, r = e / GP_NB, c = e % GP_NB;
        if (c <= r && r < b)
            Ab[(long)r * g.n + c] = S[r][c];
    }
    if (t < b)
        g.rd[j0 + t] = rs[t];
}

// Step j of the factorization: CTA 0 the diagonal block; CTAs 1 .. T - 1
// the lower blocks (i, k), j <= k <= i, other than (j, j), of the trailing
// matrix; then the right-hand-side blocks (i, column block c), i >= j, all
// with the update of block column j - 1 (A -= L_i,j-1 L_k,j-1^T, F_i -=
// L_i,j-1 Z_j-1).
__global__ void __launch_bounds__(GP_T) gp_factor_k(Gp g, int j)
{
    extern __shared__ __align__(16) double gp_sm[];
    if (blockIdx.x == 0) {
        diag_factor(g, j, gp_sm);
        return;
    }
    const int p0 = (j - 1) * GP_NB, m = g.nb - j;
    const long nk = (long)m * (m + 1) / 2;
    const long e = blockIdx.x;
    if (e < nk) {
        int ii = (int)((sqrt(8.0 * (double)e + 1.0) - 1.0) * 0.5);
        while ((long)(ii + 1) * (ii + 2) / 2 <= e)
            ii++;
        while ((long)ii * (ii + 1) / 2 > e)
            ii--;
        const int kk = (int)(e - (long)ii * (ii + 1) / 2);
        const int i0 = (j + ii) * GP_NB, k0 = (j + kk) * GP_NB;
        tile_sub(g.A + (long)i0 * g.n + k0, g.n, block_rows(g.n, j + ii),
                 block_rows(g.n, j + kk), GP_NB, g.A + (long)i0 * g.n + p0, g.n, 1,
                 g.A + (long)k0 * g.n + p0, 1, g.n, gp_sm);
        return;
    }
    const long f = e - nk;
    const int i = j + (int)(f / g.db), c0 = (int)(f % g.db) * GP_NB, i0 = i * GP_NB;
    tile_sub(g.R + (long)i0 * g.d + c0, g.d, block_rows(g.n, i), min(GP_NB, g.d - c0), GP_NB,
             g.A + (long)i0 * g.n + p0, g.n, 1, g.R + (long)p0 * g.d + c0, g.d, 1, gp_sm);
}

// Block column j: CTAs 0 .. nb - j - 2 the rows of the blocks below the
// diagonal (L_ij = A_ij L_jj^-T: each row solved against L_jj); then one
// CTA per 64 right-hand-side columns, Z_j = L_jj^-1 F_j.
__global__ void __launch_bounds__(GP_T) gp_panel_k(Gp g, int j)
{
    extern __shared__ __align__(16) double gp_sm[];
    stage_factor<true>(g, j, gp_sm);
    const int t = threadIdx.x, q = t & 3, vi = t >> 2;
    const int j0 = j * GP_NB, b = block_rows(g.n, j), nk = g.nb - 1 - j;
    const double *rd = gp_sm + GP_NB * GP_LP;
    double v[16];
    if ((int)blockIdx.x < nk) {
        const int i = j + 1 + blockIdx.x, rows = block_rows(g.n, i);
        double *row = g.A + (long)(i * GP_NB + vi) * g.n + j0 + 16 * q;
        // Scalar accesses: the rows are 16-byte aligned only for even n.
        const bool in = vi < rows;
#pragma unroll
        for (int u = 0; u < 16; u++)
            v[u] = in ? row[u] : 0.0;
        tri_solve<true>(v, q, gp_sm, rd);
        if (in)
#pragma unroll
            for (int u = 0; u < 16; u++)
                row[u] = v[u];
        return;
    }
    const int c = ((int)blockIdx.x - nk) * GP_NB + vi;
    double *col = g.R + (long)(j0 + 16 * q) * g.d + c;
#pragma unroll
    for (int u = 0; u < 16; u++)
        v[u] = c < g.d && 16 * q + u < b ? col[(long)u * g.d] : 0.0;
    tri_solve<true>(v, q, gp_sm, rd);
#pragma unroll
    for (int u = 0; u < 16; u++)
        if (c < g.d && 16 * q + u < b)
            col[(long)u * g.d] = v[u];
}

// Backward step j: CTAs 0 .. db - 1 take Z_j's 64-column blocks, subtract
// L_j+1,j^T X_j+1 (j < nb - 1) and solve L_jj^T X_j = Z_j, storing X_j in
// double and in float; the other CTAs subtract L_j+1,i^T X_j+1 from the
// blocks Z_i, i < j.
__global__ void __launch_bounds__(GP_T) gp_back_k(Gp g, int j)
{
    extern __shared__ __align__(16) double gp_sm[];
    const int j0 = j * GP_NB, b = block_rows(g.n, j);
    const bool next = j + 1 < g.nb;
    const int k0 = j0 + GP_NB, kd = next ? block_rows(g.n, j + 1) : 0;
    if ((int)blockIdx.x >= g.db) {
        const int e = (int)blockIdx.x - g.db, i0 = (e / g.db) * GP_NB, c0 = (e % g.db) * GP_NB;
        tile_sub(g.R + (long)i0 * g.d + c0, g.d, GP_NB, min(GP_NB, g.d - c0), kd,
                 g.A + (long)k0 * g.n + i0, 1, g.n, g.R + (long)k0 * g.d + c0, g.d, 1, gp_sm);
        return;
    }
    const int c0 = (int)blockIdx.x * GP_NB;
    if (next)
        tile_sub(g.R + (long)j0 * g.d + c0, g.d, b, min(GP_NB, g.d - c0), kd,
                 g.A + (long)k0 * g.n + j0, 1, g.n, g.R + (long)k0 * g.d + c0, g.d, 1, gp_sm);
    stage_factor<false>(g, j, gp_sm);
    const int t = threadIdx.x, q = t & 3, c = c0 + (t >> 2);
    double v[16];
    const long off = (long)(j0 + 16 * q) * g.d + c;
#pragma unroll
    for (int u = 0; u < 16; u++)
        v[u] = c < g.d && 16 * q + u < b ? g.R[off + (long)u * g.d] : 0.0;
    tri_solve<false>(v, q, gp_sm, gp_sm + GP_NB * GP_LP);
#pragma unroll
    for (int u = 0; u < 16; u++)
        if (c < g.d && 16 * q + u < b) {
            g.R[off + (long)u * g.d] = v[u];
            g.X[off + (long)u * g.d] = (float)v[u];
        }
}

// A = K + noise I (lower triangle in double), R = F in double.
__global__ void gp_init_k(const float *K, const float *F, Gp g, double noise)
{
    const long nn = (long)g.n * g.n, nd = (long)g.n * g.d;
    for (long e = (long)blockIdx.x * blockDim.x + threadIdx.x; e < nn + nd;
         e += (long)gridDim.x * blockDim.x) {
        if (e < nn) {
            const long i = e / g.n, c = e % g.n;
            if (c <= i)
                g.A[e] = (double)K[e] + (i == c ? noise : 0.0);
        }
        else
            g.R[e - nn] = F[e - nn];
    }
}

bool opt_in_all()
{
    static unsigned mask = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (mask >> (dev & 31) & 1)
        return true;
    for (const void *fn : {(const void *)gp_factor_k, (const void *)gp_panel_k,
                           (const void *)gp_back_k})
        if (!cuda_ok(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)GP_SMEM),
                     "gp kernels"))
            return false;
    mask |= 1u << (dev & 31);
    return true;
}

}  // namespace

// Work: A (n x n), R (n x d) and the n reciprocals, in doubles.
size_t gp_work_doubles(int n, int d)
{
    return (size_t)n * n + (size_t)n * d + (size_t)n;
}

void gp_solve_dev(cudaStream_t st, const float *K, int n, const float *F_in, int d,
                  double noise, float *X_out, double *work, int *flag)
{
    if (!opt_in_all())
        return;
    Gp g;
    g.A = work;
    g.R = work + (size_t)n * n;
    g.rd = g.R + (size_t)n * d;
    g.X = X_out;
    g.n = n;
    g.d = d;
    g.nb = (int)cdiv(n, GP_NB);
    g.db = (int)cdiv(d, GP_NB);
    g.flag = flag;
    const long total = (long)n * n + (long)n * d;
    gp_init_k<<<(int)std::min<long>(cdiv(total, 256), 148 * 16), 256, 0, st>>>(K, F_in, g, noise);
    for (int j = 0; j < g.nb; j++) {
        const long m = g.nb - j;
        const long grid = j == 0 ? 1 : m * (m + 1) / 2 + m * g.db;
        gp_factor_k<<<(unsigned)grid, GP_T, GP_SMEM, st>>>(g, j);
        gp_panel_k<<<(unsigned)(m - 1 + g.db), GP_T, GP_SMEM, st>>>(g, j);
    }
    for (int j = g.nb - 1; j >= 0; j--) {
        const int grid = g.db + (j + 1 < g.nb ? j * g.db : 0);
        gp_back_k<<<grid, GP_T, GP_SMEM, st>>>(g, j);
    }
}

}  // namespace coreg
