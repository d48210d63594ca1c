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
// place in R. Three kernels:
//   gp_factor_k (j)  CTA 0: the diagonal block j receives the update of
//                    block column j - 1 and is factored (L_jj, the
//                    reciprocals 1 / L_kk and the inverse L_jj^-1, by
//                    block inversion); the other CTAs apply the same
//                    update to the rest of the trailing matrix (lower
//                    blocks) and to the right-hand sides below block j-1;
//   gp_panel_k (j)   the blocks below the diagonal, L_ij = A_ij L_jj^-T,
//                    and Z_j = L_jj^-1 F_j, as products with the inverse
//                    L_jj^-1 that the diagonal factor stored, each block's
//                    product split over four CTAs;
//   gp_back_k (j)    from the last block up: Z_j receives the update of
//                    X_{j+1} and X_j = L_jj^-T Z_j (products with the
//                    operands staged in one round, the second with the
//                    stored inverse; also rounded to float into the
//                    output), while the other CTAs apply X_{j+1}'s update
//                    to Z_i, i < j (Z_j in 16-column slabs, four CTAs a
//                    block).
// The diagonal block is factored 16 columns at a time, each panel by one
// warp in registers, and inverted by block inversion (a 16-step chain);
// everything else is 64 x 64 block products. Operands are staged in shared
// memory by asynchronous copies. Every chain here is latency-bound (one
// pivot after another), so the kernels are written for short dependency
// chains and few instructions per step.
// A non-positive pivot sets *flag (the reference stops with "kernel not
// positive definite"); the host reads it after the tile.

#include "common.cuh"

namespace coreg {

#define GP_NB 64

namespace {

constexpr int GP_T = 256;         // threads per CTA
constexpr int GP_SP = GP_NB + 1;  // pitch of the staged product operands and of the block
// Staging: two padded 64 x 64 blocks, then (diagonal factor) 64
// reciprocals and a 32 x 32 scratch block.
constexpr int GP_RS = 2 * GP_NB * GP_SP, GP_US = GP_RS + GP_NB;
constexpr size_t GP_SMEM = (GP_US + 32 * 32) * sizeof(double);
static_assert(2 * GP_NB * 68 <= GP_US + 32 * 32, "tile_sub's staging fits");

struct Gp {
    double *A;   // n x n, pitch n: K + noise I (lower triangle), then L
    double *R;   // n x d: F, then Z, then X
    double *rd;  // n: 1 / L_kk
    double *Li;  // nb blocks of 64 x 64: the inverses L_jj^-1, row-major
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

// Programmatic dependent launch across the chain of kernels: the next
// kernel may be scheduled as soon as every CTA of this one has started,
// and waits (griddepcontrol.wait) until this one has completed and its
// writes are visible, before it reads anything. Launch gaps overlap the
// previous kernel's tail.
__device__ __forceinline__ void chain_enter()
{
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Pitch of tile_sub's staged operands: with 68, the eight rows times four
// k of a warp's fragment loads fall on distinct banks in each half warp.
constexpr int GP_TP = 68;

// D += A B on the double-precision tensor cores (m8n8k4): a = A[g][q], b =
// B[q][g], d = D[g][2 q .. 2 q + 1] with g = lane / 4, q = lane % 4.
__device__ __forceinline__ void dmma(double d[2], double a, double b)
{
    asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
                 : "+d"(d[0]), "+d"(d[1])
                 : "d"(a), "d"(b));
}

// C (rows x cols, pitch ldc) -= P Q over kd terms (C = P Q with ASSIGN,
// and then also Cf = C in float where Cf is given), P(r, k) = P[r psr + k
// psk], Q(k, c) = Q[k qsk + c qsc]; operand entries beyond rows, cols or kd
// read as zero. Both operands are staged k-major in shared memory by
// asynchronous copies (all 32 of a thread in flight at once, each operand
// read along its unit-stride dimension) before C is written, so that Q may
// be C itself; the thread's 16 elements of C are read while they land. The
// product runs on the double-precision tensor cores: warp w owns the rows 8
// w .. 8 w + 7 and all eight 8-column tiles.
template <bool ASSIGN = false>
__device__ void tile_sub(double *C, long ldc, int rows, int cols, int kd, const double *P,
                         long psr, long psk, const double *Q, long qsk, long qsc, double *sm,
                         float *Cf = nullptr, double *Cs = nullptr)
{
    double *Ps = sm, *Qs = sm + GP_NB * GP_TP;  // Ps[k][r], Qs[k][c]
    const int t = threadIdx.x;
    const bool pk = psk == 1, qk = qsk == 1;
#pragma unroll
    for (int u = 0; u < 16; u++) {
        const int e = t + GP_T * u, hi = e / GP_NB, lo = e % GP_NB;
        int r = pk ? hi : lo, k = pk ? lo : hi;
        bool in = r < rows && k < kd;
        cp8(Ps + k * GP_TP + r, in ? P + r * psr + k * psk : P, in);
        r = qk ? hi : lo;
        k = qk ? lo : hi;
        in = r < cols && k < kd;
        cp8(Qs + k * GP_TP + r, in ? Q + k * qsk + r * qsc : Q, in);
    }
    const int w = t >> 5, lane = t & 31, gr = lane >> 2, q = lane & 3, r = 8 * w + gr;
    double acc[8][2];
#pragma unroll
    for (int n = 0; n < 8; n++)
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const int cc = 8 * n + 2 * q + i;
            acc[n][i] = !ASSIGN && r < rows && cc < cols ? C[r * ldc + cc] : 0.0;
        }
    cp_wait_all();
    __syncthreads();
#pragma unroll 4
    for (int k4 = 0; k4 < GP_NB / 4; k4++) {
        const double *pr = Ps + (4 * k4 + q) * GP_TP, *qr = Qs + (4 * k4 + q) * GP_TP;
        const double a = ASSIGN ? pr[8 * w + gr] : -pr[8 * w + gr];
#pragma unroll
        for (int n = 0; n < 8; n++)
            dmma(acc[n], a, qr[8 * n + gr]);
    }
    if (Cs) {
        // The result into shared memory (pitch GP_SP, over the staging):
        // every warp has read its operands first.
        __syncthreads();
#pragma unroll
        for (int n = 0; n < 8; n++)
#pragma unroll
            for (int i = 0; i < 2; i++)
                Cs[r * GP_SP + 8 * n + 2 * q + i] = acc[n][i];
        __syncthreads();
        return;
    }
#pragma unroll
    for (int n = 0; n < 8; n++)
#pragma unroll
        for (int i = 0; i < 2; i++) {
            const int cc = 8 * n + 2 * q + i;
            if (r < rows && cc < cols) {
                C[r * ldc + cc] = acc[n][i];
                if (Cf)
                    Cf[r * ldc + cc] = (float)acc[n][i];
            }
        }
    // The staging may be reused, and C's new values are visible to the
    // whole CTA.
    __syncthreads();
}

// A slab of a 64 x 64 block product on one CTA, four outputs a thread:
// C (R x CC, CC = 1024 / R, pitch ldc) -= P Q over kd terms (C = P Q with
// ASSIGN, and then Cf = C in float where Cf is given), P(r, k) = P[r psr +
// k psk] (R x 64), Q(k, c) = Q[k qsk + c qsc] (64 x CC); entries beyond
// rows, cols or kd read as zero. R = 64 with CC = 16 (a column slab) or R =
// 16 with CC = 64 (a row slab): a quarter of the block's work, so that four
// CTAs share one block product and each finishes four times sooner. The
// slab reads only its own rows of P and columns of Q, so that a product
// may overwrite its operand slab by slab.
template <int R, bool ASSIGN>
__device__ void slab_prod(double *C, long ldc, int rows, int cols, int kd, const double *P,
                          long psr, long psk, const double *Q, long qsk, long qsc, double *sm,
                          float *Cf = nullptr)
{
    constexpr int CC = GP_NB * GP_NB / 4 / R, RP = R + 1, CP = CC + 1, RT = GP_T / CC;
    double *Ps = sm;            // Ps[k * RP + r]
    double *Qs = sm + GP_NB * RP;  // Qs[k * CP + c]
    const int t = threadIdx.x;
    const bool pk = psk == 1, qk = qsk == 1;
#pragma unroll
    for (int u = 0; u < R * GP_NB / GP_T; u++) {
        const int e = t + GP_T * u;
        const int r = pk ? e / GP_NB : e % R, k = pk ? e % GP_NB : e / R;
        const bool in = r < rows && k < kd;
        cp8(Ps + k * RP + r, in ? P + r * psr + k * psk : P, in);
    }
#pragma unroll
    for (int u = 0; u < CC * GP_NB / GP_T; u++) {
        const int e = t + GP_T * u;
        const int c = qk ? e / GP_NB : e % CC, k = qk ? e % GP_NB : e / CC;
        const bool in = c < cols && k < kd;
        cp8(Qs + k * CP + c, in ? Q + k * qsk + c * qsc : Q, in);
    }
    const int tx = t % CC, ty = t / CC;
    double acc[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = ty + RT * i;
        acc[i] = !ASSIGN && r < rows && tx < cols ? C[r * ldc + tx] : 0.0;
    }
    cp_wait_all();
    __syncthreads();
#pragma unroll 16
    for (int k = 0; k < GP_NB; k++) {
        const double q = Qs[k * CP + tx];
#pragma unroll
        for (int i = 0; i < 4; i++)
            acc[i] = fma(ASSIGN ? Ps[k * RP + ty + RT * i] : -Ps[k * RP + ty + RT * i], q, acc[i]);
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = ty + RT * i;
        if (r < rows && tx < cols) {
            C[r * ldc + tx] = acc[i];
            if (Cf)
                Cf[r * ldc + tx] = (float)acc[i];
        }
    }
    __syncthreads();
}

// One join of the block inversion at width W: for each pair of W x W
// diagonal blocks of the inverse at o and o + W, the block below them,
// -C^-1 (B A^-1), with B the factor's block there. Every thread computes
// NC columns of one row, NC independent sums.
template <int W>
__device__ __forceinline__ void invert_join(double (*S)[GP_SP], double (*T)[GP_SP],
                                            double (*U)[32])
{
    constexpr int P = GP_NB / (2 * W), NC = P * W * W / GP_T, PER = W * W / NC;
    const int t = threadIdx.x, pr = t / PER, rem = t % PER, r = rem / (W / NC),
              c0 = (rem % (W / NC)) * NC, o = 2 * W * pr;
    double acc[NC];
#pragma unroll
    for (int i = 0; i < NC; i++)
        acc[i] = 0.0;
#pragma unroll
    for (int k = 0; k < W; k++) {
        const double bk = S[o + W + r][o + k];
#pragma unroll
        for (int i = 0; i < NC; i++)
            acc[i] = fma(bk, T[o + k][o + c0 + i], acc[i]);
    }
#pragma unroll
    for (int i = 0; i < NC; i++)
        U[pr * W + r][c0 + i] = acc[i];
    __syncthreads();
#pragma unroll
    for (int i = 0; i < NC; i++)
        acc[i] = 0.0;
#pragma unroll
    for (int k = 0; k < W; k++) {
        const double ck = T[o + W + r][o + W + k];
#pragma unroll
        for (int i = 0; i < NC; i++)
            acc[i] = fma(ck, U[pr * W + k][c0 + i], acc[i]);
    }
#pragma unroll
    for (int i = 0; i < NC; i++)
        T[o + W + r][o + c0 + i] = -acc[i];
    __syncthreads();
}

__device__ void invert_factor(double (*S)[GP_SP], const double *rs, double *sm, double *Li)
{
    const int t = threadIdx.x;
    double(*T)[GP_SP] = reinterpret_cast<double(*)[GP_SP]>(sm + GP_NB * GP_SP);
    double(*U)[32] = reinterpret_cast<double(*)[32]>(sm + GP_US);
    // Zeros above the diagonal blocks as they are built.
    for (int e = t; e < GP_NB * GP_SP; e += GP_T)
        (&T[0][0])[e] = 0.0;
    __syncthreads();
    if (t < GP_NB) {
        // Diagonal block p, column c: D y = e_c, right-looking (each step
        // one multiply, then independent updates of the later entries).
        const int p = t >> 4, c = t & 15, o = 16 * p;
        double y[16];
#pragma unroll
        for (int m = 0; m < 16; m++)
            y[m] = m == c ? 1.0 : 0.0;
#pragma unroll
        for (int m = 0; m < 16; m++) {
            y[m] *= rs[o + m];
#pragma unroll
            for (int q = m + 1; q < 16; q++)
                y[q] = fma(-S[o + q][o + m], y[m], y[q]);
        }
#pragma unroll
        for (int m = 0; m < 16; m++)
            T[o + m][o + c] = y[m];
    }
    __syncthreads();
    invert_join<16>(S, T, U);
    invert_join<32>(S, T, U);
    for (int e = t; e < GP_NB * GP_NB; e += GP_T)
        Li[e] = T[e >> 6][e & 63];
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
    double(*S)[GP_SP] = reinterpret_cast<double(*)[GP_SP]>(sm);
    double *rs = sm + GP_RS;  // 1 / L_kk
    if (j > 0) {
        // The update of block column j - 1 straight into S (rows and
        // columns beyond b come out zero).
        tile_sub(Ab, g.n, b, b, GP_NB, Ab - GP_NB, g.n, 1, Ab - GP_NB, 1, g.n, sm, nullptr,
                 &S[0][0]);
    }
    else {
#pragma unroll
        for (int u = 0; u < GP_NB * GP_NB / GP_T; u++) {
            const int e = t + GP_T * u, r = e / GP_NB, c = e % GP_NB;
            const bool in = c <= r && r < b;
            cp8(&S[r][c], in ? Ab + (long)r * g.n + c : Ab, in);
        }
        cp_wait_all();
        __syncthreads();
    }
    // Zeros above the diagonal, the identity beyond the block's rows.
#pragma unroll
    for (int u = 0; u < GP_NB * GP_NB / GP_T; u++) {
        const int e = t + GP_T * u, r = e / GP_NB, c = e % GP_NB;
        if (c > r || r >= b)
            S[r][c] = r == c ? 1.0 : 0.0;
    }
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
            // The scaled column's entries of the panel's own rows pass
            // through shared memory (two buffers, one warp barrier a step).
            double *colb = sm + GP_US;
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
                double *cb = colb + 16 * (k & 1);
                if (lane < 16)
                    cb[lane] = a0[k];
                __syncwarp();
#pragma unroll
                for (int c = k + 1; c < 16; c++) {
                    const double lc = cb[c];
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
    invert_factor(S, rs, sm, g.Li + (long)j * GP_NB * GP_NB);
}

// Step j of the factorization: CTA 0 the diagonal block; CTAs 1 .. T - 1
// the lower blocks (i, k), j <= k <= i, other than (j, j), of the trailing
// matrix; then the right-hand-side blocks (i, column block c), i >= j, all
// with the update of block column j - 1 (A -= L_i,j-1 L_k,j-1^T, F_i -=
// L_i,j-1 Z_j-1).
__global__ void __launch_bounds__(GP_T, 1) gp_factor_k(Gp g, int j)
{
    extern __shared__ __align__(16) double gp_sm[];
    chain_enter();
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

// Block column j, products with the inverse that the diagonal factor
// stored, each block split over four CTAs (blockIdx.y = slab): CTAs 0 ..
// nb - j - 2 the blocks below the diagonal, L_ij = A_ij L_jj^-T (16-row
// slabs, each overwriting its own rows); then one CTA per 64
// right-hand-side columns, Z_j = L_jj^-1 F_j (16-column slabs).
__global__ void __launch_bounds__(GP_T) gp_panel_k(Gp g, int j)
{
    extern __shared__ __align__(16) double gp_sm[];
    chain_enter();
    const int j0 = j * GP_NB, b = block_rows(g.n, j), nk = g.nb - 1 - j, sl = 16 * blockIdx.y;
    const double *li = g.Li + (long)j * GP_NB * GP_NB;
    if ((int)blockIdx.x < nk) {
        const int i = j + 1 + (int)blockIdx.x, rows = block_rows(g.n, i) - sl;
        if (rows <= 0)
            return;
        double *blk = g.A + (long)(i * GP_NB + sl) * g.n + j0;
        // (L_jj^-T)_kc = Li[c][k].
        slab_prod<16, true>(blk, g.n, min(16, rows), GP_NB, GP_NB, blk, g.n, 1, li, 1, GP_NB,
                            gp_sm);
        return;
    }
    const int c0 = ((int)blockIdx.x - nk) * GP_NB + sl;
    if (c0 >= g.d)
        return;
    double *zj = g.R + (long)j0 * g.d + c0;
    slab_prod<64, true>(zj, g.d, b, min(16, g.d - c0), b, li, GP_NB, 1, zj, g.d, 1, gp_sm);
}

// Shared memory of the backward kernel: two staged 64 x 64 blocks and two
// 64 x 16 slabs.
constexpr int GP_SL = 17;  // pitch of a staged 16-column slab
constexpr size_t GP_SMEM_BACK = (2 * GP_NB * GP_SP + 2 * GP_NB * GP_SL) * sizeof(double);

// X_j = L_jj^-T (Z_j - L_j+1,j^T X_j+1) for the 16 columns from c0 (no
// update for the last block), stored in double and in float. One round of
// asynchronous copies stages L_j+1,j, the inverse and the slab of X_j+1
// while the slab of Z_j comes into registers; the updated slab goes through
// shared memory into the second product. Thread (ty, tx): rows ty + 16 i,
// column tx.
__device__ void back_slab(const Gp &g, int j, int c0, double *sm)
{
    const int t = threadIdx.x, tx = t % 16, ty = t / 16;
    const int j0 = j * GP_NB, b = block_rows(g.n, j), cols = min(16, g.d - c0);
    const bool next = j + 1 < g.nb;
    const int k0 = j0 + GP_NB, kd = next ? block_rows(g.n, j + 1) : 0;
    double(*Ps)[GP_SP] = reinterpret_cast<double(*)[GP_SP]>(sm);
    double(*Ls)[GP_SP] = reinterpret_cast<double(*)[GP_SP]>(sm + GP_NB * GP_SP);
    double(*Qs)[GP_SL] = reinterpret_cast<double(*)[GP_SL]>(sm + 2 * GP_NB * GP_SP);
    double(*Zs)[GP_SL] = reinterpret_cast<double(*)[GP_SL]>(sm + 2 * GP_NB * GP_SP + GP_NB * GP_SL);
    const double *li = g.Li + (long)j * GP_NB * GP_NB;
    double *zj = g.R + (long)j0 * g.d + c0;
#pragma unroll
    for (int u = 0; u < GP_NB * GP_NB / GP_T; u++) {
        const unsigned e = t + GP_T * u;
        const int k = (int)(e >> 6), m = (int)(e & 63);
        // Ps[k][m] = L_j+1,j[k][m], Ls[k][m] = Li[k][m].
        const bool in = k < kd;
        cp8(&Ps[k][m], in ? g.A + (long)(k0 + k) * g.n + j0 + m : g.A, in);
        cp8(&Ls[k][m], li + e, true);
    }
#pragma unroll
    for (int u = 0; u < GP_NB * 16 / GP_T; u++) {
        const int e = t + GP_T * u, k = e / 16, c = e % 16;
        const bool in = k < kd && c < cols;
        cp8(&Qs[k][c], in ? g.R + (long)(k0 + k) * g.d + c0 + c : g.R, in);
    }
    double z[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = ty + 16 * i;
        z[i] = r < b && tx < cols ? zj[(long)r * g.d + tx] : 0.0;
    }
    cp_wait_all();
    __syncthreads();
    if (next) {
#pragma unroll 16
        for (int k = 0; k < GP_NB; k++) {
            const double q = Qs[k][tx];
#pragma unroll
            for (int i = 0; i < 4; i++)
                z[i] = fma(-Ps[k][ty + 16 * i], q, z[i]);
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++)
        Zs[ty + 16 * i][tx] = z[i];
    __syncthreads();
    double x[4] = {0.0, 0.0, 0.0, 0.0};
#pragma unroll 16
    for (int k = 0; k < GP_NB; k++) {
        const double q = Zs[k][tx];
#pragma unroll
        for (int i = 0; i < 4; i++)
            x[i] = fma(Ls[k][ty + 16 * i], q, x[i]);
    }
    float *xf = g.X + (long)j0 * g.d + c0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = ty + 16 * i;
        if (r < b && tx < cols) {
            zj[(long)r * g.d + tx] = x[i];
            xf[(long)r * g.d + tx] = (float)x[i];
        }
    }
}

// Backward step j: CTAs 0 .. 4 db - 1 take Z_j's 16-column slabs
// (back_slab: the update by X_j+1 and the product with the inverse, X_j =
// L_jj^-T Z_j; split four ways, they are the step's critical path); the
// other CTAs subtract L_j+1,i^T X_j+1 from the whole 64 x 64 blocks Z_i, i <
// j (whole blocks read each factor block once).
__global__ void __launch_bounds__(GP_T) gp_back_k(Gp g, int j)
{
    extern __shared__ __align__(16) double gp_sm[];
    chain_enter();
    if ((int)blockIdx.x < 4 * g.db) {
        const int c0 = (int)blockIdx.x * 16;
        if (c0 < g.d)
            back_slab(g, j, c0, gp_sm);
        return;
    }
    const int k0 = (j + 1) * GP_NB, kd = block_rows(g.n, j + 1);
    const int e = (int)blockIdx.x - 4 * g.db, i0 = (e / g.db) * GP_NB, c0 = (e % g.db) * GP_NB;
    tile_sub(g.R + (long)i0 * g.d + c0, g.d, GP_NB, min(GP_NB, g.d - c0), kd,
             g.A + (long)k0 * g.n + i0, 1, g.n, g.R + (long)k0 * g.d + c0, g.d, 1, gp_sm);
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
    for (const void *fn : {(const void *)gp_factor_k, (const void *)gp_panel_k})
        if (!cuda_ok(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)GP_SMEM),
                     "gp kernels"))
            return false;
    if (!cuda_ok(cudaFuncSetAttribute((const void *)gp_back_k,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)GP_SMEM_BACK),
                 "gp kernels"))
        return false;
    mask |= 1u << (dev & 31);
    return true;
}

// A kernel of the chain with programmatic stream serialization (see
// chain_enter).
void chain_launch(void (*k)(Gp, int), dim3 grid, size_t smem, cudaStream_t st, Gp g, int j)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(GP_T);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, k, g, j);
}

}  // namespace

// Work: A (n x n), R (n x d), the n reciprocals and the block inverses, in
// doubles.
size_t gp_work_doubles(int n, int d)
{
    return (size_t)n * n + (size_t)n * d + (size_t)n + (size_t)cdiv(n, GP_NB) * GP_NB * GP_NB;
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
    g.Li = g.rd + n;
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
        chain_launch(gp_factor_k, dim3((unsigned)grid), GP_SMEM, st, g, j);
        chain_launch(gp_panel_k, dim3((unsigned)(m - 1 + g.db), 4), GP_SMEM, st, g, j);
    }
    for (int j = g.nb - 1; j >= 0; j--) {
        const int grid = 4 * g.db + (j + 1 < g.nb ? j * g.db : 0);
        chain_launch(gp_back_k, dim3(grid), GP_SMEM_BACK, st, g, j);
    }
}

}  // namespace coreg
