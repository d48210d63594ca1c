// SPDX-License-Identifier: Unlicense
//
// AdaLAM outlier filtering of nearest-neighbour matches (adalam.h), with
// the results of the reference's adalam.c (which follows
// kornia.feature.adalam step by step): seeds (adalam.c:336-350),
// neighbourhoods (:352-369), the problems' samples (:392-420), the
// hypotheses through kornia's "first k couples" (:225-244, :422-446), the
// half-precision duplicate weights (:130-177, :448-460), the
// confidence-based inlier selection (:179-209, :462-476), the refit
// (:478-541) and the acceptance (:543-560).
//
// The nearest neighbours come from the device (desc_nearest). Seeds and
// neighbourhoods are built on the host (O(n^2) comparisons). The two
// RANSAC passes, which are nearly all of the work (every hypothesis of
// every neighbourhood: residuals, a sort, then the duplicate test or the
// inlier selection), run on the device with one CTA per (hypothesis,
// neighbourhood); the O(N) steps between them (duplicate weights, the
// best hypothesis, the refit, the final selection) run on the host.
// adalam_filter without a device runs the same passes on host threads
// instead, problem by problem.
//
// A neighbourhood's hypotheses need only its own samples. The one
// coupling between neighbourhoods (the duplicate test compares the last
// sorted residual of one with the first of the next, as kornia's
// unique_consecutive over the concatenated columns does) is carried as
// each neighbourhood's first and last residual per hypothesis. Every
// floating-point expression keeps the reference's types and order, so
// that the matches and confidences agree bit for bit.

#include <cuda_fp16.h>
#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <thread>
#include <utility>
#include <vector>

#include "adalam.h"
#include "common.cuh"
#include "disk.h"

using coreg::fail;
using coreg::pending;

namespace {

// A value rounded to IEEE binary16 (to nearest, ties to even) and back:
// kornia compares the sorted residuals of the hypotheses in half
// precision. Bit arithmetic on the float: normal halves keep 10 mantissa
// bits, subnormal ones are multiples of 2^-24, 65520 and above overflow.
// Equal to the compiler's float -> _Float16 -> float conversion for all
// 2^32 inputs (checked exhaustively when this was written).
inline float via_half(float f)
{
    uint32_t u, r;
    memcpy(&u, &f, 4);
    const uint32_t sign = u & 0x80000000u, a = u & 0x7fffffffu;
    if (a >= 0x7f800000u)
        r = a;
    else if (a >= 0x477ff000u)
        r = 0x7f800000u;
    else if (a >= 0x38800000u)
        r = (a + 0xfffu + ((a >> 13) & 1u)) & 0xffffe000u;
    else {
        const float back = nearbyintf(fabsf(f) * 16777216.0f) / 16777216.0f;
        memcpy(&r, &back, 4);
    }
    r |= sign;
    float out;
    memcpy(&out, &r, 4);
    return out;
}

inline float sqdist(const float *a, const float *b)
{
    const float dx = a[0] - b[0], dy = a[1] - b[1];
    return dx * dx + dy * dy;
}

// Inverse of the 2 x 2 matrix (m0 m1; m2 m3), a determinant smaller than
// 1e-10 in magnitude replaced by 1e-10.
void inverse2(const double *m, double *o)
{
    double det = m[0] * m[3] - m[1] * m[2];
    if (fabs(det) < 1e-10)
        det = 1e-10;
    o[0] = m[3] / det;
    o[1] = -m[1] / det;
    o[2] = -m[2] / det;
    o[3] = m[0] / det;
}

// Radius of the seed circles: kornia takes the image to be the keypoints'
// bounding box when it is given no shape.
double seed_radius(const float *k, int n, double area_ratio)
{
    float x0 = FLT_MAX, y0 = FLT_MAX, x1 = -FLT_MAX, y1 = -FLT_MAX;
    for (int i = 0; i < n; i++) {
        x0 = fminf(x0, k[2 * i]);
        x1 = fmaxf(x1, k[2 * i]);
        y0 = fminf(y0, k[2 * i + 1]);
        y1 = fmaxf(y1, k[2 * i + 1]);
    }
    return sqrt((double)(x1 - x0) * (y1 - y0) / area_ratio / M_PI);
}

// kornia's draw_first_k_couples: every pair (a, b), b < a, of the first
// samples in order of a, then (rest, b) for b < rest.
void first_couples(int k, std::vector<int> &ca, std::vector<int> &cb)
{
    const int m = (int)(sqrt(2.0 * k + 0.25) - 0.5);
    const int rest = k - m * (m + 1) / 2;
    for (int a = 1; a <= m; a++)
        for (int b = 0; b < a; b++) {
            ca.push_back(a);
            cb.push_back(b);
        }
    for (int b = 0; b < rest; b++) {
        ca.push_back(rest);
        cb.push_back(b);
    }
}

struct Affine {
    float a00, a01, a10, a11;
};

// The neighbourhoods' samples, problem after problem, each problem's in
// ascending order of the match score: positions relative to the seed in
// both images over the search radius, and the keypoints they come from.
struct Samples {
    std::vector<int> off, len;  // Per problem.
    std::vector<float> x0, x1, y0, y1;
    std::vector<int> kp1, kp2;
    int count() const { return (int)x0.size(); }
};

// The affinity through samples a and b of a problem (ca, cb taken modulo
// its size): the transpose of X^-1 Y.
Affine hypothesis(const Samples &s, int r, int ca, int cb)
{
    const int a = s.off[r] + ca % s.len[r], b = s.off[r] + cb % s.len[r];
    const double X[4] = {s.x0[a], s.x1[a], s.x0[b], s.x1[b]};
    const double Y[4] = {s.y0[a], s.y1[a], s.y0[b], s.y1[b]};
    double Xi[4];
    inverse2(X, Xi);
    const double m00 = Xi[0] * Y[0] + Xi[1] * Y[2], m01 = Xi[0] * Y[1] + Xi[1] * Y[3];
    const double m10 = Xi[2] * Y[0] + Xi[3] * Y[2], m11 = Xi[2] * Y[1] + Xi[3] * Y[3];
    return {(float)m00, (float)m10, (float)m01, (float)m11};
}

// Per-thread scratch for one problem's residuals.
struct Scratch {
    std::vector<std::pair<float, int>> key;
    std::vector<int> order;
    std::vector<float> sq;
};

// The residuals |A x - y| of problem r, ascending (ties by sample index):
// sample indices into w.order, squared residuals into w.sq.
void sorted_residuals(const Samples &s, int r, const Affine &A, Scratch &w)
{
    const int o = s.off[r], n = s.len[r];
    w.key.resize(n);
    w.order.resize(n);
    w.sq.resize(n);
    for (int k = 0; k < n; k++) {
        const int t = o + k;
        const float px = A.a00 * s.x0[t] + A.a01 * s.x1[t];
        const float py = A.a10 * s.x0[t] + A.a11 * s.x1[t];
        w.key[k] = {hypotf(px - s.y0[t], py - s.y1[t]), t};
    }
    std::sort(w.key.begin(), w.key.end());
    for (int k = 0; k < n; k++) {
        w.order[k] = w.key[k].second;
        w.sq[k] = w.key[k].first * w.key[k].first;
    }
}

struct Selection {
    long cnt = -1;
    double bal = 0;
    float hi = 0;
};

// Confidence-based inlier selection on one problem's sorted squared
// residuals sq with column weights wt: the truncated weighted count of
// samples whose squared residual times min_conf stays within the
// progressive inlier rate, the weight total and the squared residual of
// the last counted sample. Residuals of at most 1e-8 count, weightless.
Selection select_inliers(const float *sq, const float *wt, int n, double min_conf)
{
    double b = 0, cum = 0, c = 0;
    for (int k = 0; k < n; k++)
        b += sq[k] <= 1e-8f ? 0.0 : wt[k];
    for (int k = 0; k < n; k++) {
        const bool perfect = sq[k] <= 1e-8f;
        const double w = perfect ? 0.0 : wt[k];
        cum += w;
        if (perfect || sq[k] * min_conf <= cum / b)
            c += w;
    }
    Selection sel;
    sel.cnt = (long)c;
    sel.bal = b;
    sel.hi = sel.cnt > 0 ? sq[sel.cnt - 1] : 0.0f;
    return sel;
}

// Column weights: 1 / the length of each run of columns equal to the next.
void duplicate_weights(const std::vector<unsigned char> &eq, std::vector<float> &w)
{
    const int N = (int)eq.size();
    w.resize(N);
    for (int j = 0; j < N;) {
        int e = j;
        while (e < N - 1 && eq[e])
            e++;
        const float v = 1.0f / (e - j + 1);
        for (int k = j; k <= e; k++)
            w[k] = v;
        j = e + 1;
    }
}

// Run body(r, scratch) for every problem r on up to 32 host threads.
template <class F>
void for_problems(int nr, F body)
{
    const int nt = std::max(1, std::min({nr, 32, (int)std::thread::hardware_concurrency()}));
    if (nt == 1) {
        Scratch w;
        for (int r = 0; r < nr; r++)
            body(r, w);
        return;
    }
    std::vector<std::thread> pool;
    for (int t = 0; t < nt; t++)
        pool.emplace_back([&, t] {
            Scratch w;
            for (int r = t; r < nr; r += nt)
                body(r, w);
        });
    for (auto &th : pool)
        th.join();
}

// Run fn(i) for every i < n on up to 32 host threads.
template <class F>
void parallel_for(int n, F fn)
{
    const int nt = std::max(1, std::min({n, 32, (int)std::thread::hardware_concurrency()}));
    if (nt == 1) {
        for (int i = 0; i < n; i++)
            fn(i);
        return;
    }
    std::vector<std::thread> pool;
    for (int t = 0; t < nt; t++)
        pool.emplace_back([&, t] {
            for (int i = t; i < n; i += nt)
                fn(i);
        });
    for (auto &th : pool)
        th.join();
}

struct Match {
    int i1, i2;
    float dist;
};

// The matches ordered by (i1, i2), the first of each repeated pair kept;
// returns their number.
int emit(std::vector<Match> &m, int **pairs, float **dist)
{
    std::stable_sort(m.begin(), m.end(), [](const Match &a, const Match &b) {
        return a.i1 != b.i1 ? a.i1 < b.i1 : a.i2 < b.i2;
    });
    *pairs = (int *)malloc((2 * m.size() + 2) * sizeof(int));
    *dist = (float *)malloc((m.size() + 1) * sizeof(float));
    int k = 0;
    for (size_t i = 0; i < m.size(); i++) {
        if (k > 0 && (*pairs)[2 * k - 2] == m[i].i1 && (*pairs)[2 * k - 1] == m[i].i2)
            continue;
        (*pairs)[2 * k] = m[i].i1;
        (*pairs)[2 * k + 1] = m[i].i2;
        (*dist)[k++] = m[i].dist;
    }
    return k;
}

// The least-squares affinity of a problem's inliers (the first cnt of
// order), the identity where its scale change exceeds det_thr.
Affine refit(const Samples &s, const int *order, long cnt, double det_thr)
{
    const double dt2 = det_thr * det_thr;
    double sxx[4] = {0, 0, 0, 0}, syx[4] = {0, 0, 0, 0}, xi[4];
    for (long k = 0; k < cnt; k++) {
        const int t = order[k];
        const double x0 = s.x0[t], x1 = s.x1[t], y0 = s.y0[t], y1 = s.y1[t];
        sxx[0] += x0 * x0;
        sxx[1] += x0 * x1;
        sxx[2] += x1 * x0;
        sxx[3] += x1 * x1;
        syx[0] += y0 * x0;
        syx[1] += y0 * x1;
        syx[2] += y1 * x0;
        syx[3] += y1 * x1;
    }
    inverse2(sxx, xi);
    double a00 = syx[0] * xi[0] + syx[1] * xi[2], a01 = syx[0] * xi[1] + syx[1] * xi[3];
    double a10 = syx[2] * xi[0] + syx[3] * xi[2], a11 = syx[2] * xi[1] + syx[3] * xi[3];
    // The eigenvalues of A A^T bound the affinity's scale change.
    const double ea = a00 * a00 + a01 * a01, eb = a00 * a10 + a01 * a11;
    const double ed = a10 * a10 + a11 * a11;
    const double trh = 0.5 * (ea + ed), df = 0.5 * (ea - ed), disc = hypot(df, eb);
    const double e1 = fmax(trh + disc, 0.0), e2 = fmax(trh - disc, 0.0);
    if (e2 < 1.0 / dt2 || e1 > dt2) {
        a00 = a11 = 1;
        a01 = a10 = 0;
    }
    return {(float)a00, (float)a01, (float)a10, (float)a11};
}

// Boundaries of the duplicate test: a problem's last column equals the
// next problem's first when their half-precision residuals agree under
// every hypothesis.
void join_boundaries(const Samples &s, int iters, const std::vector<float> &first,
                     const std::vector<float> &last, std::vector<unsigned char> &eq)
{
    const int nr = (int)s.off.size();
    for (int r = 0; r < nr; r++) {
        unsigned char same = r + 1 < nr;
        for (int it = 0; it < iters && same; it++)
            same = last[(size_t)r * iters + it] == first[(size_t)(r + 1) * iters + it];
        eq[s.off[r] + s.len[r] - 1] = same;
    }
}

// The final round, shared by both paths: under the refit affinities, the
// sorted residuals of every problem (order, sq: N each) give the duplicate
// weights and one selection per problem.
void final_round(const Samples &s, const std::vector<float> &sq, double min_conf,
                 std::vector<Selection> &best)
{
    const int N = s.count(), nr = (int)s.off.size();
    constexpr int CHUNK = 1 << 16;
    std::vector<float> h(N);
    parallel_for((N + CHUNK - 1) / CHUNK, [&](int c) {
        for (int k = c * CHUNK; k < std::min(N, (c + 1) * CHUNK); k++)
            h[k] = via_half(sq[k]);
    });
    std::vector<unsigned char> eq(N);
    for (int k = 0; k + 1 < N; k++)
        eq[k] = h[k] == h[k + 1];
    eq[N - 1] = 0;
    std::vector<float> wt;
    duplicate_weights(eq, wt);
    parallel_for(nr, [&](int r) {
        best[r] = select_inliers(sq.data() + s.off[r], wt.data() + s.off[r], s.len[r], min_conf);
    });
}

// The hypotheses' affinities, problem-major: A[(r * iters + it)].
std::vector<Affine> all_hypotheses(const Samples &s, const std::vector<int> &ca,
                                   const std::vector<int> &cb)
{
    const int nr = (int)s.off.size(), iters = (int)ca.size();
    std::vector<Affine> A((size_t)nr * iters);
    for (int r = 0; r < nr; r++)
        for (int it = 0; it < iters; it++)
            A[(size_t)r * iters + it] = hypothesis(s, r, ca[it], cb[it]);
    return A;
}

// ------------------------------------------------------------ host path

// Both passes and the final round on host threads: best[r] and the
// inliers inl (problem-major, the first best[r].cnt of each problem).
void host_passes(const Samples &s, const std::vector<int> &ca, const std::vector<int> &cb,
                 const struct adalam_config *cfg, std::vector<Selection> &best,
                 std::vector<int> &inl)
{
    const int nr = (int)s.off.size(), N = s.count(), iters = (int)ca.size();
    std::vector<unsigned char> eq(N, 1);
    std::vector<float> first((size_t)nr * iters), last((size_t)nr * iters);
    for_problems(nr, [&](int r, Scratch &w) {
        const int o = s.off[r], n = s.len[r];
        for (int it = 0; it < iters; it++) {
            sorted_residuals(s, r, hypothesis(s, r, ca[it], cb[it]), w);
            float prev = via_half(w.sq[0]);
            first[(size_t)r * iters + it] = prev;
            for (int k = 0; k + 1 < n; k++) {
                const float next = via_half(w.sq[k + 1]);
                if (eq[o + k] && prev != next)
                    eq[o + k] = 0;
                prev = next;
            }
            last[(size_t)r * iters + it] = prev;
        }
    });
    join_boundaries(s, iters, first, last, eq);
    std::vector<float> wt;
    duplicate_weights(eq, wt);

    best.assign(nr, Selection());
    inl.assign(N, 0);
    for_problems(nr, [&](int r, Scratch &w) {
        const int o = s.off[r], n = s.len[r];
        for (int it = 0; it < iters; it++) {
            sorted_residuals(s, r, hypothesis(s, r, ca[it], cb[it]), w);
            const Selection sel = select_inliers(w.sq.data(), wt.data() + o, n,
                                                 cfg->min_confidence);
            if (sel.cnt > best[r].cnt) {
                best[r] = sel;
                std::copy(w.order.begin(), w.order.begin() + sel.cnt, inl.begin() + o);
            }
        }
    });

    long total = 0;
    for (int r = 0; r < nr; r++)
        total += best[r].cnt;
    if (total <= 0)
        return;
    std::vector<Affine> fit(nr);
    for (int r = 0; r < nr; r++)
        fit[r] = refit(s, inl.data() + s.off[r], best[r].cnt, cfg->det_thr);
    std::vector<float> sq(N);
    for_problems(nr, [&](int r, Scratch &w) {
        sorted_residuals(s, r, fit[r], w);
        std::copy(w.order.begin(), w.order.end(), inl.begin() + s.off[r]);
        std::copy(w.sq.begin(), w.sq.end(), sq.begin() + s.off[r]);
    });
    final_round(s, sq, cfg->min_confidence, best);
}

// ---------------------------------------------------------- device path
//
// One CTA per (hypothesis, problem): the problem's residuals under the
// hypothesis, a bitonic sort of (residual, sample) pairs in shared memory,
// then either the duplicate test of adjacent columns (pass 1) or the
// inlier selection (pass 2). The affinities come from the host (the same
// double arithmetic as the host path); on the device every float and
// double operation is written with its rounding intrinsic, so nothing is
// contracted, and the residual is the correctly rounded sqrt of the
// double sum of squares, which is what the host's hypotf returns.

constexpr int DEV_THREADS = 256;
constexpr int DEV_MAX_SAMPLES = 16384;  // Per problem: 128 KiB of sort keys.

struct DevView {
    const float *x0, *x1, *y0, *y1;
    const int *off, *len;
};

__device__ __forceinline__ float dev_hypot(float x, float y)
{
    const double xd = x, yd = y;
    return __double2float_rn(__dsqrt_rn(__dadd_rn(__dmul_rn(xd, xd), __dmul_rn(yd, yd))));
}

__device__ __forceinline__ float dev_sq(float v) { return __fmul_rn(v, v); }

__device__ __forceinline__ float dev_half(float v) { return __half2float(__float2half_rn(v)); }

// The smallest power of two >= n (n >= 1).
__device__ __forceinline__ int pow2_at_least(int n)
{
    int p = 1;
    while (p < n)
        p <<= 1;
    return p;
}

// Problem (o, n)'s residuals under A, sorted ascending by (residual,
// sample index) into key / idx; entries n..P-1 are padding (+inf).
__device__ void dev_sorted_residuals(const DevView &v, int o, int n, int P, const float *A,
                                     float *key, int *idx)
{
    for (int k = threadIdx.x; k < P; k += blockDim.x) {
        if (k < n) {
            const int t = o + k;
            const float px = __fadd_rn(__fmul_rn(A[0], v.x0[t]), __fmul_rn(A[1], v.x1[t]));
            const float py = __fadd_rn(__fmul_rn(A[2], v.x0[t]), __fmul_rn(A[3], v.x1[t]));
            key[k] = dev_hypot(__fsub_rn(px, v.y0[t]), __fsub_rn(py, v.y1[t]));
            idx[k] = t;
        }
        else {
            key[k] = __int_as_float(0x7f800000);
            idx[k] = 0x7fffffff;
        }
    }
    __syncthreads();
    for (int size = 2; size <= P; size <<= 1)
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < P; i += blockDim.x) {
                const int j = i ^ stride;
                if (j <= i)
                    continue;
                const float ki = key[i], kj = key[j];
                const int ii = idx[i], ij = idx[j];
                const bool greater = ki > kj || (ki == kj && ii > ij);
                if (greater == ((i & size) == 0)) {
                    key[i] = kj;
                    key[j] = ki;
                    idx[i] = ij;
                    idx[j] = ii;
                }
            }
            __syncthreads();
        }
}

// Pass 1: clear eq[o + k] where sorted columns k and k + 1 differ in half
// precision; record the first and last column of the problem.
__global__ void __launch_bounds__(DEV_THREADS)
    dup_k(DevView v, const float *A, int iters, unsigned char *eq, float *first, float *last)
{
    extern __shared__ float smem[];
    const int it = blockIdx.x, r = blockIdx.y;
    const int o = v.off[r], n = v.len[r], P = pow2_at_least(n);
    float *key = smem;
    int *idx = (int *)(smem + P);
    const size_t h = (size_t)r * iters + it;
    dev_sorted_residuals(v, o, n, P, A + 4 * h, key, idx);
    for (int k = threadIdx.x; k + 1 < n; k += blockDim.x)
        if (dev_half(dev_sq(key[k])) != dev_half(dev_sq(key[k + 1])))
            eq[o + k] = 0;
    if (threadIdx.x == 0) {
        first[h] = dev_half(dev_sq(key[0]));
        last[h] = dev_half(dev_sq(key[n - 1]));
    }
}

// Exclusive prefix sum over the block of one double per thread, and the
// total. Used only where every partial sum is exact, so the result is the
// sequential one.
__device__ double block_exclusive_sum(double x, double *total, double *warp_tot)
{
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    double incl = x;
    for (int d = 1; d < 32; d <<= 1) {
        const double y = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d)
            incl = __dadd_rn(incl, y);
    }
    if (lane == 31)
        warp_tot[wid] = incl;
    __syncthreads();
    if (threadIdx.x == 0) {
        double run = 0;
        for (int w = 0; w < nw; w++) {
            const double t = warp_tot[w];
            warp_tot[w] = run;
            run = __dadd_rn(run, t);
        }
        warp_tot[nw] = run;
    }
    __syncthreads();
    const double out = __dadd_rn(warp_tot[wid], __dsub_rn(incl, x));
    *total = warp_tot[nw];
    __syncthreads();
    return out;
}

// Pass 2: the confidence-based selection of each (hypothesis, problem).
// With exact = 1 (every column weight at least 2^-16 and at most 2^14
// columns, so that all partial sums of weights are exact in double) the
// sums run in parallel; otherwise one thread runs them in order.
__global__ void __launch_bounds__(DEV_THREADS)
    select_k(DevView v, const float *A, int iters, const float *wt, double min_conf, int exact,
             int *cnt, double *bal, float *hi)
{
    extern __shared__ float smem[];
    __shared__ double warp_tot[DEV_THREADS / 32 + 1];
    const int it = blockIdx.x, r = blockIdx.y;
    const int o = v.off[r], n = v.len[r], P = pow2_at_least(n);
    float *key = smem;
    int *idx = (int *)(smem + P);
    const size_t h = (size_t)r * iters + it;
    dev_sorted_residuals(v, o, n, P, A + 4 * h, key, idx);
    double b = 0, c = 0;
    if (exact) {
        const int per = (n + blockDim.x - 1) / blockDim.x;
        const int k0 = threadIdx.x * per, k1 = min(n, k0 + per);
        double part = 0;
        for (int k = k0; k < k1; k++)
            if (!(dev_sq(key[k]) <= 1e-8f))
                part = __dadd_rn(part, (double)wt[o + k]);
        double cum = block_exclusive_sum(part, &b, warp_tot);
        double mine = 0;
        for (int k = k0; k < k1; k++) {
            const float q = dev_sq(key[k]);
            const bool perfect = q <= 1e-8f;
            const double w = perfect ? 0.0 : (double)wt[o + k];
            cum = __dadd_rn(cum, w);
            if (perfect || __dmul_rn((double)q, min_conf) <= __ddiv_rn(cum, b))
                mine = __dadd_rn(mine, w);
        }
        block_exclusive_sum(mine, &c, warp_tot);
    }
    else if (threadIdx.x == 0) {
        for (int k = 0; k < n; k++)
            if (!(dev_sq(key[k]) <= 1e-8f))
                b = __dadd_rn(b, (double)wt[o + k]);
        double cum = 0;
        for (int k = 0; k < n; k++) {
            const float q = dev_sq(key[k]);
            const bool perfect = q <= 1e-8f;
            const double w = perfect ? 0.0 : (double)wt[o + k];
            cum = __dadd_rn(cum, w);
            if (perfect || __dmul_rn((double)q, min_conf) <= __ddiv_rn(cum, b))
                c = __dadd_rn(c, w);
        }
    }
    if (threadIdx.x == 0) {
        const long ct = (long)c;
        cnt[h] = (int)ct;
        bal[h] = b;
        hi[h] = ct > 0 ? dev_sq(key[ct - 1]) : 0.0f;
    }
}

// The sorted residuals of problem r under A[r]: sample order and squared
// residuals, problem-major.
__global__ void __launch_bounds__(DEV_THREADS)
    order_k(DevView v, const float *A, int *order, float *sq)
{
    extern __shared__ float smem[];
    const int r = blockIdx.x;
    const int o = v.off[r], n = v.len[r], P = pow2_at_least(n);
    float *key = smem;
    int *idx = (int *)(smem + P);
    dev_sorted_residuals(v, o, n, P, A + 4 * r, key, idx);
    for (int k = threadIdx.x; k < n; k += blockDim.x) {
        order[o + k] = idx[k];
        sq[o + k] = dev_sq(key[k]);
    }
}

// Byte offsets of the arrays in one device allocation.
struct DevLayout {
    size_t x0, x1, y0, y1, off, len, A, eq, first, last, wt, cnt, bal, hi, fit, order, sq, bytes;
    DevLayout(int N, int nr, int iters)
    {
        size_t at = 0;
        auto take = [&at](size_t n) {
            const size_t p = at;
            at += (n + 255) / 256 * 256;
            return p;
        };
        const size_t H = (size_t)nr * iters;
        x0 = take(4 * (size_t)N);
        x1 = take(4 * (size_t)N);
        y0 = take(4 * (size_t)N);
        y1 = take(4 * (size_t)N);
        off = take(4 * (size_t)nr);
        len = take(4 * (size_t)nr);
        A = take(16 * (H > 0 ? H : 1));
        eq = take((size_t)N);
        first = take(4 * H + 4);
        last = take(4 * H + 4);
        wt = take(4 * (size_t)N);
        cnt = take(4 * H + 4);
        bal = take(8 * H + 8);
        hi = take(4 * H + 4);
        fit = take(16 * (size_t)nr);
        order = take(4 * (size_t)N);
        sq = take(4 * (size_t)N);
        bytes = at;
    }
};

// Both passes on the device of o, the refit and final round on the host
// (as in host_passes); false with a recorded error on failure.
bool device_passes(struct ops *o, const Samples &s, const std::vector<int> &ca,
                   const std::vector<int> &cb, const struct adalam_config *cfg,
                   std::vector<Selection> &best, std::vector<int> &inl)
{
    using coreg::cuda_ok;
    using coreg::launch_ok;
    const int nr = (int)s.off.size(), N = s.count(), iters = (int)ca.size();
    int maxlen = 0;
    for (int r = 0; r < nr; r++)
        maxlen = std::max(maxlen, s.len[r]);
    if (nr > 65535) {
        fail("adalam: %d neighbourhoods exceed the device grid", nr);
        return false;
    }
    if (maxlen > DEV_MAX_SAMPLES) {
        fail("adalam: a neighbourhood of %d matches exceeds the device limit of %d", maxlen,
             DEV_MAX_SAMPLES);
        return false;
    }
    int P = 1;
    while (P < maxlen)
        P <<= 1;
    const size_t smem = (size_t)P * 8;
    struct ocl_backend *ocl = o->ocl;
    cudaSetDevice(ocl->device);
    cudaStream_t st = coreg::stream_of(ocl);
    if (!cuda_ok(cudaFuncSetAttribute(dup_k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem),
                 "adalam dup_k smem") ||
        !cuda_ok(cudaFuncSetAttribute(select_k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem),
                 "adalam select_k smem") ||
        !cuda_ok(cudaFuncSetAttribute(order_k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem),
                 "adalam order_k smem"))
        return false;

    const DevLayout L(N, nr, iters);
    cl_mem buf = ocl_alloc(ocl, L.bytes, "adalam");
    if (pending())
        return false;
    char *base = (char *)buf->ptr;
    DevView v = {(const float *)(base + L.x0), (const float *)(base + L.x1),
                 (const float *)(base + L.y0), (const float *)(base + L.y1),
                 (const int *)(base + L.off), (const int *)(base + L.len)};
    const std::vector<Affine> hyp = iters ? all_hypotheses(s, ca, cb) : std::vector<Affine>();
    ocl_write(ocl, buf, L.x0, s.x0.data(), 4 * (size_t)N);
    ocl_write(ocl, buf, L.x1, s.x1.data(), 4 * (size_t)N);
    ocl_write(ocl, buf, L.y0, s.y0.data(), 4 * (size_t)N);
    ocl_write(ocl, buf, L.y1, s.y1.data(), 4 * (size_t)N);
    ocl_write(ocl, buf, L.off, s.off.data(), 4 * (size_t)nr);
    ocl_write(ocl, buf, L.len, s.len.data(), 4 * (size_t)nr);
    if (iters)
        ocl_write(ocl, buf, L.A, hyp.data(), hyp.size() * sizeof(Affine));
    cuda_ok(cudaMemsetAsync(base + L.eq, 1, (size_t)N, st), "adalam eq");

    best.assign(nr, Selection());
    inl.assign(N, 0);
    std::vector<unsigned char> eq(N, 1);
    std::vector<float> first((size_t)nr * iters), last((size_t)nr * iters), wt;
    if (iters && !pending()) {
        const dim3 grid(iters, nr);
        dup_k<<<grid, DEV_THREADS, smem, st>>>(v, (const float *)(base + L.A), iters,
                                               (unsigned char *)(base + L.eq),
                                               (float *)(base + L.first),
                                               (float *)(base + L.last));
        if (launch_ok("adalam dup_k")) {
            ocl_read(ocl, buf, L.eq, eq.data(), (size_t)N);
            ocl_read(ocl, buf, L.first, first.data(), 4 * first.size());
            ocl_read(ocl, buf, L.last, last.data(), 4 * last.size());
        }
    }
    join_boundaries(s, iters, first, last, eq);
    duplicate_weights(eq, wt);

    if (iters && !pending()) {
        // Exact parallel sums need every weight >= 2^-16 and <= 2^14 columns.
        const float wmin = *std::min_element(wt.begin(), wt.end());
        const int exact = wmin >= 1.0f / 65536.0f && maxlen <= 16384;
        ocl_write(ocl, buf, L.wt, wt.data(), 4 * (size_t)N);
        const dim3 grid(iters, nr);
        select_k<<<grid, DEV_THREADS, smem, st>>>(
            v, (const float *)(base + L.A), iters, (const float *)(base + L.wt),
            cfg->min_confidence, exact, (int *)(base + L.cnt), (double *)(base + L.bal),
            (float *)(base + L.hi));
        std::vector<int> cnt((size_t)nr * iters);
        std::vector<double> bal((size_t)nr * iters);
        std::vector<float> hi((size_t)nr * iters);
        if (launch_ok("adalam select_k")) {
            ocl_read(ocl, buf, L.cnt, cnt.data(), 4 * cnt.size());
            ocl_read(ocl, buf, L.bal, bal.data(), 8 * bal.size());
            ocl_read(ocl, buf, L.hi, hi.data(), 4 * hi.size());
        }
        // Each problem's best hypothesis: the first with the highest count.
        std::vector<int> best_it(nr, -1);
        for (int r = 0; r < nr; r++)
            for (int it = 0; it < iters; it++) {
                const size_t h = (size_t)r * iters + it;
                if (cnt[h] > best[r].cnt) {
                    best[r].cnt = cnt[h];
                    best[r].bal = bal[h];
                    best[r].hi = hi[h];
                    best_it[r] = it;
                }
            }
        long total = 0;
        for (int r = 0; r < nr; r++)
            total += best[r].cnt;
        if (total > 0 && !pending()) {
            // The inliers of each best hypothesis, for the host's refit.
            std::vector<Affine> A(nr);
            for (int r = 0; r < nr; r++)
                A[r] = hyp[(size_t)r * iters + best_it[r]];
            ocl_write(ocl, buf, L.fit, A.data(), A.size() * sizeof(Affine));
            order_k<<<nr, DEV_THREADS, smem, st>>>(v, (const float *)(base + L.fit),
                                                   (int *)(base + L.order),
                                                   (float *)(base + L.sq));
            if (launch_ok("adalam order_k"))
                ocl_read(ocl, buf, L.order, inl.data(), 4 * (size_t)N);
            for (int r = 0; r < nr; r++)
                A[r] = refit(s, inl.data() + s.off[r], best[r].cnt, cfg->det_thr);
            ocl_write(ocl, buf, L.fit, A.data(), A.size() * sizeof(Affine));
            order_k<<<nr, DEV_THREADS, smem, st>>>(v, (const float *)(base + L.fit),
                                                   (int *)(base + L.order),
                                                   (float *)(base + L.sq));
            std::vector<float> sq(N);
            if (launch_ok("adalam order_k")) {
                ocl_read(ocl, buf, L.order, inl.data(), 4 * (size_t)N);
                ocl_read(ocl, buf, L.sq, sq.data(), 4 * (size_t)N);
            }
            if (!pending())
                final_round(s, sq, cfg->min_confidence, best);
        }
    }
    ocl_release(&buf);
    return !pending();
}

}  // namespace

extern "C" void adalam_defaults(struct adalam_config *c)
{
    c->area_ratio = 100;
    c->search_expansion = 16;
    c->ransac_iters = 256;
    c->min_inliers = 6;
    c->min_confidence = 200;
    c->det_thr = 5;
    c->force_seed_mnn = 0;
}

extern "C" int adalam_filter(struct ops *o, const float *k1, int n1, const float *k2, int n2,
                             const int *nn12, const float *score, const int *nn21,
                             const struct adalam_config *cfg, int **pairs, float **dist)
{
    *pairs = nullptr;
    *dist = nullptr;
    if (pending() || n1 <= 1 || n2 <= 1)
        return 0;
    for (int i = 0; i < n1; i++)
        if (nn12[i] < 0 || nn12[i] >= n2) {
            fail("adalam_filter: nearest neighbour %d of keypoint %d outside 0..%d", nn12[i], i,
                 n2 - 1);
            return 0;
        }
    std::vector<unsigned char> mnn;
    if (cfg->force_seed_mnn) {
        if (!nn21) {
            fail("adalam_filter: force_seed_mnn needs nn21");
            return 0;
        }
        mnn.resize(n1);
        for (int i = 0; i < n1; i++)
            mnn[i] = nn21[nn12[i]] == i;
    }
    const auto mutual = [&](int i) { return mnn.empty() || mnn[i]; };

    const double R1 = seed_radius(k1, n1, cfg->area_ratio);
    const double R2 = seed_radius(k2, n2, cfg->area_ratio);
    const double rr1 = R1 * R1;
    const double se1 = cfg->search_expansion * R1, se2 = cfg->search_expansion * R2;
    const double se1sq = se1 * se1, se2sq = se2 * se2;

    // Seeds: a ratio below 0.8^2 and the best (lowest) within R1.
    std::vector<int> seeds;
    for (int i = 0; i < n1; i++) {
        bool seed = score[i] < 0.64f && mutual(i);
        for (int j = 0; j < n1 && seed; j++)
            if (sqdist(k1 + 2 * i, k1 + 2 * j) < rr1 && score[i] > score[j] && mutual(j))
                seed = false;
        if (seed)
            seeds.push_back(i);
    }

    // Neighbourhoods: the matches within the expanded radius of the seed
    // in both images, in ascending order of score (ties by index); seeds
    // with fewer than min_inliers of them are dropped. Walking the matches
    // in that order once sorted, each neighbourhood comes out sorted; the
    // seeds are counted, then filled, on host threads.
    std::vector<std::pair<float, int>> by_score(n1);
    for (int j = 0; j < n1; j++)
        by_score[j] = {score[j], j};
    std::sort(by_score.begin(), by_score.end());
    const int ns = (int)seeds.size();
    const auto member = [&](int si, int j) {
        return sqdist(k1 + 2 * si, k1 + 2 * j) < se1sq &&
               sqdist(k2 + 2 * nn12[si], k2 + 2 * nn12[j]) < se2sq;
    };
    std::vector<int> count(ns);
    parallel_for(ns, [&](int q) {
        int c = 0;
        for (int j = 0; j < n1; j++)
            c += member(seeds[q], j);
        count[q] = c;
    });
    Samples s;
    std::vector<int> kept, at;
    int N = 0;
    for (int q = 0; q < ns; q++)
        if (count[q] >= cfg->min_inliers && count[q] > 0) {
            kept.push_back(seeds[q]);
            s.off.push_back(N);
            s.len.push_back(count[q]);
            N += count[q];
        }
    const int nr = (int)kept.size();
    for (auto *v : {&s.x0, &s.x1, &s.y0, &s.y1})
        v->resize(N);
    s.kp1.resize(N);
    s.kp2.resize(N);
    parallel_for(nr, [&](int r) {
        const int si = kept[r];
        const float *t1 = k1 + 2 * si, *t2 = k2 + 2 * nn12[si];
        int t = s.off[r];
        for (const auto &e : by_score) {
            const int j = e.second;
            if (!member(si, j))
                continue;
            const int q = nn12[j];
            s.x0[t] = (float)((k1[2 * j] - t1[0]) / se1);
            s.x1[t] = (float)((k1[2 * j + 1] - t1[1]) / se1);
            s.y0[t] = (float)((k2[2 * q] - t2[0]) / se2);
            s.y1[t] = (float)((k2[2 * q + 1] - t2[1]) / se2);
            s.kp1[t] = j;
            s.kp2[t] = q;
            t++;
        }
    });

    std::vector<Match> out;
    if (nr == 0) {
        // No neighbourhood: every match with a ratio up to 0.95.
        for (int i = 0; i < n1; i++)
            if (score[i] <= 0.95f)
                out.push_back({i, nn12[i], score[i]});
        return emit(out, pairs, dist);
    }

    std::vector<int> ca, cb;
    first_couples(std::max(0, cfg->ransac_iters), ca, cb);
    std::vector<Selection> best;
    std::vector<int> inl;
    if (o) {
        if (!device_passes(o, s, ca, cb, cfg, best, inl))
            return 0;
    }
    else
        host_passes(s, ca, cb, cfg, best, inl);

    // Accept the inliers of the confident problems that keep enough.
    for (int r = 0; r < nr; r++) {
        const Selection &b = best[r];
        const float conf = b.cnt > 0 ? (float)(b.cnt / (b.bal * b.hi)) : 0.0f;
        const float ratio = 1.0f / conf;
        if (!(conf >= cfg->min_confidence && (float)b.cnt * (1.0f - ratio) >= cfg->min_inliers))
            continue;
        for (long k = 0; k < b.cnt; k++) {
            const int t = inl[s.off[r] + k];
            out.push_back({s.kp1[t], s.kp2[t], ratio});
        }
    }
    return emit(out, pairs, dist);
}

extern "C" int adalam_match(struct ops *o, const float *k1, const float *d1, int n1,
                            const float *k2, const float *d2, int n2, int dim,
                            const struct adalam_config *cfg, int **pairs, float **dist)
{
    *pairs = nullptr;
    *dist = nullptr;
    if (pending() || n1 <= 1 || n2 <= 1)
        return 0;
    if (!o) {
        fail("adalam_match: no device (ops) given");
        return 0;
    }
    std::vector<int> nn12(n1), nn21(cfg->force_seed_mnn ? n2 : 0);
    std::vector<float> score(n1);
    desc_nearest(o, d1, n1, d2, n2, dim, nn12.data(), score.data(),
                 cfg->force_seed_mnn ? nn21.data() : nullptr);
    if (pending())
        return 0;
    return adalam_filter(o, k1, n1, k2, n2, nn12.data(), score.data(),
                         cfg->force_seed_mnn ? nn21.data() : nullptr, cfg, pairs, dist);
}
