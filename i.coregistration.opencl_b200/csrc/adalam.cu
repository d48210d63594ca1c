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
// The nearest neighbours come from the device (desc_nearest). The
// filtering runs on the host, problem by problem: a neighbourhood's
// hypotheses need only its own samples, so the problems are spread over
// host threads, and the one coupling between problems (the duplicate test
// compares the last sorted residual of a problem with the first of the
// next, as kornia's unique_consecutive over the concatenated columns does)
// is carried as each problem's first and last residual per hypothesis.
// Every floating-point expression keeps the reference's types and order,
// so that the matches and confidences agree bit for bit.

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

// A value rounded to IEEE binary16 and back (kornia compares the sorted
// residuals of the hypotheses in half precision).
inline float via_half(float v) { return __half2float(__float2half_rn(v)); }

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

extern "C" int adalam_filter(const float *k1, int n1, const float *k2, int n2, const int *nn12,
                             const float *score, const int *nn21,
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
    // with fewer than min_inliers of them are dropped.
    Samples s;
    std::vector<int> kept;
    std::vector<std::pair<float, int>> nb;
    for (int si : seeds) {
        const float *t1 = k1 + 2 * si, *t2 = k2 + 2 * nn12[si];
        nb.clear();
        for (int j = 0; j < n1; j++)
            if (sqdist(t1, k1 + 2 * j) < se1sq && sqdist(t2, k2 + 2 * nn12[j]) < se2sq)
                nb.push_back({score[j], j});
        if ((int)nb.size() < cfg->min_inliers || nb.empty())
            continue;
        std::sort(nb.begin(), nb.end());
        kept.push_back(si);
        s.off.push_back(s.count());
        s.len.push_back((int)nb.size());
        for (const auto &e : nb) {
            const int j = e.second, q = nn12[j];
            s.x0.push_back((float)((k1[2 * j] - t1[0]) / se1));
            s.x1.push_back((float)((k1[2 * j + 1] - t1[1]) / se1));
            s.y0.push_back((float)((k2[2 * q] - t2[0]) / se2));
            s.y1.push_back((float)((k2[2 * q + 1] - t2[1]) / se2));
            s.kp1.push_back(j);
            s.kp2.push_back(q);
        }
    }
    const int nr = (int)kept.size(), N = s.count();

    std::vector<Match> out;
    if (nr == 0) {
        // No neighbourhood: every match with a ratio up to 0.95.
        for (int i = 0; i < n1; i++)
            if (score[i] <= 0.95f)
                out.push_back({i, nn12[i], score[i]});
        return emit(out, pairs, dist);
    }

    std::vector<int> ca, cb;
    first_couples(cfg->ransac_iters, ca, cb);
    const int iters = (int)ca.size();

    // Pass 1, the duplicate columns: a column equals the next when their
    // sorted squared residuals agree in half precision under every
    // hypothesis. Inside a problem that is tracked per column; across a
    // problem boundary through the first and last residual of each.
    std::vector<unsigned char> eq(N, 1);
    std::vector<float> first((size_t)nr * iters), last((size_t)nr * iters);
    for_problems(nr, [&](int r, Scratch &w) {
        const int o = s.off[r], n = s.len[r];
        for (int it = 0; it < iters; it++) {
            sorted_residuals(s, r, hypothesis(s, r, ca[it], cb[it]), w);
            for (int k = 0; k + 1 < n; k++)
                if (eq[o + k] && via_half(w.sq[k]) != via_half(w.sq[k + 1]))
                    eq[o + k] = 0;
            first[(size_t)r * iters + it] = via_half(w.sq[0]);
            last[(size_t)r * iters + it] = via_half(w.sq[n - 1]);
        }
    });
    for (int r = 0; r < nr; r++) {
        unsigned char same = r + 1 < nr;
        for (int it = 0; it < iters && same; it++)
            same = last[(size_t)r * iters + it] == first[(size_t)(r + 1) * iters + it];
        eq[s.off[r] + s.len[r] - 1] = same;
    }
    std::vector<float> wt;
    duplicate_weights(eq, wt);

    // Pass 2: each problem's best hypothesis (the first with the highest
    // inlier count) and its inliers.
    std::vector<Selection> best(nr);
    std::vector<int> inl(N);
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
    if (total > 0) {
        // Refit: the least-squares affinity of each problem's inliers, the
        // identity where its scale change exceeds det_thr; then one
        // selection round under it.
        const double dt2 = cfg->det_thr * cfg->det_thr;
        std::vector<Affine> fit(nr);
        for (int r = 0; r < nr; r++) {
            double sxx[4] = {0, 0, 0, 0}, syx[4] = {0, 0, 0, 0}, xi[4];
            for (long k = 0; k < best[r].cnt; k++) {
                const int t = inl[s.off[r] + k];
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
            fit[r] = {(float)a00, (float)a01, (float)a10, (float)a11};
        }
        std::vector<float> sq(N);
        for_problems(nr, [&](int r, Scratch &w) {
            sorted_residuals(s, r, fit[r], w);
            std::copy(w.order.begin(), w.order.end(), inl.begin() + s.off[r]);
            std::copy(w.sq.begin(), w.sq.end(), sq.begin() + s.off[r]);
        });
        for (int k = 0; k + 1 < N; k++)
            eq[k] = via_half(sq[k]) == via_half(sq[k + 1]);
        eq[N - 1] = 0;
        duplicate_weights(eq, wt);
        for (int r = 0; r < nr; r++)
            best[r] = select_inliers(sq.data() + s.off[r], wt.data() + s.off[r], s.len[r],
                                     cfg->min_confidence);
    }

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
    std::vector<int> nn12(n1), nn21(cfg->force_seed_mnn ? n2 : 0);
    std::vector<float> score(n1);
    desc_nearest(o, d1, n1, d2, n2, dim, nn12.data(), score.data(),
                 cfg->force_seed_mnn ? nn21.data() : nullptr);
    if (pending())
        return 0;
    return adalam_filter(k1, n1, k2, n2, nn12.data(), score.data(),
                         cfg->force_seed_mnn ? nn21.data() : nullptr, cfg, pairs, dist);
}
