// SPDX-License-Identifier: Unlicense
//
// The matcher interface (matcher.h) and the RoMa matcher
// (matcher_roma.h): the device stage through roma_match, the host stage
// (roma_sample_matches, roma_dense_field) with the reference's sampling
// rules (matcher_roma.c:41-232).

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <vector>

#include "common.cuh"
#include "matcher_roma.h"
#include "roma.h"

using coreg::cuda_ok;
using coreg::fail;
using coreg::pending;

extern "C" void match_add(struct match_list *l, const struct match *m)
{
    if (l->n == l->cap) {
        l->cap = l->cap ? 2 * l->cap : 1024;
        l->v = (struct match *)realloc(l->v, l->cap * sizeof(*l->v));
    }
    l->v[l->n++] = *m;
}

extern "C" void matcher_dump_file(const char *dir, int tile, const char *what,
                                  const void *data, size_t bytes)
{
    char path[4096];
    snprintf(path, sizeof(path), "%s/tile%03d_%s", dir, tile, what);
    FILE *fp = fopen(path, "wb");
    if (!fp || fwrite(data, 1, bytes, fp) != bytes)
        fail("Unable to write debug dump <%s>", path);
    if (fp)
        fclose(fp);
}

// ---------------------------------------------- RoMa's host stage
//
// The warp (2, H, W) is normalized to [-1, 1] over the padded tile with
// align_corners false, so a warp value f lands at ((f + 1) n - 1) / 2
// cells along an axis of n cells.

namespace {

inline double landing(float f, int n) { return (f + 1.0) * 0.5 * n - 0.5; }

// Whether (x, y), rounded half away from zero, is a cell of the h x w tile
// that valid (NULL: all) marks.
bool lands_valid(const unsigned char *valid, int h, int w, double x, double y)
{
    const long ix = lround(x), iy = lround(y);
    if (ix < 0 || iy < 0 || ix >= w || iy >= h)
        return false;
    return !valid || valid[(size_t)iy * w + ix];
}

// Distance in cells from (x, y) to where the reverse warp bflow sends
// (xr, yr): (xr, yr) clamped into the h x w tile, the reverse landing
// interpolated bilinearly over the 2 x 2 cells at or left / above it (the
// last pair when it lies on the last row or column) (matcher_roma.c:61-90).
float cycle_distance(const float *bflow, int H, int W, int h, int w, int x, int y,
                     double xr, double yr)
{
    if (w == 1 || h == 1)
        return NAN;
    xr = xr < 0 ? 0 : xr > w - 1 ? w - 1 : xr;
    yr = yr < 0 ? 0 : yr > h - 1 ? h - 1 : yr;
    const int cx = (int)xr < w - 2 ? (int)xr : w - 2;
    const int cy = (int)yr < h - 2 ? (int)yr : h - 2;
    const double fx = xr - cx, fy = yr - cy;
    const size_t plane = (size_t)H * W;
    double sx = 0, sy = 0;
    for (int j = 0; j < 2; j++)
        for (int i = 0; i < 2; i++) {
            const size_t k = (size_t)(cy + j) * W + cx + i;
            const double wgt = (i ? fx : 1 - fx) * (j ? fy : 1 - fy);
            sx += wgt * landing(bflow[k], W);
            sy += wgt * landing(bflow[plane + k], H);
        }
    return (float)hypot(sx - x, sy - y);
}

}  // namespace

extern "C" int roma_sample_matches(const float *flow, const float *cert, const float *sd,
                                   const float *bflow, int H, int W, int h, int w,
                                   int spacing, float min_cert,
                                   const unsigned char *valid1,
                                   const unsigned char *valid2, struct match_list *out)
{
    if (pending())
        return 0;
    if (spacing < 1 || h > H || w > W) {
        fail("roma_sample_matches: spacing %d, tile %d x %d of %d x %d", spacing, h, w, H, W);
        return 0;
    }
    const size_t plane = (size_t)H * W;
    int n = 0;
    for (int by = 0; by < h; by += spacing)
        for (int bx = 0; bx < w; bx += spacing) {
            // The block's first valid cell of highest certainty.
            const int ye = by + spacing < h ? by + spacing : h;
            const int xe = bx + spacing < w ? bx + spacing : w;
            long best = -1;
            for (int y = by; y < ye; y++)
                for (int x = bx; x < xe; x++)
                    if (!valid1 || valid1[(size_t)y * w + x]) {
                        const long i = (long)y * W + x;
                        if (best < 0 || cert[i] > cert[best])
                            best = i;
                    }
            if (best < 0 || !(cert[best] >= min_cert))
                continue;
            const int x = (int)(best % W), y = (int)(best / W);
            struct match mt;
            mt.x1 = x;
            mt.y1 = y;
            mt.x2 = landing(flow[best], W);
            mt.y2 = landing(flow[plane + best], H);
            if (!lands_valid(valid2, h, w, mt.x2, mt.y2))
                continue;
            mt.cost = 1.0f - cert[best];
            mt.sd = sd ? sd[best] : NAN;
            mt.cycle = bflow ? cycle_distance(bflow, H, W, h, w, x, y, mt.x2, mt.y2) : NAN;
            match_add(out, &mt);
            n++;
        }
    return n;
}

extern "C" void roma_dense_field(const float *flow, const float *cert, const float *sd,
                                 int H, int W, int h, int w, const unsigned char *valid1,
                                 const unsigned char *valid2, float *dx, float *dy,
                                 float *certo, float *sdo)
{
    if (pending())
        return;
    if (h > H || w > W) {
        fail("roma_dense_field: tile %d x %d of %d x %d", h, w, H, W);
        return;
    }
    const size_t plane = (size_t)H * W;
    for (int y = 0; y < h; y++)
        for (int x = 0; x < w; x++) {
            const size_t i = (size_t)y * W + x, o = (size_t)y * w + x;
            const double xr = landing(flow[i], W), yr = landing(flow[plane + i], H);
            if ((valid1 && !valid1[o]) || !lands_valid(valid2, h, w, xr, yr)) {
                dx[o] = dy[o] = NAN;
                certo[o] = 0.0f;
                if (sdo)
                    sdo[o] = NAN;
                continue;
            }
            dx[o] = (float)(xr - x);
            dy[o] = (float)(yr - y);
            certo[o] = cert[i];
            if (sdo)
                sdo[o] = sd ? sd[i] : NAN;
        }
}

// ----------------------------------------- RoMa's host stage on the device
//
// The same two stages as kernels over the device-resident results: one
// thread per spacing x spacing block scans its cells in the host stage's
// order (so ties and NaN certainties resolve as there), one thread per
// cell for the dense field. Every double operation is written with its
// rounding intrinsic, so nothing is contracted into an FMA and the landing
// positions, shifts and cycle distances are those of the host stage.

namespace {

// One block's sample, copied back and appended on the host in block order.
struct BlockMatch {
    double x2, y2;
    float cost, sd, cycle;
    int x1, y1, keep;
};

__device__ __forceinline__ double landing_d(float f, int n)
{
    return __dadd_rn(__dmul_rn(__dmul_rn(__dadd_rn((double)f, 1.0), 0.5), (double)n), -0.5);
}

__device__ __forceinline__ bool lands_valid_d(const unsigned char *valid, int h, int w, double x,
                                              double y)
{
    const long long ix = llround(x), iy = llround(y);
    if (ix < 0 || iy < 0 || ix >= w || iy >= h)
        return false;
    return !valid || valid[iy * w + ix];
}

__device__ float cycle_distance_d(const float *bflow, int H, int W, int h, int w, int x, int y,
                                  double xr, double yr)
{
    if (w == 1 || h == 1)
        return __int_as_float(0x7fc00000);
    xr = xr < 0 ? 0 : xr > w - 1 ? w - 1 : xr;
    yr = yr < 0 ? 0 : yr > h - 1 ? h - 1 : yr;
    const int cx = (int)xr < w - 2 ? (int)xr : w - 2;
    const int cy = (int)yr < h - 2 ? (int)yr : h - 2;
    const double fx = __dsub_rn(xr, (double)cx), fy = __dsub_rn(yr, (double)cy);
    const size_t plane = (size_t)H * W;
    double sx = 0, sy = 0;
    for (int j = 0; j < 2; j++)
        for (int i = 0; i < 2; i++) {
            const size_t k = (size_t)(cy + j) * W + cx + i;
            const double wgt = __dmul_rn(i ? fx : __dsub_rn(1.0, fx), j ? fy : __dsub_rn(1.0, fy));
            sx = __dadd_rn(sx, __dmul_rn(wgt, landing_d(bflow[k], W)));
            sy = __dadd_rn(sy, __dmul_rn(wgt, landing_d(bflow[plane + k], H)));
        }
    const double dx = __dsub_rn(sx, (double)x), dy = __dsub_rn(sy, (double)y);
    return (float)__dsqrt_rn(__dadd_rn(__dmul_rn(dx, dx), __dmul_rn(dy, dy)));
}

__global__ void sample_blocks_k(const float *flow, const float *cert, const float *sd,
                                const float *bflow, int H, int W, int h, int w, int spacing,
                                float min_cert, const unsigned char *valid1,
                                const unsigned char *valid2, int bw, int nblk, BlockMatch *out)
{
    const int b = blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblk)
        return;
    const int by = (b / bw) * spacing, bx = (b % bw) * spacing;
    const int ye = by + spacing < h ? by + spacing : h;
    const int xe = bx + spacing < w ? bx + spacing : w;
    long best = -1;
    for (int y = by; y < ye; y++)
        for (int x = bx; x < xe; x++)
            if (!valid1 || valid1[(size_t)y * w + x]) {
                const long i = (long)y * W + x;
                if (best < 0 || cert[i] > cert[best])
                    best = i;
            }
    BlockMatch r;
    r.keep = 0;
    if (best >= 0 && cert[best] >= min_cert) {
        const size_t plane = (size_t)H * W;
        r.x1 = (int)(best % W);
        r.y1 = (int)(best / W);
        r.x2 = landing_d(flow[best], W);
        r.y2 = landing_d(flow[plane + best], H);
        if (lands_valid_d(valid2, h, w, r.x2, r.y2)) {
            r.keep = 1;
            r.cost = __fsub_rn(1.0f, cert[best]);
            r.sd = sd ? sd[best] : __int_as_float(0x7fc00000);
            r.cycle = bflow ? cycle_distance_d(bflow, H, W, h, w, r.x1, r.y1, r.x2, r.y2)
                            : __int_as_float(0x7fc00000);
        }
    }
    out[b] = r;
}

__global__ void dense_field_k(const float *flow, const float *cert, const float *sd, int H,
                              int W, int h, int w, const unsigned char *valid1,
                              const unsigned char *valid2, float *dx, float *dy, float *certo,
                              float *sdo)
{
    const long o = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (o >= (long)h * w)
        return;
    const int y = (int)(o / w), x = (int)(o % w);
    const size_t i = (size_t)y * W + x, plane = (size_t)H * W;
    const double xr = landing_d(flow[i], W), yr = landing_d(flow[plane + i], H);
    const float nan = __int_as_float(0x7fc00000);
    if ((valid1 && !valid1[o]) || !lands_valid_d(valid2, h, w, xr, yr)) {
        dx[o] = dy[o] = nan;
        certo[o] = 0.0f;
        if (sdo)
            sdo[o] = nan;
        return;
    }
    dx[o] = (float)__dsub_rn(xr, (double)x);
    dy[o] = (float)__dsub_rn(yr, (double)y);
    certo[o] = cert[i];
    if (sdo)
        sdo[o] = sd ? sd[i] : nan;
}

// o->scratch grown to at least bytes (stream-ordered reuse: the entry
// points below finish with a blocking read).
char *scratch_bytes(struct ops *o, size_t bytes)
{
    if (bytes > o->scratch_bytes) {
        ocl_release(&o->scratch);
        o->scratch = ocl_alloc(o->ocl, bytes, "matcher stage");
        o->scratch_bytes = bytes;
    }
    return pending() ? nullptr : (char *)o->scratch->ptr;
}

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

}  // namespace

extern "C" int roma_sample_matches_dev(struct ops *o, const float *flow, const float *cert,
                                       const float *sd, const float *bflow, int H, int W,
                                       int h, int w, int spacing, float min_cert,
                                       const unsigned char *valid1,
                                       const unsigned char *valid2, struct match_list *out)
{
    if (pending())
        return 0;
    if (!o || !flow || !cert || spacing < 1 || h > H || w > W || h < 1 || w < 1) {
        fail("roma_sample_matches_dev: spacing %d, tile %d x %d of %d x %d", spacing, h, w, H,
             W);
        return 0;
    }
    const int bw = (w + spacing - 1) / spacing, bh = (h + spacing - 1) / spacing;
    const int nblk = bw * bh;
    const size_t cells = (size_t)h * w;
    const size_t rb = align256((size_t)nblk * sizeof(BlockMatch));
    char *base = scratch_bytes(o, rb + 2 * align256(cells));
    if (!base)
        return 0;
    BlockMatch *rec = (BlockMatch *)base;
    unsigned char *v1 = nullptr, *v2 = nullptr;
    cudaStream_t st = coreg::stream_of(o->ocl);
    cudaSetDevice(o->ocl->device);
    if (valid1) {
        v1 = (unsigned char *)base + rb;
        cudaMemcpyAsync(v1, valid1, cells, cudaMemcpyHostToDevice, st);
    }
    if (valid2) {
        v2 = (unsigned char *)base + rb + align256(cells);
        cudaMemcpyAsync(v2, valid2, cells, cudaMemcpyHostToDevice, st);
    }
    sample_blocks_k<<<coreg::cdiv(nblk, 128), 128, 0, st>>>(flow, cert, sd, bflow, H, W, h, w,
                                                           spacing, min_cert, v1, v2, bw, nblk,
                                                           rec);
    if (!coreg::launch_ok("roma_sample_matches_dev"))
        return 0;
    std::vector<BlockMatch> host(nblk);
    if (!cuda_ok(cudaMemcpyAsync(host.data(), rec, (size_t)nblk * sizeof(BlockMatch),
                                 cudaMemcpyDeviceToHost, st),
                 "roma_sample_matches_dev") ||
        !cuda_ok(cudaStreamSynchronize(st), "roma_sample_matches_dev"))
        return 0;
    int n = 0;
    for (const BlockMatch &r : host)
        if (r.keep) {
            struct match mt;
            mt.x1 = r.x1;
            mt.y1 = r.y1;
            mt.x2 = r.x2;
            mt.y2 = r.y2;
            mt.cost = r.cost;
            mt.sd = r.sd;
            mt.cycle = r.cycle;
            match_add(out, &mt);
            n++;
        }
    return n;
}

extern "C" void roma_dense_field_dev(struct ops *o, const float *flow, const float *cert,
                                     const float *sd, int H, int W, int h, int w,
                                     const unsigned char *valid1,
                                     const unsigned char *valid2, float *dx, float *dy,
                                     float *certo, float *sdo)
{
    if (pending())
        return;
    if (!o || !flow || !cert || h > H || w > W || h < 1 || w < 1) {
        fail("roma_dense_field_dev: tile %d x %d of %d x %d", h, w, H, W);
        return;
    }
    const size_t cells = (size_t)h * w, cb = align256(cells), fb = align256(cells * 4);
    char *base = scratch_bytes(o, 2 * cb + 4 * fb);
    if (!base)
        return;
    cudaStream_t st = coreg::stream_of(o->ocl);
    cudaSetDevice(o->ocl->device);
    unsigned char *v1 = valid1 ? (unsigned char *)base : nullptr;
    unsigned char *v2 = valid2 ? (unsigned char *)base + cb : nullptr;
    if (v1)
        cudaMemcpyAsync(v1, valid1, cells, cudaMemcpyHostToDevice, st);
    if (v2)
        cudaMemcpyAsync(v2, valid2, cells, cudaMemcpyHostToDevice, st);
    float *f = (float *)(base + 2 * cb);
    float *ddx = f, *ddy = (float *)((char *)f + fb), *dc = (float *)((char *)f + 2 * fb),
          *ds = (float *)((char *)f + 3 * fb);
    dense_field_k<<<coreg::cdiv((long)cells, 256), 256, 0, st>>>(
        flow, cert, sd, H, W, h, w, v1, v2, ddx, ddy, dc, sdo ? ds : nullptr);
    if (!coreg::launch_ok("roma_dense_field_dev"))
        return;
    cudaMemcpyAsync(dx, ddx, cells * 4, cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(dy, ddy, cells * 4, cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(certo, dc, cells * 4, cudaMemcpyDeviceToHost, st);
    if (sdo)
        cudaMemcpyAsync(sdo, ds, cells * 4, cudaMemcpyDeviceToHost, st);
    cuda_ok(cudaStreamSynchronize(st), "roma_dense_field_dev");
}

namespace {

struct roma_state {
    struct roma_model net;
    int spacing;
    float min_cert;
    float *bflow;      // with m->cycle: reverse warp (2, H, W), host
    float *bflow_dev;  // and its device copy, which the device stage reads
};

void roma_m_alloc(struct matcher *m, int H, int W)
{
    roma_state *s = (roma_state *)m->state;
    roma_alloc(&s->net, H, W);
    if (m->cycle && !pending()) {
        s->bflow = (float *)realloc(s->bflow, 2 * (size_t)H * W * sizeof(float));
        if (!s->bflow_dev)
            cuda_ok(cudaMalloc((void **)&s->bflow_dev, 2 * (size_t)H * W * sizeof(float)),
                    "RoMa reverse warp");
    }
}

// matcher_roma.c:41-55: the reverse warp first, so that the forward one
// stays in the model (and the dumps).
void roma_m_run(struct matcher *m, const struct matcher_tile *t)
{
    roma_state *s = (roma_state *)m->state;
    if (pending())
        return;
    if (t->H != s->net.H || t->W != s->net.W) {
        fail("RoMa tile %d x %d differs from its buffers", t->H, t->W);
        return;
    }
    if (m->cycle) {
        roma_match(&s->net, t->img2, t->img1, NULL, t->index);
        memcpy(s->bflow, s->net.flow, 2 * (size_t)t->H * t->W * sizeof(float));
        float *f = nullptr;
        roma_results_dev(&s->net, &f, nullptr, nullptr);
        if (f && s->bflow_dev)
            cuda_ok(cudaMemcpyAsync(s->bflow_dev, f, 2 * (size_t)t->H * t->W * sizeof(float),
                                    cudaMemcpyDeviceToDevice, coreg::stream_of(s->net.ocl)),
                    "RoMa reverse warp");
    }
    roma_match(&s->net, t->img1, t->img2, m->dump_dir, t->index);
}

int roma_m_match(struct matcher *m, const struct matcher_tile *t,
                 struct match_list *out)
{
    roma_state *s = (roma_state *)m->state;
    if (pending())
        return 0;
    // On the device, from the results run left there (the host copies
    // stay for field users and dumps); the same matches as the host stage.
    float *flow = nullptr, *cert = nullptr, *sd = nullptr;
    roma_results_dev(&s->net, &flow, &cert, &sd);
    return roma_sample_matches_dev(m->ops, flow, cert, sd, m->cycle ? s->bflow_dev : nullptr,
                                   t->H, t->W, t->h, t->w, s->spacing, s->min_cert, t->valid1,
                                   t->valid2, out);
}

void roma_m_field(struct matcher *m, const struct matcher_tile *t, float *dx,
                  float *dy, float *cert, float *sdo)
{
    roma_state *s = (roma_state *)m->state;
    if (pending())
        return;
    float *flow = nullptr, *ce = nullptr, *sd = nullptr;
    roma_results_dev(&s->net, &flow, &ce, &sd);
    roma_dense_field_dev(m->ops, flow, ce, sd, t->H, t->W, t->h, t->w, t->valid1, t->valid2,
                         dx, dy, cert, sdo);
}

void roma_m_dump(struct matcher *m, const struct matcher_tile *t,
                 const char *dir)
{
    roma_state *s = (roma_state *)m->state;
    char path[4096];
    snprintf(path, sizeof(path), "%s/tile%03d_roma.txt", dir, t->index);
    FILE *fp = fopen(path, "w");
    if (!fp) {
        fail("Unable to write debug dump <%s>", path);
        return;
    }
    fprintf(fp, "x0 %d y0 %d w %d h %d H %d W %d coarse %d\n", t->x0, t->y0,
            t->w, t->h, t->H, t->W, s->net.coarse);
    fclose(fp);
}

void roma_m_destroy(struct matcher *m)
{
    roma_state *s = (roma_state *)m->state;
    if (!s)
        return;
    roma_free(&s->net);
    free(s->bflow);
    if (s->bflow_dev)
        cudaFree(s->bflow_dev);
    free(s);
    m->state = NULL;
}

}  // namespace

extern "C" void matcher_roma_create(struct matcher *m, struct ops *ops,
                                    struct pth_file *pf, struct pth_file *dino,
                                    struct pth_file *v2, const char *name,
                                    int imagenet, int spacing, float min_cert)
{
    roma_state *s = (roma_state *)calloc(1, sizeof(*s));
    memset(m, 0, sizeof(*m));
    roma_load(&s->net, ops, pf, dino);
    if (v2)
        roma_load_v2(&s->net, v2);
    s->net.imagenet = imagenet;
    s->spacing = spacing;
    s->min_cert = min_cert;
    m->name = name;
    m->multiple = ROMA_MULTIPLE;
    m->ops = ops;
    m->state = s;
    m->alloc = roma_m_alloc;
    m->run = roma_m_run;
    m->match = roma_m_match;
    m->dump = roma_m_dump;
    m->field = roma_m_field;
    m->has_sd = v2 != NULL;
    m->destroy = roma_m_destroy;
}
