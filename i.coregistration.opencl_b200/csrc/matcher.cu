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

#include "common.cuh"
#include "matcher_roma.h"
#include "roma.h"

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

namespace {

struct roma_state {
    struct roma_model net;
    int spacing;
    float min_cert;
    float *bflow; // with m->cycle: reverse warp (2, H, W)
};

void roma_m_alloc(struct matcher *m, int H, int W)
{
    roma_state *s = (roma_state *)m->state;
    roma_alloc(&s->net, H, W);
    if (m->cycle)
        s->bflow = (float *)realloc(s->bflow, 2 * (size_t)H * W * sizeof(float));
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
    }
    roma_match(&s->net, t->img1, t->img2, m->dump_dir, t->index);
}

int roma_m_match(struct matcher *m, const struct matcher_tile *t,
                 struct match_list *out)
{
    roma_state *s = (roma_state *)m->state;
    if (pending())
        return 0;
    return roma_sample_matches(s->net.flow, s->net.cert, s->net.sd,
                               m->cycle ? s->bflow : nullptr, t->H, t->W, t->h,
                               t->w, s->spacing, s->min_cert, t->valid1,
                               t->valid2, out);
}

void roma_m_field(struct matcher *m, const struct matcher_tile *t, float *dx,
                  float *dy, float *cert, float *sdo)
{
    roma_state *s = (roma_state *)m->state;
    if (pending())
        return;
    roma_dense_field(s->net.flow, s->net.cert, s->net.sd, t->H, t->W, t->h,
                     t->w, t->valid1, t->valid2, dx, dy, cert, sdo);
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
