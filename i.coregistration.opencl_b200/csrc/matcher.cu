// SPDX-License-Identifier: Unlicense
//
// The matcher interface (matcher.h) and the RoMa matcher
// (matcher_roma.h): the device stage through roma_match, the host stage
// with the reference's sampling rules (matcher_roma.c:41-232).

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

// Cycle error (matcher_roma.c:61-90): distance from (x, y) to the reverse
// warp at (xr, yr), bilinear between the tile's cells.
float cycle_error(const roma_state *s, const struct matcher_tile *t, int x,
                  int y, double xr, double yr)
{
    const size_t hw = (size_t)t->H * t->W;
    double bx = 0, by = 0;
    xr = xr < 0 ? 0 : xr > t->w - 1 ? t->w - 1 : xr;
    yr = yr < 0 ? 0 : yr > t->h - 1 ? t->h - 1 : yr;
    int x0 = (int)xr < t->w - 1 ? (int)xr : t->w - 1;
    int y0 = (int)yr < t->h - 1 ? (int)yr : t->h - 1;
    if (t->w == 1 || t->h == 1)
        return NAN;
    if (x0 == t->w - 1)
        x0--;
    if (y0 == t->h - 1)
        y0--;
    const double fx = xr - x0, fy = yr - y0;
    for (int j = 0; j < 2; j++)
        for (int i = 0; i < 2; i++) {
            const size_t k = (size_t)(y0 + j) * t->W + x0 + i;
            const double wgt = (i ? fx : 1 - fx) * (j ? fy : 1 - fy);
            bx += wgt * ((s->bflow[k] + 1.0) * 0.5 * t->W - 0.5);
            by += wgt * ((s->bflow[hw + k] + 1.0) * 0.5 * t->H - 0.5);
        }
    return (float)hypot(bx - x, by - y);
}

int valid_at(const unsigned char *v, int h, int w, double x, double y)
{
    const long ix = lround(x), iy = lround(y);
    return ix >= 0 && iy >= 0 && ix < w && iy < h &&
           (!v || v[(size_t)iy * w + ix]);
}

// matcher_roma.c:103-145.
int roma_m_match(struct matcher *m, const struct matcher_tile *t,
                 struct match_list *out)
{
    roma_state *s = (roma_state *)m->state;
    const float *cert = s->net.cert, *flow = s->net.flow, *sd = s->net.sd;
    const size_t hw = (size_t)t->H * t->W;
    const int S = s->spacing;
    int n = 0;
    if (pending())
        return 0;
    for (int by = 0; by < t->h; by += S)
        for (int bx = 0; bx < t->w; bx += S) {
            const int bxe = bx + S < t->w ? bx + S : t->w;
            const int bye = by + S < t->h ? by + S : t->h;
            long best = -1;
            for (int y = by; y < bye; y++)
                for (int x = bx; x < bxe; x++) {
                    const size_t i = (size_t)y * t->W + x;
                    if (t->valid1 && !t->valid1[(size_t)y * t->w + x])
                        continue;
                    if (best < 0 || cert[i] > cert[best])
                        best = (long)i;
                }
            if (best < 0 || !(cert[best] >= s->min_cert))
                continue;
            struct match mt;
            mt.x1 = best % t->W;
            mt.y1 = best / t->W;
            mt.x2 = (flow[best] + 1.0) * 0.5 * t->W - 0.5;
            mt.y2 = (flow[hw + best] + 1.0) * 0.5 * t->H - 0.5;
            mt.cost = 1.0f - cert[best];
            mt.sd = sd ? sd[best] : NAN;
            if (!valid_at(t->valid2, t->h, t->w, mt.x2, mt.y2))
                continue;
            mt.cycle = m->cycle ? cycle_error(s, t, (int)mt.x1, (int)mt.y1, mt.x2,
                                              mt.y2)
                                : NAN;
            match_add(out, &mt);
            n++;
        }
    return n;
}

// matcher_roma.c:150-178.
void roma_m_field(struct matcher *m, const struct matcher_tile *t, float *dx,
                  float *dy, float *cert, float *sdo)
{
    roma_state *s = (roma_state *)m->state;
    const float *c = s->net.cert, *flow = s->net.flow;
    const size_t hw = (size_t)t->H * t->W;
    for (int y = 0; y < t->h; y++)
        for (int x = 0; x < t->w; x++) {
            const size_t i = (size_t)y * t->W + x, o = (size_t)y * t->w + x;
            const double xr = (flow[i] + 1.0) * 0.5 * t->W - 0.5;
            const double yr = (flow[hw + i] + 1.0) * 0.5 * t->H - 0.5;
            if ((t->valid1 && !t->valid1[o]) ||
                !valid_at(t->valid2, t->h, t->w, xr, yr)) {
                dx[o] = dy[o] = NAN;
                cert[o] = 0.0f;
                if (sdo)
                    sdo[o] = NAN;
                continue;
            }
            dx[o] = (float)(xr - x);
            dy[o] = (float)(yr - y);
            cert[o] = c[i];
            if (sdo)
                sdo[o] = s->net.sd ? s->net.sd[i] : NAN;
        }
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
