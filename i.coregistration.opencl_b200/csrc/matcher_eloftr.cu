// SPDX-License-Identifier: Unlicense
//
// The Efficient LoFTR matcher (matcher_eloftr.h): the struct matcher glue of
// the reference's matcher_eloftr.c around eloftr.h, with its semantics
// (grey conversion, the npe position scale, cost 1 - confidence, the
// +3.5 pixel offset of the keypoint convention, validity by rounded
// position).

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <vector>

#include "common.cuh"
#include "eloftr.h"
#include "matcher_eloftr.h"

namespace {

constexpr double KP_OFFSET = 3.5;

struct eloftr_state {
    struct eloftr_model net;
    int npe = 0;
    std::vector<float> grey0, grey1;
};

void to_grey(const float *rgb, int H, int W, float *grey)
{
    const size_t p = (size_t)H * W;
    for (size_t i = 0; i < p; i++)
        grey[i] = 0.2989f * rgb[i] + 0.5870f * rgb[p + i] + 0.1140f * rgb[2 * p + i];
}

void el_alloc(struct matcher *m, int H, int W)
{
    eloftr_state *s = (eloftr_state *)m->state;
    if (s->npe)
        s->net.pos_scale = (float)ELOFTR_TRAIN_RES / (H > W ? H : W);
    eloftr_alloc(&s->net, H, W);
    s->grey0.resize((size_t)H * W);
    s->grey1.resize((size_t)H * W);
}

void el_run(struct matcher *m, const struct matcher_tile *t)
{
    eloftr_state *s = (eloftr_state *)m->state;
    if (coreg::pending())
        return;
    if (t->H != s->net.H || t->W != s->net.W) {
        coreg::fail("ELoFTR tile %d x %d differs from its buffers", t->H, t->W);
        return;
    }
    to_grey(t->img1, t->H, t->W, s->grey0.data());
    to_grey(t->img2, t->H, t->W, s->grey1.data());
    eloftr_match(&s->net, s->grey0.data(), s->grey1.data(), m->dump_dir, t->index);
}

int el_match(struct matcher *m, const struct matcher_tile *t, struct match_list *out)
{
    eloftr_state *s = (eloftr_state *)m->state;
    if (coreg::pending())
        return 0;
    return eloftr_sample_matches(s->net.kp, s->net.mconf, s->net.nm, t->h, t->w, t->valid1,
                                 t->valid2, out);
}

void el_dump(struct matcher *m, const struct matcher_tile *t, const char *dir)
{
    eloftr_state *s = (eloftr_state *)m->state;
    const size_t bytes = (size_t)t->H * t->W * sizeof(float);
    matcher_dump_file(dir, t->index, "eloftr_grey_0.f32", s->grey0.data(), bytes);
    matcher_dump_file(dir, t->index, "eloftr_grey_1.f32", s->grey1.data(), bytes);
    char path[4096];
    snprintf(path, sizeof(path), "%s/tile%03d_eloftr_matches.txt", dir, t->index);
    FILE *fp = fopen(path, "w");
    if (!fp) {
        coreg::fail("Unable to write debug dump <%s>", path);
        return;
    }
    fprintf(fp, "# x0 %d y0 %d w %d h %d H %d W %d pos_scale %.9g\n", t->x0, t->y0, t->w, t->h,
            t->H, t->W, s->net.pos_scale);
    for (int i = 0; i < s->net.nm; i++) {
        const float *k = s->net.kp + 4 * (size_t)i;
        fprintf(fp, "%d %d %.9g %.6f %.6f %.6f %.6f\n", s->net.mi[i], s->net.mj[i],
                s->net.mconf[i], k[0], k[1], k[2], k[3]);
    }
    fclose(fp);
}

void el_destroy(struct matcher *m)
{
    eloftr_state *s = (eloftr_state *)m->state;
    if (s) {
        eloftr_free(&s->net);
        delete s;
    }
    m->state = nullptr;
}

}  // namespace

// The matches of the keypoint pairs kp (x0, y0, x1, y1 in the network's
// convention, KP_OFFSET from the cells') whose both ends round to valid
// cells (matcher_eloftr.c:66-96).
extern "C" int eloftr_sample_matches(const float *kp, const float *mconf, int nm, int h, int w,
                                     const unsigned char *valid1,
                                     const unsigned char *valid2, struct match_list *out)
{
    if (coreg::pending())
        return 0;
    const auto on_valid = [h, w](const unsigned char *v, double x, double y) {
        const long ix = lround(x), iy = lround(y);
        return ix >= 0 && iy >= 0 && ix < w && iy < h && (!v || v[(size_t)iy * w + ix]);
    };
    int n = 0;
    for (int i = 0; i < nm; i++) {
        const float *k = kp + 4 * (size_t)i;
        struct match mt;
        mt.x1 = k[0] + KP_OFFSET;
        mt.y1 = k[1] + KP_OFFSET;
        mt.x2 = k[2] + KP_OFFSET;
        mt.y2 = k[3] + KP_OFFSET;
        if (!on_valid(valid1, mt.x1, mt.y1) || !on_valid(valid2, mt.x2, mt.y2))
            continue;
        mt.cost = 1.0f - mconf[i];
        mt.sd = NAN;
        mt.cycle = NAN;
        match_add(out, &mt);
        n++;
    }
    return n;
}

extern "C" void matcher_eloftr_create(struct matcher *m, struct ops *ops, struct pth_file *pf,
                                      const char *name, int npe)
{
    memset(m, 0, sizeof(*m));
    if (coreg::pending())
        return;
    eloftr_state *s = new eloftr_state();
    eloftr_load(&s->net, ops, pf);
    s->npe = npe;
    m->name = name;
    m->multiple = ELOFTR_MULTIPLE;
    m->ops = ops;
    m->state = s;
    m->alloc = el_alloc;
    m->run = el_run;
    m->match = el_match;
    m->dump = el_dump;
    m->destroy = el_destroy;
}
