// SPDX-License-Identifier: Unlicense
//
// The DISK matcher (matcher_disk.h): the struct matcher glue of the
// reference's matcher_disk.c around disk.h and adalam.h. run detects the
// keypoints of both images (disk_detect); match pairs them (adalam_match:
// nearest neighbours on the device, AdaLAM on the host) and reports each
// accepted pair at its whole cells with AdaLAM's inverse confidence as
// cost; dump writes the reference's dump files (inputs, keypoint rows x,
// y, score, descriptor, and the matches as "i1 i2 dist").

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <vector>

#include "common.cuh"
#include "disk.h"
#include "matcher_disk.h"

namespace {

struct disk_state {
    struct disk_model disk;
    struct disk_matcher_config cfg;
    std::vector<int> xy1, xy2;
    std::vector<float> s1, s2, d1, d2;
    int n1 = 0, n2 = 0;
    // The last tile's matches, for dump.
    int nm = 0;
    int *pairs = nullptr;
    float *dist = nullptr;
};

void dk_alloc(struct matcher *m, int H, int W)
{
    disk_state *s = (disk_state *)m->state;
    const int n = s->cfg.features;
    disk_alloc(&s->disk, H, W, n);
    s->xy1.resize(2 * (size_t)n);
    s->xy2.resize(2 * (size_t)n);
    s->s1.resize(n);
    s->s2.resize(n);
    s->d1.resize((size_t)n * DISK_DESC);
    s->d2.resize((size_t)n * DISK_DESC);
}

void dk_run(struct matcher *m, const struct matcher_tile *t)
{
    disk_state *s = (disk_state *)m->state;
    if (coreg::pending())
        return;
    const int n = s->cfg.features;
    const float th = s->cfg.threshold;
    s->n1 = disk_detect(&s->disk, t->img1, t->H, t->W, t->h, t->w, n, th, t->valid1,
                        s->xy1.data(), s->s1.data(), s->d1.data());
    s->n2 = disk_detect(&s->disk, t->img2, t->H, t->W, t->h, t->w, n, th, t->valid2,
                        s->xy2.data(), s->s2.data(), s->d2.data());
}

int dk_match(struct matcher *m, const struct matcher_tile *t, struct match_list *out)
{
    (void)t;
    disk_state *s = (disk_state *)m->state;
    free(s->pairs);
    free(s->dist);
    s->pairs = nullptr;
    s->dist = nullptr;
    s->nm = 0;
    if (coreg::pending())
        return 0;
    std::vector<float> k1(s->xy1.begin(), s->xy1.begin() + 2 * (size_t)s->n1);
    std::vector<float> k2(s->xy2.begin(), s->xy2.begin() + 2 * (size_t)s->n2);
    s->nm = adalam_match(m->ops, k1.data(), s->d1.data(), s->n1, k2.data(), s->d2.data(), s->n2,
                         DISK_DESC, &s->cfg.adalam, &s->pairs, &s->dist);
    for (int i = 0; i < s->nm; i++) {
        const int a = s->pairs[2 * i], b = s->pairs[2 * i + 1];
        struct match mt;
        mt.x1 = s->xy1[2 * a];
        mt.y1 = s->xy1[2 * a + 1];
        mt.x2 = s->xy2[2 * b];
        mt.y2 = s->xy2[2 * b + 1];
        mt.cost = s->dist[i];
        mt.sd = NAN;
        mt.cycle = NAN;
        match_add(out, &mt);
    }
    return s->nm;
}

// Keypoint rows of float32: x, y, score, then the descriptor.
void dump_keypoints(const char *dir, int tile, const char *what, const int *xy,
                    const float *score, const float *desc, int n)
{
    const size_t row = 3 + DISK_DESC;
    std::vector<float> v(n * row);
    for (int i = 0; i < n; i++) {
        v[i * row] = (float)xy[2 * i];
        v[i * row + 1] = (float)xy[2 * i + 1];
        v[i * row + 2] = score[i];
        memcpy(&v[i * row + 3], desc + (size_t)i * DISK_DESC, DISK_DESC * sizeof(float));
    }
    matcher_dump_file(dir, tile, what, v.data(), v.size() * sizeof(float));
}

void dk_dump(struct matcher *m, const struct matcher_tile *t, const char *dir)
{
    disk_state *s = (disk_state *)m->state;
    const size_t bytes = 3 * (size_t)t->H * t->W * sizeof(float);
    matcher_dump_file(dir, t->index, "src_input.f32", t->img1, bytes);
    matcher_dump_file(dir, t->index, "ref_input.f32", t->img2, bytes);
    dump_keypoints(dir, t->index, "src_kp.f32", s->xy1.data(), s->s1.data(), s->d1.data(),
                   s->n1);
    dump_keypoints(dir, t->index, "ref_kp.f32", s->xy2.data(), s->s2.data(), s->d2.data(),
                   s->n2);
    char path[4096];
    snprintf(path, sizeof(path), "%s/tile%03d_matches.txt", dir, t->index);
    FILE *fp = fopen(path, "w");
    if (!fp) {
        coreg::fail("Unable to write debug dump <%s>", path);
        return;
    }
    fprintf(fp, "# x0 %d y0 %d w %d h %d H %d W %d\n", t->x0, t->y0, t->w, t->h, t->H, t->W);
    for (int i = 0; i < s->nm; i++)
        fprintf(fp, "%d %d %.9g\n", s->pairs[2 * i], s->pairs[2 * i + 1], s->dist[i]);
    fclose(fp);
}

void dk_destroy(struct matcher *m)
{
    disk_state *s = (disk_state *)m->state;
    if (s) {
        disk_free(&s->disk);
        free(s->pairs);
        free(s->dist);
        delete s;
    }
    m->state = nullptr;
}

}  // namespace

extern "C" void matcher_disk_create(struct matcher *m, struct ops *ops, struct pth_file *pf,
                                    const struct disk_matcher_config *cfg)
{
    memset(m, 0, sizeof(*m));
    if (coreg::pending())
        return;
    disk_state *s = new disk_state();
    s->cfg = *cfg;
    disk_load(&s->disk, ops, pf);
    m->name = "disk";
    m->multiple = DISK_MULTIPLE;
    m->ops = ops;
    m->state = s;
    m->alloc = dk_alloc;
    m->run = dk_run;
    m->match = dk_match;
    m->dump = dk_dump;
    m->destroy = dk_destroy;
}
