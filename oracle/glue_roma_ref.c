/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the reference's match list (matcher.c) and RoMa
 * matcher glue (matcher_roma.c), compiled where they lie (the Makefile
 * names them by path in REF_MATCHER_C and REF_MATCHER_ROMA_C), with
 * matcher_roma.c's static host stage (roma_m_match, matcher_roma.c:103-145,
 * with cycle_error :61-90; roma_m_field :150-178) called on given results.
 * The network entry points the glue references are never reached here and
 * are stubs. Built into _ref/libglue_ref.so by oracle/Makefile. */

#include REF_MATCHER_C
#include REF_MATCHER_ROMA_C

#include <stdlib.h>

void roma_load(struct roma_model *m, struct ops *ops, struct pth_file *pf,
               struct pth_file *dino)
{
    (void)m, (void)ops, (void)pf, (void)dino;
}
void roma_load_v2(struct roma_model *m, struct pth_file *pf) { (void)m, (void)pf; }
void roma_alloc(struct roma_model *m, int H, int W) { (void)m, (void)H, (void)W; }
void roma_match(struct roma_model *m, const float *a, const float *b, const char *dump,
                int tile)
{
    (void)m, (void)a, (void)b, (void)dump, (void)tile;
}
void roma_free(struct roma_model *m) { (void)m; }

/* Copies a match list to rows of 7 doubles (x1, y1, x2, y2, cost, sd,
 * cycle), at most cap rows, and frees it; returns its length. */
int glue_rows(struct match_list *l, double *rows, int cap)
{
    int i;

    for (i = 0; i < l->n && i < cap; i++) {
        const struct match *m = &l->v[i];
        double *r = rows + 7 * (size_t)i;

        r[0] = m->x1;
        r[1] = m->y1;
        r[2] = m->x2;
        r[3] = m->y2;
        r[4] = m->cost;
        r[5] = m->sd;
        r[6] = m->cycle;
    }
    free(l->v);
    return l->n;
}

static void glue_setup(struct roma_state *s, struct matcher *m, struct matcher_tile *t,
                       const float *flow, const float *cert, const float *sd,
                       const float *bflow, int H, int W, int h, int w, int spacing,
                       float min_cert, const unsigned char *valid1,
                       const unsigned char *valid2)
{
    memset(s, 0, sizeof(*s));
    memset(m, 0, sizeof(*m));
    memset(t, 0, sizeof(*t));
    s->net.flow = (float *)flow;
    s->net.cert = (float *)cert;
    s->net.sd = (float *)sd;
    s->net.H = H;
    s->net.W = W;
    s->spacing = spacing;
    s->min_cert = min_cert;
    s->bflow = (float *)bflow;
    m->state = s;
    m->cycle = bflow != NULL;
    t->H = H;
    t->W = W;
    t->h = h;
    t->w = w;
    t->valid1 = valid1;
    t->valid2 = valid2;
    t->index = 1;
}

int ref_roma_sample(const float *flow, const float *cert, const float *sd, const float *bflow,
                    int H, int W, int h, int w, int spacing, float min_cert,
                    const unsigned char *valid1, const unsigned char *valid2, double *rows,
                    int cap)
{
    struct roma_state s;
    struct matcher m;
    struct matcher_tile t;
    struct match_list l = {0, 0, NULL};

    glue_setup(&s, &m, &t, flow, cert, sd, bflow, H, W, h, w, spacing, min_cert, valid1,
               valid2);
    roma_m_match(&m, &t, &l);
    return glue_rows(&l, rows, cap);
}

void ref_roma_field(const float *flow, const float *cert, const float *sd, int H, int W, int h,
                    int w, const unsigned char *valid1, const unsigned char *valid2, float *dx,
                    float *dy, float *certo, float *sdo)
{
    struct roma_state s;
    struct matcher m;
    struct matcher_tile t;

    glue_setup(&s, &m, &t, flow, cert, sd, NULL, H, W, h, w, 1, 0.0f, valid1, valid2);
    roma_m_field(&m, &t, dx, dy, certo, sdo);
}
