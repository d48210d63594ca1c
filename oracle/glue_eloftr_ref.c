/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the reference's Efficient LoFTR matcher glue
 * (matcher_eloftr.c), compiled where it lies (the Makefile names it by
 * path in REF_MATCHER_ELOFTR_C), with its static host stage
 * (eloftr_m_match, matcher_eloftr.c:66-96) called on given keypoints. The
 * network entry points are never reached here and are stubs. Built with
 * glue_roma_ref.c into _ref/libglue_ref.so by oracle/Makefile. */

#include REF_MATCHER_ELOFTR_C

void eloftr_load(struct eloftr_model *m, struct ops *ops, struct pth_file *pf)
{
    (void)m, (void)ops, (void)pf;
}
void eloftr_alloc(struct eloftr_model *m, int H, int W) { (void)m, (void)H, (void)W; }
void eloftr_match(struct eloftr_model *m, const float *g0, const float *g1, const char *dump,
                  int tile)
{
    (void)m, (void)g0, (void)g1, (void)dump, (void)tile;
}
void eloftr_free(struct eloftr_model *m) { (void)m; }

int glue_rows(struct match_list *l, double *rows, int cap);

int ref_eloftr_sample(const float *kp, const float *mconf, int nm, int h, int w,
                      const unsigned char *valid1, const unsigned char *valid2, double *rows,
                      int cap)
{
    struct eloftr_state s;
    struct matcher m;
    struct matcher_tile t;
    struct match_list l = {0, 0, NULL};

    memset(&s, 0, sizeof(s));
    memset(&m, 0, sizeof(m));
    memset(&t, 0, sizeof(t));
    s.net.nm = nm;
    s.net.kp = (float *)kp;
    s.net.mconf = (float *)mconf;
    m.state = &s;
    t.h = h;
    t.w = w;
    t.valid1 = valid1;
    t.valid2 = valid2;
    t.index = 1;
    eloftr_m_match(&m, &t, &l);
    return glue_rows(&l, rows, cap);
}
