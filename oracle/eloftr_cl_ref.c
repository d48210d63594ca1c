/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the reference's Efficient LoFTR kernels
 * (eloftr_kernels.cl: the blockwise dual-softmax passes and the two-stage
 * fine matching) compiled as C through cl_emul.h and run on the CPU with
 * the reference's work-group sizes. The build compiles a copy of the file
 * whose float4 literals are rewritten to emul_float4 (oracle/Makefile,
 * REF_ELOFTR_KERNELS_CL). Built into _ref/libeloftr_cl_ref.so. */

#include "cl_emul.h"

#include REF_ELOFTR_KERNELS_CL

#define LAUNCH(body, a, g0, l0)                                                              \
    do {                                                                                     \
        const size_t g_[3] = {(g0), 1, 1}, l_[3] = {(l0), 1, 1};                             \
        emul_launch((body), &(a), g_, l_);                                                   \
    } while (0)

struct a_rl { const float *S; int N, r0, R; float *lse; };
static void b_rl(void *p)
{
    struct a_rl *a = p;
    eloftr_row_lse(a->S, a->N, a->r0, a->lse);
}
/* Row log-sum-exp of the block S (R x N) into lse[r0 ..]. */
void ref_row_lse(const float *S, int R, int N, int r0, float *lse)
{
    struct a_rl a = {S, N, r0, R, lse};
    LAUNCH(b_rl, a, (size_t)R * 256, 256);
}

struct a_cl { const float *S; int R, N; float *cm, *cs; };
static void b_cl(void *p)
{
    struct a_cl *a = p;
    eloftr_col_lse(a->S, a->R, a->N, a->cm, a->cs);
}
void ref_col_lse(const float *S, int R, int N, float *cm, float *cs)
{
    struct a_cl a = {S, R, N, cm, cs};
    LAUNCH(b_cl, a, (size_t)N, 1);
}

struct a_cr { const float *S; int N, r0; const float *lse, *cm, *cs; float *rmax; int *rarg; };
static void b_cr(void *p)
{
    struct a_cr *a = p;
    eloftr_conf_row(a->S, a->N, a->r0, a->lse, a->cm, a->cs, a->rmax, a->rarg);
}
void ref_conf_row(const float *S, int R, int N, int r0, const float *lse, const float *cm,
                  const float *cs, float *rmax, int *rarg)
{
    struct a_cr a = {S, N, r0, lse, cm, cs, rmax, rarg};
    LAUNCH(b_cr, a, (size_t)R * 256, 256);
}

struct a_cc { const float *S; int R, N, r0; const float *lse, *cm, *cs; float *cmax; int *carg; };
static void b_cc(void *p)
{
    struct a_cc *a = p;
    eloftr_conf_col(a->S, a->R, a->N, a->r0, a->lse, a->cm, a->cs, a->cmax, a->carg);
}
void ref_conf_col(const float *S, int R, int N, int r0, const float *lse, const float *cm,
                  const float *cs, float *cmax, int *carg)
{
    struct a_cc a = {S, R, N, r0, lse, cm, cs, cmax, carg};
    LAUNCH(b_cc, a, (size_t)N, 1);
}

struct a_fine { const float *f0, *f1; int H, W; const int4 *cells; int M; float T; float4 *out; };
static void b_fine(void *p)
{
    struct a_fine *a = p;
    eloftr_fine(a->f0, a->f1, a->H, a->W, a->cells, a->M, a->T, a->out);
}
/* Both fine stages for M matches: cells (x0, y0, x1, y1) per match,
 * out (x0, y0, x1, y1) in pixels. */
void ref_fine(const float *f0, const float *f1, int H, int W, const int *cells, int M, float T,
              float *out)
{
    struct a_fine a = {f0, f1, H, W, (const int4 *)cells, M, T, (float4 *)out};
    LAUNCH(b_fine, a, (size_t)M * 256, 256);
}
