/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the reference's RoMa kernels (roma_kernels.cl),
 * compiled where they lie as C through cl_emul.h (the Makefile names the
 * file by path in REF_ROMA_KERNELS_CL) and run on the CPU with the
 * work-group sizes the reference launches them with. One ref_<kernel>
 * entry point per kernel, with the kernel's arguments. Built into
 * _ref/libroma_cl_ref.so by oracle/Makefile. */

#include "cl_emul.h"

#include REF_ROMA_KERNELS_CL

#define LAUNCH(body, a, g0, g1, g2, l0, l1, l2)                                              \
    do {                                                                                     \
        const size_t g_[3] = {(g0), (g1), (g2)}, l_[3] = {(l0), (l1), (l2)};                 \
        emul_launch((body), &(a), g_, l_);                                                   \
    } while (0)

static size_t up(size_t n, size_t m) { return (n + m - 1) / m * m; }

struct a_row_norm { const float *X; int rows, C; float *out; };
static void b_row_norm(void *p)
{
    struct a_row_norm *a = p;
    roma_row_norm(a->X, a->rows, a->C, a->out);
}
void ref_row_norm(const float *X, int rows, int C, float *out)
{
    struct a_row_norm a = {X, rows, C, out};
    LAUNCH(b_row_norm, a, (size_t)rows, 1, 1, 1, 1, 1);
}

struct a_cos_exp { float *S; const float *nx, *ny; int N, M; float T, eps; };
static void b_cos_exp(void *p)
{
    struct a_cos_exp *a = p;
    roma_cos_exp(a->S, a->nx, a->ny, a->N, a->M, a->T, a->eps);
}
void ref_cos_exp(float *S, const float *nx, const float *ny, int N, int M, float T, float eps)
{
    struct a_cos_exp a = {S, nx, ny, N, M, T, eps};
    LAUNCH(b_cos_exp, a, (size_t)M, (size_t)N, 1, 1, 1, 1);
}

struct a_cls { const float *L; int ld, C, res, n; float *flow, *cert; };
static void b_cls(void *p)
{
    struct a_cls *a = p;
    roma_cls_to_flow(a->L, a->ld, a->C, a->res, a->n, a->flow, a->cert);
}
void ref_cls_to_flow(const float *L, int ld, int C, int res, int n, float *flow, float *cert)
{
    struct a_cls a = {L, ld, C, res, n, flow, cert};
    LAUNCH(b_cls, a, (size_t)n * 256, 1, 1, 256, 1, 1);
}

struct a_ws { const float *in; int C, H, W; const float *flow; float *out; int coff; };
static void b_ws(void *p)
{
    struct a_ws *a = p;
    roma_warp_sample(a->in, a->C, a->H, a->W, a->flow, a->out, a->coff);
}
void ref_warp_sample(const float *in, int C, int H, int W, const float *flow, float *out, int coff)
{
    struct a_ws a = {in, C, H, W, flow, out, coff};
    LAUNCH(b_ws, a, (size_t)H * W, (size_t)C, 1, 1, 1, 1);
}

struct a_lc { const float *f1, *f2; int C, H, W, r; const float *flow; float *out; int coff; };
static void b_lc(void *p)
{
    struct a_lc *a = p;
    roma_local_corr(a->f1, a->f2, a->C, a->H, a->W, a->r, a->flow, a->out, a->coff);
}
void ref_local_corr(const float *f1, const float *f2, int C, int H, int W, int r,
                    const float *flow, float *out, int coff)
{
    struct a_lc a = {f1, f2, C, H, W, r, flow, out, coff};
    LAUNCH(b_lc, a, (size_t)H * W * CORR_WG, 1, 1, CORR_WG, 1, 1);
}

struct a_disp { const float *flow; int H, W; float fx, fy; float *out; };
static void b_disp(void *p)
{
    struct a_disp *a = p;
    roma_disp(a->flow, a->H, a->W, a->fx, a->fy, a->out);
}
void ref_disp(const float *flow, int H, int W, float fx, float fy, float *out)
{
    struct a_disp a = {flow, H, W, fx, fy, out};
    LAUNCH(b_disp, a, (size_t)H * W, 1, 1, 1, 1, 1);
}

struct a_up { float *flow, *cert; const float *d; int n; float scale, Wf, Hf; };
static void b_up(void *p)
{
    struct a_up *a = p;
    roma_update(a->flow, a->cert, a->d, a->n, a->scale, a->Wf, a->Hf);
}
void ref_update(float *flow, float *cert, const float *d, int n, float scale, float Wf, float Hf)
{
    struct a_up a = {flow, cert, d, n, scale, Wf, Hf};
    LAUNCH(b_up, a, (size_t)n, 1, 1, 1, 1, 1);
}

struct a_up2 { float *flow, *conf; const float *d; int n; float W, H; };
static void b_up2(void *p)
{
    struct a_up2 *a = p;
    roma2_update(a->flow, a->conf, a->d, a->n, a->W, a->H);
}
void ref_update2(float *flow, float *conf, const float *d, int n, float W, float H)
{
    struct a_up2 a = {flow, conf, d, n, W, H};
    LAUNCH(b_up2, a, (size_t)n, 1, 1, 1, 1, 1);
}

struct a_dw { const float *in; int H, W; const float *wt, *bias; float *out; int C; };
static void b_dw(void *p)
{
    struct a_dw *a = p;
    roma_dwconv5(a->in, a->H, a->W, a->wt, a->bias, a->out);
}
void ref_dwconv5(const float *in, int C, int H, int W, const float *wt, const float *bias,
                 float *out)
{
    struct a_dw a = {in, H, W, wt, bias, out, C};
    LAUNCH(b_dw, a, up((size_t)W, 16), up((size_t)H, 16), (size_t)C, 16, 16, 1);
}
