// SPDX-License-Identifier: Unlicense
//
// roma_ops.h: RoMa's kernels on channel-major float32 buffers, for
// callers of the reference's kernel argument lists.

#include "gemm.cuh"
#include "roma_kernels.cuh"
#include "ops_b200.h"
#include "roma_ops.h"

using namespace coreg;

static bool bufs_ok(std::initializer_list<cl_mem> l, const char *what)
{
    if (pending())
        return false;
    for (cl_mem m : l)
        if (!m) {
            fail("%s: required buffer is NULL", what);
            return false;
        }
    return true;
}

extern "C" void roma_row_norm(struct ops *o, cl_mem X, int rows, int C,
                              cl_mem out)
{
    if (!bufs_ok({X, out}, "roma_row_norm"))
        return;
    Prof p(o->ocl, "roma_row_norm");
    roma_row_norm_l(stream_of(o->ocl), fptr(X), rows, C, fptr(out));
    launch_ok("roma_row_norm");
}

extern "C" void roma_cos_exp(struct ops *o, cl_mem S, cl_mem nx, cl_mem ny,
                             int N, int M, float T, float eps)
{
    if (!bufs_ok({S, nx, ny}, "roma_cos_exp"))
        return;
    Prof p(o->ocl, "roma_cos_exp");
    roma_cos_exp_l(stream_of(o->ocl), fptr(S), fptr(nx), fptr(ny), N, M, T, eps);
    launch_ok("roma_cos_exp");
}

extern "C" void roma_cls_to_flow(struct ops *o, cl_mem L, int ld, int C,
                                 int res, int n, cl_mem flow, cl_mem cert)
{
    if (!bufs_ok({L, flow, cert}, "roma_cls_to_flow"))
        return;
    Prof p(o->ocl, "roma_cls_to_flow");
    roma_cls_to_flow_l(stream_of(o->ocl), fptr(L), ld, C, res, n, fptr(flow),
                       fptr(cert));
    launch_ok("roma_cls_to_flow");
}

extern "C" void roma_warp_sample(struct ops *o, cl_mem in, int C, int H, int W,
                                 cl_mem flow, cl_mem out, int coff)
{
    if (!bufs_ok({in, flow, out}, "roma_warp_sample"))
        return;
    const long n = (long)H * W;
    Prof p(o->ocl, "roma_warp_sample");
    roma_warp_sample_l(stream_of(o->ocl), cm_map(fptr(in), n), C, H, W,
                       fptr(flow), cm_out(fptr(out), n), coff);
    launch_ok("roma_warp_sample");
}

extern "C" void roma_local_corr(struct ops *o, cl_mem f1, cl_mem f2, int C,
                                int H, int W, int r, cl_mem flow, cl_mem out,
                                int coff)
{
    if (!bufs_ok({f1, f2, flow, out}, "roma_local_corr"))
        return;
    const long n = (long)H * W;
    Prof p(o->ocl, "roma_local_corr");
    roma_local_corr_l(stream_of(o->ocl), cm_map(fptr(f1), n), cm_map(fptr(f2), n),
                      C, H, W, r, fptr(flow), cm_out(fptr(out), n), coff);
    launch_ok("roma_local_corr");
}

extern "C" void roma_disp(struct ops *o, cl_mem flow, int H, int W, float fx,
                          float fy, cl_mem out)
{
    if (!bufs_ok({flow, out}, "roma_disp"))
        return;
    Prof p(o->ocl, "roma_disp");
    roma_disp_l(stream_of(o->ocl), fptr(flow), H, W, fx, fy, fptr(out));
    launch_ok("roma_disp");
}

extern "C" void roma_update(struct ops *o, cl_mem flow, cl_mem cert, cl_mem d,
                            int n, float scale, float Wf, float Hf)
{
    if (!bufs_ok({flow, cert, d}, "roma_update"))
        return;
    Prof p(o->ocl, "roma_update");
    roma_update_l(stream_of(o->ocl), fptr(flow), fptr(cert), cm_map(fptr(d), n),
                  n, scale, Wf, Hf);
    launch_ok("roma_update");
}

extern "C" void roma2_update(struct ops *o, cl_mem flow, cl_mem conf, cl_mem d,
                             int n, float W, float H)
{
    if (!bufs_ok({flow, conf, d}, "roma2_update"))
        return;
    Prof p(o->ocl, "roma2_update");
    roma2_update_l(stream_of(o->ocl), fptr(flow), fptr(conf), cm_map(fptr(d), n),
                   n, W, H);
    launch_ok("roma2_update");
}

extern "C" void roma_dwconv5(struct ops *o, cl_mem in, int C, int H, int W,
                             cl_mem wt, cl_mem bias, cl_mem out)
{
    if (!bufs_ok({in, wt, bias, out}, "roma_dwconv5"))
        return;
    const long n = (long)H * W;
    Prof p(o->ocl, "roma_dwconv5");
    roma_dwconv5_l(stream_of(o->ocl), cm_map(fptr(in), n), C, H, W, fptr(wt),
                   fptr(bias), cm_out(fptr(out), n));
    launch_ok("roma_dwconv5");
}

extern "C" void roma_dwconv5_cl(struct ops *o, cl_mem in, int H, int W, int C, cl_mem wt,
                                cl_mem bias, cl_mem out)
{
    if (!bufs_ok({in, wt, bias, out}, "roma_dwconv5_cl"))
        return;
    const long n = (long)H * W;
    if (n <= 0 || C <= 0 || !count_ok(n * C, "roma_dwconv5_cl map"))
        return;
    cudaStream_t st = stream_of(o->ocl);
    Prof p(o->ocl, "roma_dwconv5");
    if (o->precision != OPS_BF16) {
        roma_dwconv5_l(st, tm_map(fptr(in), C), C, H, W, fptr(wt), fptr(bias),
                       tm_out(fptr(out), C));
        launch_ok("roma_dwconv5_cl");
        return;
    }
    // bfloat16 mode: the map rounded to bfloat16, the model's kernel, the
    // result widened back.
    const size_t half = ((size_t)n * C * 2 + 255) / 256 * 256;
    if (2 * half > o->scratch16_bytes) {
        ocl_release(&o->scratch16);
        o->scratch16 = ocl_alloc(o->ocl, 2 * half, "dwconv5 operands");
        o->scratch16_bytes = 2 * half;
        if (pending())
            return;
    }
    char *a16 = (char *)o->scratch16->ptr, *o16 = a16 + half;
    copy2d(st, fptr(in), DT_F32, C, a16, DT_BF16, C, n, C);
    roma_dwconv5_l(st, tm_map(a16, C, DT_BF16), C, H, W, fptr(wt), fptr(bias),
                   tm_out(o16, C, DT_BF16));
    copy2d(st, o16, DT_BF16, C, fptr(out), DT_F32, C, n, C);
    launch_ok("roma_dwconv5_cl");
}

extern "C" void roma_refiner_block_cl(struct ops *o, cl_mem in, int H, int W, int C,
                                      cl_mem dw_w, cl_mem dw_b, cl_mem pw_w, cl_mem pw_b,
                                      cl_mem out)
{
    if (!bufs_ok({in, dw_w, dw_b, pw_w, pw_b, out}, "roma_refiner_block_cl"))
        return;
    const long n = (long)H * W;
    if (n <= 0 || C <= 0 || !count_ok(n * C, "roma_refiner_block_cl map"))
        return;
    cudaStream_t st = stream_of(o->ocl);
    Prof p(o->ocl, "refiner_block");
    const bool bf = o->precision == OPS_BF16;
    const size_t es = bf ? 2 : 4;
    const size_t mapb = ((size_t)n * C * es + 255) / 256 * 256;
    const size_t wb = ((size_t)C * C * 2 + 255) / 256 * 256;
    const size_t need = bf ? 3 * mapb + wb : mapb;
    if (need > o->scratch16_bytes) {
        ocl_release(&o->scratch16);
        o->scratch16 = ocl_alloc(o->ocl, need, "refiner block operands");
        o->scratch16_bytes = need;
        if (pending())
            return;
    }
    char *mid = (char *)o->scratch16->ptr;
    GemmArgs g = gemm_args((int)n, C, C);
    g.lda = C;
    g.ldb = C;
    g.transb = 1;
    g.ldc = C;
    g.bias = fptr(pw_b);
    if (!bf) {
        // float32: the depthwise kernel, then the float32 product.
        roma_dwconv5_l(st, tm_map(fptr(in), C), C, H, W, fptr(dw_w), fptr(dw_b),
                       tm_out(mid, C));
        g.A = mid;
        g.B = fptr(pw_w);
        g.C = fptr(out);
        gemm_run(o->ocl, g, "refiner_pw");
        launch_ok("roma_refiner_block_cl");
        return;
    }
    // bfloat16: the map and the weights rounded to bfloat16, the fused
    // kernel (or, for other widths, the model's two kernels), the result
    // widened back.
    char *a16 = mid + mapb, *o16 = a16 + mapb, *w16 = o16 + mapb;
    copy2d(st, fptr(in), DT_F32, C, a16, DT_BF16, C, n, C);
    copy2d(st, fptr(pw_w), DT_F32, C, w16, DT_BF16, C, C, C);
    if (!dwpw_tc(st, a16, H, W, C, fptr(dw_w), fptr(dw_b), w16, fptr(pw_b), o16,
                 o->ocl->sm_count)) {
        roma_dwconv5_l(st, tm_map(a16, C, DT_BF16), C, H, W, fptr(dw_w), fptr(dw_b),
                       tm_out(mid, C, DT_BF16));
        g.A = mid;
        g.B = w16;
        g.C = o16;
        g.ab = DT_BF16;
        g.c = DT_BF16;
        gemm_run(o->ocl, g, "refiner_pw");
    }
    copy2d(st, o16, DT_BF16, C, fptr(out), DT_F32, C, n, C);
    launch_ok("roma_refiner_block_cl");
}

extern "C" void roma_local_corr_cl(struct ops *o, cl_mem f1, cl_mem f2, int C, int H, int W,
                                   int r, cl_mem flow, cl_mem out)
{
    if (!bufs_ok({f1, f2, flow, out}, "roma_local_corr_cl"))
        return;
    const long n = (long)H * W;
    if (n <= 0 || C <= 0 || !count_ok(n * C, "roma_local_corr_cl map"))
        return;
    const int side = 2 * r + 1;
    cudaStream_t st = stream_of(o->ocl);
    Prof p(o->ocl, "roma_local_corr");
    if (o->precision != OPS_BF16) {
        roma_local_corr_l(st, tm_map(fptr(f1), C), tm_map(fptr(f2), C), C, H, W, r, fptr(flow),
                          tm_out(fptr(out), side * side), 0);
        launch_ok("roma_local_corr_cl");
        return;
    }
    const size_t half = ((size_t)n * C * 2 + 255) / 256 * 256;
    if (2 * half > o->scratch16_bytes) {
        ocl_release(&o->scratch16);
        o->scratch16 = ocl_alloc(o->ocl, 2 * half, "local_corr operands");
        o->scratch16_bytes = 2 * half;
        if (pending())
            return;
    }
    char *a16 = (char *)o->scratch16->ptr, *b16 = a16 + half;
    copy2d(st, fptr(f1), DT_F32, C, a16, DT_BF16, C, n, C);
    copy2d(st, fptr(f2), DT_F32, C, b16, DT_BF16, C, n, C);
    roma_local_corr_l(st, tm_map(a16, C, DT_BF16), tm_map(b16, C, DT_BF16), C, H, W, r,
                      fptr(flow), tm_out(fptr(out), side * side), 0);
    launch_ok("roma_local_corr_cl");
}

extern "C" int roma_gp_solve(struct ops *o, cl_mem K, int n, cl_mem F, int d, double noise,
                             cl_mem X)
{
    if (!bufs_ok({K, F, X}, "roma_gp_solve"))
        return -1;
    if (n < 1 || d < 1) {
        fail("roma_gp_solve: %d x %d", n, d);
        return -1;
    }
    cl_mem work = ocl_alloc(o->ocl, gp_work_doubles(n, d) * sizeof(double), "GP work");
    cl_mem flag = ocl_alloc(o->ocl, sizeof(int), "GP flag");
    int f = 0;
    if (!pending()) {
        cudaStream_t st = stream_of(o->ocl);
        cudaMemsetAsync(flag->ptr, 0, sizeof(int), st);
        Prof p(o->ocl, "roma_gp_solve");
        gp_solve_dev(st, fptr(K), n, fptr(F), d, noise, fptr(X), (double *)work->ptr,
                     (int *)flag->ptr);
        if (launch_ok("roma_gp_solve"))
            ocl_read(o->ocl, flag, 0, &f, sizeof(int));
    }
    ocl_release(&work);
    ocl_release(&flag);
    return pending() ? -1 : f;
}
