/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the second pass of the reference's RoMa v2 stage,
 * run on the CPU in _ref/libref_cpu.so: its roma_load_v2, roma_alloc, vgg2
 * and refiners2 (roma.c:1000-1306, reached by including roma.c, where they
 * are static) over its ops.c and kernels (cl_backend_emul.c). This is the
 * wiring of RoMa v2's refiners: feature pyramid, resampling of the warp
 * and confidence between scales, precision reset, and each refiner's
 * concatenation, correlation, depthwise-pointwise stack and update. */

#include REF_ROMA_C

/* RoMa v2's refiners of the pass at H x W (roma.c:1272-1306 with
 * zero_prec set, as roma.c:1327 runs them) on the images imgA, imgB (3 x H
 * x W, [0, 1]) with the v2 weights in the file weights, from the warp
 * flow_in (2 x h x w) and confidence conf_in (4 x h x w): writes the warp
 * (2 x H x W) and confidence (4 x H x W) of the finest refiner. The model's
 * buffers are left to the process (a checker called a few times). */
void ref_roma_v2_refiners(const char *weights, const float *imgA, const float *imgB, int H,
                          int W, int h, int w, const float *flow_in, const float *conf_in,
                          float *flow_out, float *conf_out)
{
    static struct ocl_backend ocl;
    static struct ops o;
    static struct roma_model m;
    struct pth_file pf;
    size_t hw = (size_t)H * W;
    int k, cur = 0;

    ocl_init(&ocl, "cpu", NULL);
    ops_init(&o, &ocl);
    memset(&m, 0, sizeof(m));
    m.ops = &o;
    m.ocl = &ocl;
    m.imagenet = 1;
    m.k_warp = ocl_kernel(&ocl, "roma_warp_sample");
    m.k_corr = ocl_kernel(&ocl, "roma_local_corr");
    m.k_disp = ocl_kernel(&ocl, "roma_disp");
    m.k_dw = ocl_kernel(&ocl, "roma_dwconv5");
    m.k_update2 = ocl_kernel(&ocl, "roma2_update");
    pth_open(&pf, weights);
    roma_load_v2(&m, &pf);
    pth_close(&pf);
    /* roma_alloc uploads RoMa's GP basis, which roma_load computes; the
     * refiners never read it. */
    m.gp_basis = calloc((size_t)N16 * GP_DIM, sizeof(float));
    roma_alloc(&m, H, W);
    for (k = 0; k < 2; k++) {
        prepare(k ? imgB : imgA, H, W, m.in_f[k], H, W, m.imagenet);
        ocl_write(m.ocl, m.img, 0, m.in_f[k], 3 * hw * sizeof(float));
        vgg2(&m, H, W, k);
    }
    ocl_write(m.ocl, m.fl[0], 0, flow_in, 2 * (size_t)h * w * sizeof(float));
    ocl_write(m.ocl, m.cf[0], 0, conf_in, 4 * (size_t)h * w * sizeof(float));
    refiners2(&m, 1, H, W, &h, &w, &cur, 1, NULL, 0);
    ocl_read(m.ocl, m.fl[cur], 0, flow_out, 2 * hw * sizeof(float));
    ocl_read(m.ocl, m.cf[cur], 0, conf_out, 4 * hw * sizeof(float));
}
