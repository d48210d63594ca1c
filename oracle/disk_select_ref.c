/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the reference's disk.c, compiled where it lies (the
 * Makefile names it by path in REF_DISK_C), run through disk_detect with
 * its device stage replaced by stand-ins, so that its host-side keypoint
 * selection (disk.c:210-253: the NMS candidates of the h x w crop, those
 * above the (n + 1)-th highest score, in raster order) works on a given
 * NMS mask and heatmap. The network and gather calls do nothing here; the
 * two blocking reads after the NMS return the given mask and heatmap, the
 * descriptor read returns zeros. Built into _ref/libdisk_select_ref.so by
 * oracle/Makefile. */

#include REF_DISK_C

#include <stdlib.h>
#include <string.h>

static const unsigned char *given_mask;
static const float *given_heat;
static int reads;

void ocl_check(cl_int err, const char *what) { (void)err, (void)what; }
void ocl_write(struct ocl_backend *ocl, cl_mem dst, size_t off, const void *src, size_t n)
{
    (void)ocl, (void)dst, (void)off, (void)src, (void)n;
}
void ocl_read(struct ocl_backend *ocl, cl_mem src, size_t off, void *dst, size_t n)
{
    (void)ocl, (void)src, (void)off;
    if (reads == 0)
        memcpy(dst, given_mask, n);
    else if (reads == 1)
        memcpy(dst, given_heat, n);
    else
        memset(dst, 0, n);
    reads++;
}
void ops_run(struct ocl_backend *ocl, cl_kernel k, int dims, const size_t *g, const size_t *l,
             const char *what)
{
    (void)ocl, (void)k, (void)dims, (void)g, (void)l, (void)what;
}
struct conv_geom ops_geom(int k, int s, int p)
{
    struct conv_geom g;

    memset(&g, 0, sizeof(g));
    (void)k, (void)s, (void)p;
    return g;
}
void ops_conv2d(struct ops *o, cl_mem in, int C, int H, int W, cl_mem w, cl_mem b, int K,
                const struct conv_geom *g, cl_mem mean, cl_mem rstd, cl_mem alpha, int act,
                float slope, cl_mem out)
{
    (void)o, (void)in, (void)C, (void)H, (void)W, (void)w, (void)b, (void)K, (void)g;
    (void)mean, (void)rstd, (void)alpha, (void)act, (void)slope, (void)out;
}
void ops_chan_stats(struct ops *o, cl_mem x, int C, int HW, float eps, cl_mem mean, cl_mem rstd)
{
    (void)o, (void)x, (void)C, (void)HW, (void)eps, (void)mean, (void)rstd;
}
void ops_avgpool2(struct ops *o, cl_mem in, int C, int H, int W, cl_mem out)
{
    (void)o, (void)in, (void)C, (void)H, (void)W, (void)out;
}
void ops_resize(struct ops *o, cl_mem in, int C, int h, int w, cl_mem out, int H, int W,
                int coff, int align_corners, float scale)
{
    (void)o, (void)in, (void)C, (void)h, (void)w, (void)out, (void)H, (void)W, (void)coff;
    (void)align_corners, (void)scale;
}
cl_int clSetKernelArg(cl_kernel k, cl_uint i, size_t n, const void *v)
{
    (void)k, (void)i, (void)n, (void)v;
    return 0;
}
cl_int clEnqueueCopyBuffer(cl_command_queue q, cl_mem s, cl_mem d, size_t so, size_t dof,
                           size_t n, cl_uint nw, const cl_event *w, cl_event *e)
{
    (void)q, (void)s, (void)d, (void)so, (void)dof, (void)n, (void)nw, (void)w, (void)e;
    return 0;
}

#pragma weak clReleaseKernel
#pragma weak ocl_alloc
#pragma weak ocl_kernel
#pragma weak ocl_release
#pragma weak ocl_upload
#pragma weak pth_require
#pragma weak pth_read_f32
#pragma weak pth_numel
#pragma weak pth_bytes
#pragma weak progress_begin
#pragma weak progress_end

/* Keypoints of the given NMS mask (h x w bytes) and heatmap (h rows of
 * pitch W) at most n of them, skipping cells where valid (may be NULL) is
 * 0: xy (x, y pairs) and score; returns their number. */
int ref_disk_select(const unsigned char *mask, const float *heat, int H, int W, int h, int w,
                    int n, const unsigned char *valid, int *xy, float *score)
{
    struct ocl_backend ocl;
    struct disk_model m;
    float *img = calloc((size_t)3 * H * W, sizeof(float));
    float *desc = calloc((size_t)(n > 0 ? n : 1) * DISK_DESC, sizeof(float));
    int k;

    memset(&ocl, 0, sizeof(ocl));
    memset(&m, 0, sizeof(m));
    m.ocl = &ocl;
    m.H = H;
    m.W = W;
    m.nmax = n;
    m.heat = malloc((size_t)H * W * sizeof(float));
    m.maskh = malloc((size_t)H * W);
    given_mask = mask;
    given_heat = heat;
    reads = 0;
    k = disk_detect(&m, img, H, W, h, w, n, 0.0f, valid, xy, score, desc);
    free(m.heat);
    free(m.maskh);
    free(img);
    free(desc);
    return k;
}
