/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the reference's DISK kernels (disk_kernels.cl:
 * nms5x5, gather_desc), compiled where they lie as C through cl_emul.h
 * (the Makefile names the file in REF_DISK_KERNELS_CL) and run on the CPU.
 * Built into _ref/libdisk_cl_ref.so by oracle/Makefile. */

#include "cl_emul.h"

#include REF_DISK_KERNELS_CL

struct a_nms { const float *heat; ulong off; int W, h, w; float thresh; uchar *mask; };
static void b_nms(void *p)
{
    struct a_nms *a = p;
    nms5x5(a->heat, a->off, a->W, a->h, a->w, a->thresh, a->mask);
}
/* The NMS mask (h x w bytes) of the heatmap plane at element off of
 * heat_all, row pitch W. */
void ref_nms5x5(const float *heat_all, unsigned long off, int W, int h, int w, float thresh,
                unsigned char *mask)
{
    struct a_nms a = {heat_all, off, W, h, w, thresh, mask};
    const size_t g[3] = {(size_t)w, (size_t)h, 1}, l[3] = {1, 1, 1};
    emul_launch(b_nms, &a, g, l);
}

struct a_gather { const float *feat; int H, W, D; const int *xy; int n; float *desc; };
static void b_gather(void *p)
{
    struct a_gather *a = p;
    gather_desc(a->feat, a->H, a->W, a->D, a->xy, a->n, a->desc);
}
void ref_gather_desc(const float *feat, int H, int W, int D, const int *xy, int n, float *desc)
{
    struct a_gather a = {feat, H, W, D, xy, n, desc};
    const size_t g[3] = {(size_t)n, 1, 1}, l[3] = {1, 1, 1};
    emul_launch(b_gather, &a, g, l);
}
