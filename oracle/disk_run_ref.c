/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the reference's whole DISK device stage, run on the
 * CPU in _ref/libref_cpu.so: its pth_open (here on a safetensors file),
 * disk_load, disk_alloc and disk_detect over its ops.c and kernels
 * (cl_backend_emul.c). One call loads, detects and frees. */

#include <stdlib.h>
#include <string.h>

#include "cl_backend_emul.h"
#include "disk.h"
#include "ocl_backend.h"
#include "ops.h"
#include "pth_loader.h"

/* Keypoints of img (3, H, W) with the DISK weights in the file weights:
 * returns their number, writes xy, score, desc (n x DISK_DESC) as
 * disk_detect, and the network output ((DISK_DESC + 1) x H x W) into net. */
int ref_disk_run(const char *weights, const float *img, int H, int W, int h, int w, int n,
                 float thresh, const unsigned char *valid, int *xy, float *score, float *desc,
                 float *net)
{
    struct ocl_backend ocl;
    struct ops o;
    struct disk_model m;
    struct pth_file pf;
    int k;

    ocl_init(&ocl, "cpu", NULL);
    ops_init(&o, &ocl);
    pth_open(&pf, weights);
    memset(&m, 0, sizeof(m));
    disk_load(&m, &o, &pf);
    pth_close(&pf);
    disk_alloc(&m, H, W, n);
    k = disk_detect(&m, img, H, W, h, w, n, thresh, valid, xy, score, desc);
    memcpy(net, m.out->host, (size_t)(DISK_DESC + 1) * H * W * sizeof(float));
    disk_free(&m);
    ops_free(&o);
    ocl_free(&ocl);
    return k;
}
