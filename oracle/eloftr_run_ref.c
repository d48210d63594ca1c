/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the reference's whole Efficient LoFTR device stage,
 * run on the CPU in _ref/libref_cpu.so: its pth_open (here on a safetensors
 * file), eloftr_load, eloftr_alloc and eloftr_match over its ops.c and
 * kernels (cl_backend_emul.c). One call loads, matches and frees; with a
 * dump folder it also writes the reference's own debug dumps of the
 * backbone, transformer and fusion features (eloftr.c:638-681). */

#include <stdlib.h>
#include <string.h>

#include "cl_backend_emul.h"
#include "eloftr.h"
#include "ocl_backend.h"
#include "ops.h"
#include "pth_loader.h"

/* The coarse matches of the grey pair g0, g1 (H x W each) with the weights
 * in the file weights and RoPE position scale pos_scale: returns their
 * number (at most cap) and writes mi, mj, mconf and kp (4 per match).
 * dump (may be NULL) names the folder for tile001_eloftr_*.f32. */
int ref_eloftr_run(const char *weights, const float *g0, const float *g1, int H, int W,
                   float pos_scale, int cap, int *mi, int *mj, float *mconf, float *kp,
                   const char *dump)
{
    struct ocl_backend ocl;
    struct ops o;
    struct eloftr_model m;
    struct pth_file pf;
    int n, total;

    ocl_init(&ocl, "cpu", NULL);
    ops_init(&o, &ocl);
    pth_open(&pf, weights);
    memset(&m, 0, sizeof(m));
    eloftr_load(&m, &o, &pf);
    pth_close(&pf);
    m.pos_scale = pos_scale;
    eloftr_alloc(&m, H, W);
    eloftr_match(&m, g0, g1, dump, 1);
    total = m.nm;
    n = total < cap ? total : cap;
    memcpy(mi, m.mi, n * sizeof(int));
    memcpy(mj, m.mj, n * sizeof(int));
    memcpy(mconf, m.mconf, n * sizeof(float));
    memcpy(kp, m.kp, 4 * n * sizeof(float));
    eloftr_free(&m);
    ops_free(&o);
    ocl_free(&ocl);
    return total;
}
