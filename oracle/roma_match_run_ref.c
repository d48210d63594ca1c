/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the reference's whole RoMa tile, run on the CPU in
 * _ref/libref_cpu.so: its roma_load (+ roma_load_v2), roma_alloc and
 * roma_match (roma.c:398-544, 559-643, 1357-1435), unchanged, over its
 * ops.c and kernels (cl_backend_emul.c). With a dump folder the reference
 * writes its own debug dumps there (roma.c:1188-1227): the coarse
 * inputs, DINOv2 features, GP posterior, coarse warp, every refiner's
 * warp and certainty, the fine inputs and the results. The coarse pass
 * runs at the reference's fixed ROMA_COARSE (560): about 3.5 TFLOP
 * through the emulation, an hour on one core, so this is a fixture
 * generator (tests/golden/make_roma_ref_golden.py), not a test. */

#include <string.h>

#include "ocl_backend.h"
#include "ops.h"
#include "pth_loader.h"
#include "roma.h"

/* roma_match of the tile pair imgA, imgB (3 x H x W, [0, 1]) with the
 * weights in main_w and dino_w, plus RoMa v2's refiners from v2_w unless it
 * is NULL; the warp (2 x H x W), certainty (H x W) and, with v2, standard
 * deviation (H x W) are copied to flow, cert and sd. */
void ref_roma_match(const char *main_w, const char *dino_w, const char *v2_w, int H, int W,
                    const float *imgA, const float *imgB, const char *dump, float *flow,
                    float *cert, float *sd)
{
    static struct ocl_backend ocl;
    static struct ops o;
    static struct roma_model m;
    struct pth_file pf, pd, pv;
    size_t hw = (size_t)H * W;

    ocl_init(&ocl, "cpu", NULL);
    ops_init(&o, &ocl);
    pth_open(&pf, main_w);
    pth_open(&pd, dino_w);
    roma_load(&m, &o, &pf, &pd);
    pth_close(&pf);
    pth_close(&pd);
    if (v2_w) {
        pth_open(&pv, v2_w);
        roma_load_v2(&m, &pv);
        pth_close(&pv);
    }
    roma_alloc(&m, H, W);
    roma_match(&m, imgA, imgB, dump, 1);
    memcpy(flow, m.flow, 2 * hw * sizeof(float));
    memcpy(cert, m.cert, hw * sizeof(float));
    if (v2_w && sd)
        memcpy(sd, m.sd, hw * sizeof(float));
    roma_free(&m);
}
