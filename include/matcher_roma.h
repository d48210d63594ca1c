/* SPDX-License-Identifier: Unlicense */

/* The RoMa matcher (matcher_roma.h:20-23 of i.coregistration.opencl):
 * roma_load (+ roma_load_v2 when v2 is given) with the weights, then the
 * matcher vtable: alloc, run (roma_match, the reverse warp first with
 * m->cycle), match (in each block of spacing x spacing valid cells the
 * cell of highest certainty, kept where it reaches min_cert and lands on
 * a valid reference cell, matcher_roma.c:103-145), field (the dense
 * shift, matcher_roma.c:150-178), dump, destroy.
 *
 *   matcher_roma_create replaces matcher_roma.c:207 */

#ifndef I_COREGISTRATION_B200_MATCHER_ROMA_H
#define I_COREGISTRATION_B200_MATCHER_ROMA_H

#include "matcher.h"
#include "pth_loader.h"

#ifdef __cplusplus
extern "C" {
#endif

void matcher_roma_create(struct matcher *m, struct ops *ops,
                         struct pth_file *pf, struct pth_file *dino,
                         struct pth_file *v2, const char *name, int imagenet,
                         int spacing, float min_cert);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_MATCHER_ROMA_H */
