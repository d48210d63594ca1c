/* SPDX-License-Identifier: Unlicense */

/* The Efficient LoFTR matcher (matcher_eloftr.h:14-15 of
 * i.coregistration.opencl): detector-free semi-dense matches on grey
 * images (0.2989 R + 0.587 G + 0.114 B), to a fraction of a cell, cost
 * 1 - coarse confidence, matches outside the valid cells dropped.
 *
 *   matcher_eloftr_create replaces matcher_eloftr.c:146
 *
 * name is the matcher's name in messages; with npe, the RoPE positions are
 * scaled by ELOFTR_TRAIN_RES over the tile's long side. */

#ifndef I_COREGISTRATION_B200_MATCHER_ELOFTR_H
#define I_COREGISTRATION_B200_MATCHER_ELOFTR_H

#include "matcher.h"
#include "pth_loader.h"

#ifdef __cplusplus
extern "C" {
#endif

void matcher_eloftr_create(struct matcher *m, struct ops *ops, struct pth_file *pf,
                           const char *name, int npe);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_MATCHER_ELOFTR_H */
