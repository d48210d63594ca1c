/* SPDX-License-Identifier: Unlicense */

/* The Efficient LoFTR matcher (matcher_eloftr.h:14-15 of
 * i.coregistration.opencl): detector-free semi-dense matches on grey
 * images (0.2989 R + 0.587 G + 0.114 B), to a fraction of a cell, cost
 * 1 - coarse confidence, matches outside the valid cells dropped.
 *
 *   matcher_eloftr_create replaces matcher_eloftr.c:146
 *
 * name is the matcher's name in messages; with npe, the RoPE positions are
 * scaled by ELOFTR_TRAIN_RES over the tile's long side.
 *
 * Addition without a counterpart in the reference's header: the host stage
 * on given results, which the matcher's match calls (matcher_eloftr.c:66-96). */

#ifndef I_COREGISTRATION_B200_MATCHER_ELOFTR_H
#define I_COREGISTRATION_B200_MATCHER_ELOFTR_H

#include "matcher.h"
#include "pth_loader.h"

#ifdef __cplusplus
extern "C" {
#endif

void matcher_eloftr_create(struct matcher *m, struct ops *ops, struct pth_file *pf,
                           const char *name, int npe);

/* Matches of nm keypoint pairs kp (x0, y0, x1, y1 per pair, the network's
 * convention: 3.5 px below the cells') with confidences mconf: both ends
 * moved to the cells' convention, kept where both round to cells of the
 * h x w tile that valid1 / valid2 mark (NULL: all), cost 1 - confidence.
 * Appended to out in order; returns their number. */
int eloftr_sample_matches(const float *kp, const float *mconf, int nm, int h, int w,
                          const unsigned char *valid1, const unsigned char *valid2,
                          struct match_list *out);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_MATCHER_ELOFTR_H */
