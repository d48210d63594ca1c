/* SPDX-License-Identifier: Unlicense */

/* The RoMa matcher (matcher_roma.h:20-23 of i.coregistration.opencl):
 * roma_load (+ roma_load_v2 when v2 is given) with the weights, then the
 * matcher vtable: alloc, run (roma_match, the reverse warp first with
 * m->cycle), match (in each block of spacing x spacing valid cells the
 * cell of highest certainty, kept where it reaches min_cert and lands on
 * a valid reference cell, matcher_roma.c:103-145), field (the dense
 * shift, matcher_roma.c:150-178), dump, destroy.
 *
 *   matcher_roma_create replaces matcher_roma.c:207
 *
 * Additions without a counterpart in the reference's header: the host
 * stage on given results (roma_m_match matcher_roma.c:103-145,
 * roma_m_field :150-178), and the same on the device, which the matcher's
 * match and field call. */

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

/* Matches from a warp flow (2, H, W), certainty cert (H, W) and sd (H, W,
 * may be NULL) over the top-left h x w cells: in each spacing x spacing
 * block the first valid1 cell of highest certainty, kept where it reaches
 * min_cert and lands on a valid2 cell (valid1 / valid2: h x w, NULL for
 * all valid); with the reverse warp bflow (2, H, W; may be NULL) each
 * match carries its cycle distance. Appended to out in block raster
 * order; returns their number. */
int roma_sample_matches(const float *flow, const float *cert, const float *sd,
                        const float *bflow, int H, int W, int h, int w,
                        int spacing, float min_cert, const unsigned char *valid1,
                        const unsigned char *valid2, struct match_list *out);

/* The dense shift of the top-left h x w cells (dx, dy in cells, certo, sdo:
 * h x w each, sdo may be NULL): NAN shifts and certainty 0 where the cell
 * is not valid1 or lands outside valid2. */
void roma_dense_field(const float *flow, const float *cert, const float *sd,
                      int H, int W, int h, int w, const unsigned char *valid1,
                      const unsigned char *valid2, float *dx, float *dy,
                      float *certo, float *sdo);

/* The same two stages on the device (no reference counterpart), from
 * device-resident results (flow, cert, sd, bflow: device pointers such as
 * roma_results_dev gives; sd and bflow may be NULL) on o's stream; valid1
 * and valid2 are host masks (or NULL) and the outputs host memory, as
 * above. The same matches and fields as roma_sample_matches and
 * roma_dense_field, bit for bit; synchronous. The RoMa matcher's match
 * and field use these. */
int roma_sample_matches_dev(struct ops *o, const float *flow, const float *cert,
                            const float *sd, const float *bflow, int H, int W, int h, int w,
                            int spacing, float min_cert, const unsigned char *valid1,
                            const unsigned char *valid2, struct match_list *out);
void roma_dense_field_dev(struct ops *o, const float *flow, const float *cert,
                          const float *sd, int H, int W, int h, int w,
                          const unsigned char *valid1, const unsigned char *valid2,
                          float *dx, float *dy, float *certo, float *sdo);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_MATCHER_ROMA_H */
