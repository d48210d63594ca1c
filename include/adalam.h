/* SPDX-License-Identifier: Unlicense */

/* Nearest-neighbour descriptor matching and AdaLAM outlier filtering (the
 * reference's adalam.h, i.coregistration.opencl adalam.h:11-35; AdaLAM is
 * Cavalli et al. 2020, as kornia.feature.match_adalam runs it, without the
 * orientation and scale tests since DISK keypoints carry neither).
 *
 *   struct adalam_config  the reference's adalam.h:11-19
 *   adalam_defaults       replaces adalam.c:23
 *   adalam_match          replaces adalam.c:300, with the ops handle of the
 *                         device first: the nearest neighbours (which the
 *                         reference computes on the host, adalam.c:38-98)
 *                         and the RANSAC passes of the filter run there
 *   adalam_filter         the filtering alone (adalam.c:320-600), given the
 *                         nearest neighbours, on the device of o, or on
 *                         host threads when o is NULL; no counterpart in the
 *                         reference's header
 *
 * Results are those of the reference: the same matches in the same order
 * with the same confidences, bit for bit, for the same nearest
 * neighbours and scores. */

#ifndef I_COREGISTRATION_B200_ADALAM_H
#define I_COREGISTRATION_B200_ADALAM_H

#include "ops.h"

#ifdef __cplusplus
extern "C" {
#endif

struct adalam_config {
    double area_ratio;       /* Image area over seed circle area. */
    double search_expansion; /* Neighbourhood radius over seed radius. */
    int ransac_iters;        /* Hypotheses per neighbourhood. */
    int min_inliers;         /* Inliers a neighbourhood must keep. */
    double min_confidence;   /* Confidence-based RANSAC threshold. */
    double det_thr;          /* Largest scale change of an affinity. */
    int force_seed_mnn;      /* Seeds only among mutual nearest neighbours. */
};

/* kornia's defaults with the reference's overrides (search expansion 16,
 * 256 hypotheses, seeds not restricted to mutual nearest neighbours). */
void adalam_defaults(struct adalam_config *c);

/* Match the n1 descriptors d1 of keypoints k1 (x, y pairs) to the n2 of k2
 * (dim floats each, L2-normalized; host arrays): nearest neighbour by
 * squared distance on the device of o, with Lowe's ratio of the two
 * nearest as score, then AdaLAM. Writes the accepted matches as index
 * pairs (i1, i2) sorted by i1 then i2 into *pairs and their inverse
 * confidence into *dist (both malloc'd, free() them; NULL when n1 or n2
 * is below 2); returns their number. */
int adalam_match(struct ops *o, const float *k1, const float *d1, int n1, const float *k2,
                 const float *d2, int n2, int dim, const struct adalam_config *cfg, int **pairs,
                 float **dist);

/* AdaLAM on given nearest neighbours: nn12 (the nearest k2 of each k1),
 * score (its ratio) and, when cfg->force_seed_mnn is set, nn21 (the
 * nearest k1 of each k2; may be NULL otherwise). The RANSAC passes run on
 * the device of o, or on host threads when o is NULL; the results are the
 * same. A neighbourhood may hold at most 16384 matches on the device.
 * Output as adalam_match. */
int adalam_filter(struct ops *o, const float *k1, int n1, const float *k2, int n2,
                  const int *nn12, const float *score, const int *nn21,
                  const struct adalam_config *cfg, int **pairs, float **dist);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_ADALAM_H */
