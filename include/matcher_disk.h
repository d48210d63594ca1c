/* SPDX-License-Identifier: Unlicense */

/* The DISK matcher (matcher_disk.h:12-22 of i.coregistration.opencl): DISK
 * keypoints and descriptors on both images of a tile (on the device),
 * nearest-neighbour matching (on the device) and AdaLAM filtering (on the
 * host, as the reference). Matches lie on whole cells; the cost is
 * AdaLAM's inverse confidence.
 *
 *   struct disk_matcher_config  the reference's matcher_disk.h:12-16
 *   matcher_disk_create         replaces matcher_disk.c:159 */

#ifndef I_COREGISTRATION_B200_MATCHER_DISK_H
#define I_COREGISTRATION_B200_MATCHER_DISK_H

#include "adalam.h"
#include "matcher.h"
#include "pth_loader.h"

#ifdef __cplusplus
extern "C" {
#endif

struct disk_matcher_config {
    int features;    /* Keypoints per image and tile. */
    float threshold; /* Heatmap score threshold. */
    struct adalam_config adalam;
};

/* Load the DISK weights from pf (closed by the caller afterwards). */
void matcher_disk_create(struct matcher *m, struct ops *ops, struct pth_file *pf,
                         const struct disk_matcher_config *cfg);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_MATCHER_DISK_H */
