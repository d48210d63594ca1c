/* SPDX-License-Identifier: Unlicense */

/* The matcher interface of the B200 build: the reference's matcher.h
 * (matcher.h:1-83 of i.coregistration.opencl) unchanged in its structs,
 * members and meaning; matchers are created by matcher_roma_create
 * (matcher_roma.h) and run their device stage with this build's kernels.
 *
 *   match_add          replaces matcher.c:19
 *   matcher_dump_file  replaces matcher.c:29 */

#ifndef I_COREGISTRATION_B200_MATCHER_H
#define I_COREGISTRATION_B200_MATCHER_H

#include "ops.h"

#ifdef __cplusplus
extern "C" {
#endif

/* One match between the two images of a tile, in cells of the tile
 * (column, row; cell centres at integers). */
struct match {
    double x1, y1; /* Image to co-register. */
    double x2, y2; /* Reference. */
    float cost;    /* Lower is better (1 - confidence). */
    float sd;      /* Predicted standard deviation of the reference
                      position, in cells (NAN: none given). */
    float cycle;   /* Forward-backward cycle distance in cells (NAN: not
                      computed). */
};

struct match_list {
    int n, cap;
    struct match *v;
};

void match_add(struct match_list *l, const struct match *m);

/* One tile of both images: (3, H, W) floats in 0..1 whose content covers
 * the top-left h x w cells, the rest zero padding, and the validity of
 * those cells (h x w, 0 where a band is NULL; NULL pointer: all valid). */
struct matcher_tile {
    const float *img1, *img2;
    const unsigned char *valid1, *valid2;
    int H, W, h, w;
    int x0, y0; /* Top-left cell in the region, for diagnostics. */
    int index;  /* 1-based, for diagnostics and dumps. */
};

/* A matcher: the network on the device (run) followed by host-side
 * matching (match). */
struct matcher {
    const char *name;
    int multiple; /* Tile sides must be multiples of this. */
    struct ops *ops;
    void *state;
    const char *dump_dir;
    void (*alloc)(struct matcher *m, int H, int W);
    /* Device stage on one tile; returns once its results are on the
     * host. */
    void (*run)(struct matcher *m, const struct matcher_tile *t);
    int (*match)(struct matcher *m, const struct matcher_tile *t,
                 struct match_list *out);
    void (*dump)(struct matcher *m, const struct matcher_tile *t,
                 const char *dir);
    /* Dense matchers only: shift (dx, dy) in cells, certainty, sd per
     * cell of the h x w tile; NAN shifts and certainty 0 where none. */
    void (*field)(struct matcher *m, const struct matcher_tile *t, float *dx,
                  float *dy, float *cert, float *sd);
    int has_sd;
    /* Dense matchers: when set before alloc, run also matches the
     * reference onto the image and match fills cycle. */
    int cycle;
    void (*destroy)(struct matcher *m);
};

void matcher_dump_file(const char *dir, int tile, const char *what,
                       const void *data, size_t bytes);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_MATCHER_H */
