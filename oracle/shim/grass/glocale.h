/* SPDX-License-Identifier: Unlicense */

/* GRASS's translation macro, as the identity (test infrastructure). */

#ifndef COREG_SHIM_GRASS_GLOCALE_H
#define COREG_SHIM_GRASS_GLOCALE_H

#define _(s) (s)

#endif /* COREG_SHIM_GRASS_GLOCALE_H */
