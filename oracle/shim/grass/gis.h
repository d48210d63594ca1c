/* SPDX-License-Identifier: Unlicense */

/* The few GRASS GIS library calls that the reference's tests/ops_check.c,
 * adalam.c, pth_loader.c, roma.c and matcher glue (matcher.c,
 * matcher_roma.c, matcher_eloftr.c) make, for building them without GRASS
 * (test infrastructure: oracle/Makefile). Memory calls exit on failure and
 * G_fatal_error exits 1, as in GRASS. */

#ifndef COREG_SHIM_GRASS_GIS_H
#define COREG_SHIM_GRASS_GIS_H

#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define GPATH_MAX 4096

static inline void *G__shim_check(void *p)
{
    if (!p) {
        fprintf(stderr, "ERROR: out of memory\n");
        exit(1);
    }
    return p;
}

#define G_malloc(n) G__shim_check(malloc((n) ? (n) : 1))
#define G_calloc(n, s) G__shim_check(calloc((n) ? (n) : 1, (s) ? (s) : 1))
#define G_realloc(p, n) G__shim_check(realloc((p), (n) ? (n) : 1))
#define G_free(p) free(p)

static inline void G_no_gisinit(void) {}

static inline void G_fatal_error(const char *fmt, ...)
{
    va_list ap;

    va_start(ap, fmt);
    fprintf(stderr, "ERROR: ");
    vfprintf(stderr, fmt, ap);
    fprintf(stderr, "\n");
    va_end(ap);
    exit(1);
}

static inline char *G_store(const char *s)
{
    size_t n = strlen(s) + 1;
    char *p = (char *)G__shim_check(malloc(n));

    memcpy(p, s, n);
    return p;
}

static inline void G_verbose_message(const char *fmt, ...) { (void)fmt; }

static inline void G_debug(int level, const char *fmt, ...)
{
    (void)level;
    (void)fmt;
}

static inline void G_message(const char *fmt, ...)
{
    va_list ap;

    va_start(ap, fmt);
    vfprintf(stderr, fmt, ap);
    fprintf(stderr, "\n");
    va_end(ap);
}

#endif /* COREG_SHIM_GRASS_GIS_H */
