/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: OpenCL C kernels compiled as C11 and run on the
 * CPU, so that the reference's own .cl sources serve as checkers here,
 * where no OpenCL platform exists (oracle/Makefile). The address-space
 * qualifiers vanish, local arrays become statics shared by one work-group,
 * a work-group of L work-items runs as L host threads with a barrier, and
 * the float built-ins the kernels use map to the C library's float
 * functions (OpenCL permits a few units in the last place for them; the
 * C library is one realization; mad is an unfused multiply-add, one of the
 * two forms OpenCL allows). */

#ifndef COREG_CL_EMUL_H
#define COREG_CL_EMUL_H

#include <math.h>
#include <stddef.h>

#define __kernel
#define __global
#define __constant const
#define __local static
#define CLK_LOCAL_MEM_FENCE 1
#define CLK_GLOBAL_MEM_FENCE 2

struct emul_item {
    size_t gid[3], lid[3], grp[3];
};
extern __thread struct emul_item emul_wi;

#define get_global_id(d) (emul_wi.gid[(d)])
#define get_local_id(d) (emul_wi.lid[(d)])
#define get_group_id(d) (emul_wi.grp[(d)])

void emul_barrier(void);
#define barrier(flags) emul_barrier()

static inline float emul_rsqrt(float x) { return 1.0f / sqrtf(x); }
static inline int emul_clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }

typedef unsigned char uchar;
typedef unsigned long ulong;
typedef struct {
    int x, y, z, w;
} int4;
typedef struct {
    float x, y, z, w;
} float4;

/* OpenCL's vector literal (float4)(a, b, c, d) has no C form: the build
 * recipe rewrites it to emul_float4(a, b, c, d) in its copy of the source
 * (oracle/Makefile). */
static inline float4 emul_float4(float x, float y, float z, float w)
{
    float4 v = {x, y, z, w};
    return v;
}

#define mad(a, b, c) ((a) * (b) + (c))
#define log(x) _Generic((x), float: logf, default: log)(x)
#define rsqrt(x) emul_rsqrt(x)
#define clamp(v, lo, hi) emul_clampi((v), (lo), (hi))
#define exp(x) _Generic((x), float: expf, default: exp)(x)
#define sqrt(x) _Generic((x), float: sqrtf, default: sqrt)(x)
#define floor(x) _Generic((x), float: floorf, default: floor)(x)
#define log1p(x) _Generic((x), float: log1pf, default: log1p)(x)
#define fmax(a, b) _Generic((a), float: fmaxf, default: fmax)((a), (b))

/* Run body(args) as every work-item of a dims-dimensional NDRange of
 * global size g[0..2] in work-groups of l[0..2] (each g divisible by l). */
void emul_launch(void (*body)(void *), void *args, const size_t g[3], const size_t l[3]);

#endif /* COREG_CL_EMUL_H */
