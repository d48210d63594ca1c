/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: OpenCL C kernels compiled as C11 and run on the
 * CPU, so that the reference's own .cl sources serve as checkers here,
 * where no OpenCL platform exists (oracle/Makefile). The address-space
 * qualifiers vanish, local arrays become statics shared by one work-group,
 * a work-group of L work-items runs as L coroutines that take turns at
 * each barrier, and
 * the float built-ins the kernels use map to the C library's float
 * functions (OpenCL permits a few units in the last place for them; the
 * C library is one realization; mad is an unfused multiply-add, one of the
 * two forms OpenCL allows). Kernels with vector arithmetic (ops.cl's
 * gemm_big) compile as C++, where float4 carries that arithmetic. */

#ifndef COREG_CL_EMUL_H
#define COREG_CL_EMUL_H

#include <math.h>
#include <stddef.h>
#include <string.h>

#define __kernel
#define __global
#define __constant const
#define __local static
#define CLK_LOCAL_MEM_FENCE 1
#define CLK_GLOBAL_MEM_FENCE 2

#ifdef __cplusplus
extern "C" {
#endif

struct emul_item {
    size_t gid[3], lid[3], grp[3], lsz[3], gsz[3];
};
extern __thread struct emul_item emul_wi;

void emul_barrier(void);

/* Run body(args) as every work-item of a dims-dimensional NDRange of
 * global size g[0..2] in work-groups of l[0..2] (each g divisible by l). */
void emul_launch(void (*body)(void *), void *args, const size_t g[3], const size_t l[3]);

#ifdef __cplusplus
}
#endif

#define get_global_id(d) (emul_wi.gid[(d)])
#define get_local_id(d) (emul_wi.lid[(d)])
#define get_group_id(d) (emul_wi.grp[(d)])
#define get_local_size(d) (emul_wi.lsz[(d)])
#define get_global_size(d) (emul_wi.gsz[(d)])
#define barrier(flags) emul_barrier()

typedef unsigned char uchar;
typedef unsigned long ulong;

static inline float emul_rsqrt(float x) { return 1.0f / sqrtf(x); }
static inline int emul_clampi(int v, int lo, int hi) { return v < lo ? lo : v > hi ? hi : v; }
#define rsqrt(x) emul_rsqrt(x)
#define clamp(v, lo, hi) emul_clampi((v), (lo), (hi))

#ifndef __cplusplus

/* C: the float built-ins through _Generic, vectors as plain structs. */
typedef struct {
    int x, y, z, w;
} int4;
typedef struct {
    float x, y, z, w;
} float4;
typedef struct {
    float x, y;
} float2;

/* OpenCL's vector literal (float4)(a, b, c, d) has no C form: the build
 * recipes rewrite it to emul_float4(a, b, c, d) in their copies of the
 * source (oracle/Makefile). */
static inline float4 emul_float4(float x, float y, float z, float w)
{
    float4 v = {x, y, z, w};
    return v;
}

static inline int emul_mini(int a, int b) { return a < b ? a : b; }
static inline int emul_maxi(int a, int b) { return a > b ? a : b; }
#define min(a, b) emul_mini((a), (b))
#define max(a, b) emul_maxi((a), (b))
#define mad(a, b, c) ((a) * (b) + (c))
#define exp(x) _Generic((x), float: expf, default: exp)(x)
#define log(x) _Generic((x), float: logf, default: log)(x)
#define sqrt(x) _Generic((x), float: sqrtf, default: sqrt)(x)
#define floor(x) _Generic((x), float: floorf, default: floor)(x)
#define log1p(x) _Generic((x), float: log1pf, default: log1p)(x)
#define erf(x) _Generic((x), float: erff, default: erf)(x)
#define tanh(x) _Generic((x), float: tanhf, default: tanh)(x)
#define sin(x) _Generic((x), float: sinf, default: sin)(x)
#define cos(x) _Generic((x), float: cosf, default: cos)(x)
#define fmax(a, b) _Generic((a), float: fmaxf, default: fmax)((a), (b))

#else

/* C++: the C library's float overloads (math.h) for the built-ins, and
 * vectors with the arithmetic the kernels use (gemm_big's float4 tiles). */
struct int4 {
    int x, y, z, w;
};
struct float2 {
    float x, y;
};
struct float4 {
    float x, y, z, w;
    float4() : x(0), y(0), z(0), w(0) {}
    float4(float s) : x(s), y(s), z(s), w(s) {}
    float4(float a, float b, float c, float d) : x(a), y(b), z(c), w(d) {}
};
static inline float4 operator+(float4 a, float4 b) { return float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w); }
static inline float4 operator-(float4 a, float4 b) { return float4(a.x - b.x, a.y - b.y, a.z - b.z, a.w - b.w); }
static inline float4 operator*(float4 a, float4 b) { return float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w); }
static inline float4 &operator+=(float4 &a, float4 b) { return a = a + b; }
static inline float4 &operator-=(float4 &a, float4 b) { return a = a - b; }
static inline float4 &operator*=(float4 &a, float4 b) { return a = a * b; }
static inline float4 emul_float4(float s) { return float4(s); }
static inline float4 emul_float4(float a, float b, float c, float d) { return float4(a, b, c, d); }
static inline float mad(float a, float b, float c) { return a * b + c; }
static inline float4 mad(float4 a, float4 b, float4 c) { return a * b + c; }
static inline float4 vload4(size_t off, const float *p)
{
    p += 4 * off;
    return float4(p[0], p[1], p[2], p[3]);
}
static inline void vstore4(float4 v, size_t off, float *p)
{
    p += 4 * off;
    p[0] = v.x, p[1] = v.y, p[2] = v.z, p[3] = v.w;
}
template <class T> static inline T min(T a, T b) { return a < b ? a : b; }
template <class T> static inline T max(T a, T b) { return a > b ? a : b; }

#endif

#endif /* COREG_CL_EMUL_H */
