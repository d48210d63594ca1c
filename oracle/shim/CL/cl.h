/* SPDX-License-Identifier: Unlicense */

/* The OpenCL 1.2 scalar and handle types that the reference's headers name
 * (ocl_backend.h, ops.h, roma.h, eloftr.h), as opaque types, so that its
 * host-only sources (matcher.c, matcher_roma.c, matcher_eloftr.c) compile
 * as checkers without OpenCL (test infrastructure: oracle/Makefile). No
 * OpenCL function is declared or called. */

#ifndef COREG_SHIM_CL_H
#define COREG_SHIM_CL_H

#include <stdint.h>

typedef int32_t cl_int;
typedef uint32_t cl_uint;
typedef int64_t cl_long;
typedef uint64_t cl_ulong;
typedef struct shim_cl_platform *cl_platform_id;
typedef struct shim_cl_device *cl_device_id;
typedef struct shim_cl_context *cl_context;
typedef struct shim_cl_queue *cl_command_queue;
typedef struct shim_cl_program *cl_program;
typedef struct shim_cl_kernel *cl_kernel;
typedef struct shim_cl_mem *cl_mem;

#endif /* COREG_SHIM_CL_H */
