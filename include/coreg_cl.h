/* SPDX-License-Identifier: Unlicense */

/* Scalar and handle types of the OpenCL 1.2 API that the reference's
 * ops.h / ocl_backend.h / matcher.h signatures use (cl_int, cl_long,
 * cl_mem ...), defined here without OpenCL: on this CUDA build a cl_mem
 * is an opaque handle to a device allocation of the current CUDA device
 * (see ocl_ptr / ocl_wrap in ocl_backend.h), so that callers written
 * against the reference's headers compile unchanged. */

#ifndef COREG_CL_H
#define COREG_CL_H

#include <stddef.h>
#include <stdint.h>

typedef int32_t cl_int;
typedef uint32_t cl_uint;
typedef int64_t cl_long;
typedef uint64_t cl_ulong;
typedef float cl_float;

/* A device buffer: pointer, size in bytes, owner flag. */
typedef struct _cl_mem *cl_mem;

/* The backend's in-order queue: a cudaStream_t. */
typedef void *cl_command_queue;

#define CL_SUCCESS 0

#ifdef __cplusplus
extern "C" {
#endif

/* Waits until every launch on the queue has finished; CL_SUCCESS, or the
 * CUDA error code. The reference's callers finish their queue with it
 * (tests/ops_check.c:489 of i.coregistration.opencl). */
cl_int clFinish(cl_command_queue queue);

#ifdef __cplusplus
}
#endif

#endif /* COREG_CL_H */
