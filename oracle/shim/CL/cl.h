/* SPDX-License-Identifier: Unlicense */

/* The OpenCL 1.2 scalar and handle types that the reference's headers name
 * (ocl_backend.h, ops.h, roma.h, eloftr.h), as opaque types, and the
 * prototypes (from the OpenCL 1.2 specification) of the OpenCL calls
 * that its host sources make, so that they compile without OpenCL (test
 * infrastructure: oracle/Makefile). oracle/cl_backend_emul.c defines
 * these calls over host memory, for the builds that run the reference's
 * kernels on the CPU. */

#ifndef COREG_SHIM_CL_H
#define COREG_SHIM_CL_H

#include <stdint.h>

typedef int32_t cl_int;
typedef uint32_t cl_uint;
typedef int64_t cl_long;
typedef uint64_t cl_ulong;
typedef float cl_float;
typedef struct shim_cl_platform *cl_platform_id;
typedef struct shim_cl_device *cl_device_id;
typedef struct shim_cl_context *cl_context;
typedef struct shim_cl_queue *cl_command_queue;
typedef struct shim_cl_program *cl_program;
typedef struct shim_cl_kernel *cl_kernel;
typedef struct shim_cl_mem *cl_mem;
typedef struct shim_cl_event *cl_event;

#include <stddef.h>

typedef cl_uint cl_profiling_info;
#define CL_SUCCESS 0
#define CL_PROFILING_COMMAND_START 0x1282
#define CL_PROFILING_COMMAND_END 0x1283

cl_int clSetKernelArg(cl_kernel kernel, cl_uint index, size_t size, const void *value);
cl_int clEnqueueNDRangeKernel(cl_command_queue queue, cl_kernel kernel, cl_uint dims,
                              const size_t *offset, const size_t *global, const size_t *local,
                              cl_uint n_wait, const cl_event *wait, cl_event *event);
cl_int clWaitForEvents(cl_uint n, const cl_event *events);
cl_int clGetEventProfilingInfo(cl_event event, cl_profiling_info name, size_t size,
                               void *value, size_t *size_ret);
cl_int clReleaseEvent(cl_event event);
cl_int clFinish(cl_command_queue queue);
cl_int clReleaseKernel(cl_kernel kernel);
cl_int clEnqueueCopyBuffer(cl_command_queue queue, cl_mem src, cl_mem dst, size_t src_offset,
                           size_t dst_offset, size_t size, cl_uint n_wait,
                           const cl_event *wait, cl_event *event);
cl_int clEnqueueCopyBufferRect(cl_command_queue queue, cl_mem src, cl_mem dst,
                               const size_t *src_origin, const size_t *dst_origin,
                               const size_t *region, size_t src_row_pitch,
                               size_t src_slice_pitch, size_t dst_row_pitch,
                               size_t dst_slice_pitch, cl_uint n_wait, const cl_event *wait,
                               cl_event *event);
cl_int clEnqueueFillBuffer(cl_command_queue queue, cl_mem buffer, const void *pattern,
                           size_t pattern_size, size_t offset, size_t size, cl_uint n_wait,
                           const cl_event *wait, cl_event *event);

#endif /* COREG_SHIM_CL_H */
