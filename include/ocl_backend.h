/* SPDX-License-Identifier: Unlicense */

/* Device runtime of the B200 build: the roles of the reference's
 * ocl_backend.h (ocl_backend.h:36-61 of i.coregistration.opencl) on one
 * CUDA device with one stream per backend instead of one OpenCL context
 * and in-order queue.
 *
 * Same entry points and argument meaning as the reference:
 *   ocl_init   replaces ocl_backend.c:210  (device pick)
 *   ocl_alloc  replaces ocl_backend.c:275  (fatal on failure)
 *   ocl_upload replaces ocl_backend.c:295
 *   ocl_write  replaces ocl_backend.c:304  (blocking)
 *   ocl_read   replaces ocl_backend.c:312  (blocking)
 *   ocl_release replaces ocl_backend.c:331
 * ocl_kernel (program kernels by name) has no counterpart: there is no
 * runtime-compiled program; model kernels are C functions (roma_ops.h).
 *
 * Errors: fatal by default, as the reference's G_fatal_error (message on
 * stderr, exit status 1). coreg_set_error_mode(COREG_ERRORS_RECORD) makes
 * them recorded instead (coreg_last_error); while an error is recorded,
 * every entry point returns at once without work. */

#ifndef I_COREGISTRATION_B200_OCL_BACKEND_H
#define I_COREGISTRATION_B200_OCL_BACKEND_H

#include "coreg_cl.h"

#ifdef __cplusplus
extern "C" {
#endif

struct ocl_backend {
    int device;      /* CUDA device ordinal. */
    cl_command_queue queue; /* cudaStream_t of every launch of this backend. */
    char device_name[256];
    char platform_name[256]; /* "CUDA <runtime version>". */
    cl_ulong max_alloc;
    cl_ulong global_mem;
    int is_gpu;      /* Always 1. */
    int profile;     /* Per-kernel timing (I_COREGISTRATION_OPENCL_PROFILE). */
    int sm_count;
    int cc_major, cc_minor;
    void *pinned;    /* Pinned staging buffer of ocl_write / ocl_read. */
    size_t pinned_bytes;
};

/* Select a device. device_opt: "auto" or "gpu" (CUDA device 0, or the
 * current device of the thread if one was set), or a decimal CUDA device
 * index ("0".."7"); platform_opt is accepted and ignored. Fatal if no
 * CUDA device matches (there is no CPU fallback) or if the device is not
 * compute capability 10.0 (the kernels are built for sm_100a only). */
void ocl_init(struct ocl_backend *ocl, const char *device_opt,
              const char *platform_opt);

void ocl_free(struct ocl_backend *ocl);

/* Name of a CUDA runtime error code. */
const char *ocl_errstr(cl_int err);

/* Fatal (or recorded) error if err is not 0 (a cudaError_t). */
void ocl_check(cl_int err, const char *what);

cl_mem ocl_alloc(struct ocl_backend *ocl, size_t n, const char *what);
cl_mem ocl_upload(struct ocl_backend *ocl, const void *src, size_t n,
                  const char *what);
void ocl_write(struct ocl_backend *ocl, cl_mem dst, size_t off, const void *src,
               size_t n);
void ocl_read(struct ocl_backend *ocl, cl_mem src, size_t off, void *dst,
              size_t n);
void ocl_release(cl_mem *m);

/* CUDA-native additions (no reference counterpart). */

/* A handle over n bytes of existing device memory (not freed by
 * ocl_release, which only frees the handle). */
cl_mem ocl_wrap(void *dptr, size_t n);
void *ocl_ptr(cl_mem m);
size_t ocl_bytes(cl_mem m);
/* Asynchronous device-side copy and zero fill, in bytes, on the stream. */
void ocl_copy(struct ocl_backend *ocl, cl_mem src, size_t soff, cl_mem dst,
              size_t doff, size_t n);
void ocl_zero(struct ocl_backend *ocl, cl_mem m, size_t off, size_t n);
/* Wait for every launch of the backend's stream. */
void ocl_finish(struct ocl_backend *ocl);

/* Later work on dst's stream waits for everything issued so far on src's
 * stream (both backends on the same device); returns at once. Lets several
 * backends of one device, each running its own tiles, be started and
 * finished together (no counterpart in the reference, whose queue is one
 * per device). */
void ocl_join(struct ocl_backend *dst, struct ocl_backend *src);

/* Device timing of the backend's stream: ocl_timer_start records a CUDA
 * event on it, ocl_timer_stop records a second one, waits for it and
 * returns the milliseconds between them. */
void ocl_timer_start(struct ocl_backend *ocl);
double ocl_timer_stop(struct ocl_backend *ocl);

/* Error handling of every entry point of the library. */
#define COREG_ERRORS_FATAL 0
#define COREG_ERRORS_RECORD 1
void coreg_set_error_mode(int mode);
/* The first recorded error of the calling thread, NULL if none. */
const char *coreg_last_error(void);
void coreg_clear_error(void);

#ifdef __cplusplus
}
#endif

#endif /* I_COREGISTRATION_B200_OCL_BACKEND_H */
