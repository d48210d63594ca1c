/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the reference's OpenCL runtime layer
 * (ocl_backend.h) and the OpenCL calls its host code makes, over host
 * memory, with the reference's four kernel sources compiled as C
 * (cl_programs_emul.c) and dispatched by name. A cl_mem is a host allocation;
 * clSetKernelArg stores the argument bytes; clEnqueueNDRangeKernel runs
 * the kernel's work-items (emul_launch) before it returns, so every queue
 * is always finished. With this, the reference's own ops.c, disk.c,
 * eloftr.c and tests/ops_check.c run unchanged on the CPU (oracle/Makefile
 * builds them against this file). */

#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "cl_backend_emul.h"
#include "ocl_backend.h"
#include "progress.h"

#include <grass/gis.h>

/* ------------------------------------------------------------ runtime */

void ocl_init(struct ocl_backend *ocl, const char *device_opt, const char *platform_opt)
{
    (void)device_opt, (void)platform_opt;
    memset(ocl, 0, sizeof(*ocl));
    snprintf(ocl->device_name, sizeof(ocl->device_name), "OpenCL C on the CPU (emulation)");
    snprintf(ocl->platform_name, sizeof(ocl->platform_name), "oracle/cl_backend_emul.c");
    ocl->max_alloc = (cl_ulong)1 << 34;
    ocl->global_mem = (cl_ulong)1 << 36;
    ocl->is_gpu = 0;
    ocl->profile = 0;
}

void ocl_free(struct ocl_backend *ocl) { memset(ocl, 0, sizeof(*ocl)); }

const char *ocl_errstr(cl_int err) { return err ? "emulation error" : "CL_SUCCESS"; }

void ocl_check(cl_int err, const char *what)
{
    if (err != CL_SUCCESS)
        G_fatal_error("%s failed: %d", what, (int)err);
}

cl_mem ocl_alloc(struct ocl_backend *ocl, size_t n, const char *what)
{
    cl_mem m = G_calloc(1, sizeof(*m));

    (void)ocl, (void)what;
    m->host = G_calloc(n ? n : 1, 1);
    m->bytes = n;
    return m;
}

cl_mem ocl_upload(struct ocl_backend *ocl, const void *src, size_t n, const char *what)
{
    cl_mem m = ocl_alloc(ocl, n, what);

    memcpy(m->host, src, n);
    return m;
}

void ocl_write(struct ocl_backend *ocl, cl_mem dst, size_t off, const void *src, size_t n)
{
    (void)ocl;
    if (off + n > dst->bytes)
        G_fatal_error("ocl_write past the buffer");
    memcpy((char *)dst->host + off, src, n);
}

void ocl_read(struct ocl_backend *ocl, cl_mem src, size_t off, void *dst, size_t n)
{
    (void)ocl;
    if (off + n > src->bytes)
        G_fatal_error("ocl_read past the buffer");
    memcpy(dst, (char *)src->host + off, n);
}

cl_kernel ocl_kernel(struct ocl_backend *ocl, const char *name)
{
    size_t i;

    (void)ocl;
    for (i = 0; i < (size_t)emul_nkernels; i++)
        if (!strcmp(emul_kernels[i].name, name)) {
            cl_kernel k = G_calloc(1, sizeof(*k));

            k->entry = &emul_kernels[i];
            return k;
        }
    G_fatal_error("no kernel <%s>", name);
    return NULL;
}

void ocl_release(cl_mem *m)
{
    if (*m) {
        G_free((*m)->host);
        G_free(*m);
        *m = NULL;
    }
}

cl_int clSetKernelArg(cl_kernel k, cl_uint index, size_t size, const void *value)
{
    if (index >= EMUL_MAX_ARGS || size > 16)
        return -51; /* CL_INVALID_ARG_SIZE */
    memset(k->arg[index], 0, 16);
    if (value)
        memcpy(k->arg[index], value, size);
    return CL_SUCCESS;
}

cl_int clEnqueueNDRangeKernel(cl_command_queue queue, cl_kernel k, cl_uint dims,
                              const size_t *offset, const size_t *global, const size_t *local,
                              cl_uint n_wait, const cl_event *wait, cl_event *event)
{
    size_t g[3] = {1, 1, 1}, l[3] = {1, 1, 1};
    cl_uint d;

    (void)queue, (void)n_wait, (void)wait;
    if (offset)
        return -56; /* CL_INVALID_GLOBAL_OFFSET: the reference passes none */
    for (d = 0; d < dims; d++) {
        g[d] = global[d];
        l[d] = local ? local[d] : 1;
        if (g[d] % l[d])
            return -54; /* CL_INVALID_WORK_GROUP_SIZE */
    }
    emul_launch(k->entry->body, k, g, l);
    if (event)
        *event = NULL;
    return CL_SUCCESS;
}

cl_int clWaitForEvents(cl_uint n, const cl_event *events)
{
    (void)n, (void)events;
    return CL_SUCCESS;
}

cl_int clGetEventProfilingInfo(cl_event event, cl_profiling_info name, size_t size, void *value,
                               size_t *size_ret)
{
    (void)event, (void)name, (void)size_ret;
    memset(value, 0, size);
    return CL_SUCCESS;
}

cl_int clReleaseEvent(cl_event event)
{
    (void)event;
    return CL_SUCCESS;
}

cl_int clReleaseKernel(cl_kernel k)
{
    G_free(k);
    return CL_SUCCESS;
}

cl_int clFinish(cl_command_queue queue)
{
    (void)queue;
    return CL_SUCCESS;
}

cl_int clEnqueueCopyBuffer(cl_command_queue q, cl_mem src, cl_mem dst, size_t so, size_t dof,
                           size_t n, cl_uint nw, const cl_event *w, cl_event *e)
{
    (void)q, (void)nw, (void)w;
    memmove((char *)dst->host + dof, (char *)src->host + so, n);
    if (e)
        *e = NULL;
    return CL_SUCCESS;
}

cl_int clEnqueueCopyBufferRect(cl_command_queue q, cl_mem src, cl_mem dst, const size_t *so,
                               const size_t *dor, const size_t *region, size_t srp, size_t ssp,
                               size_t drp, size_t dsp, cl_uint nw, const cl_event *w,
                               cl_event *e)
{
    size_t x, y, z;

    (void)q, (void)nw, (void)w;
    srp = srp ? srp : region[0];
    drp = drp ? drp : region[0];
    ssp = ssp ? ssp : region[1] * srp;
    dsp = dsp ? dsp : region[1] * drp;
    for (z = 0; z < region[2]; z++)
        for (y = 0; y < region[1]; y++) {
            const char *s = (char *)src->host + (so[2] + z) * ssp + (so[1] + y) * srp + so[0];
            char *d = (char *)dst->host + (dor[2] + z) * dsp + (dor[1] + y) * drp + dor[0];

            for (x = 0; x < region[0]; x++)
                d[x] = s[x];
        }
    if (e)
        *e = NULL;
    return CL_SUCCESS;
}

cl_int clEnqueueFillBuffer(cl_command_queue q, cl_mem b, const void *pattern, size_t psize,
                           size_t off, size_t size, cl_uint nw, const cl_event *w, cl_event *e)
{
    size_t i;

    (void)q, (void)nw, (void)w;
    for (i = 0; i < size; i += psize)
        memcpy((char *)b->host + off + i, pattern, psize);
    if (e)
        *e = NULL;
    return CL_SUCCESS;
}

/* The progress meter of the GRASS module: silent here. */
void progress_plan(enum progress_kind k, double units) { (void)k, (void)units; }
void progress_begin(enum progress_kind k, double units) { (void)k, (void)units; }
void progress_part(double done, double total) { (void)done, (void)total; }
void progress_end(void) {}
void progress_bytes(size_t n) { (void)n; }
double progress_seconds(enum progress_kind k)
{
    (void)k;
    return 0;
}
void progress_finish(void) {}
