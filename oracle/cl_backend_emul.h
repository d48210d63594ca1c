/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the objects of the OpenCL emulation shared by its
 * runtime (cl_backend_emul.c) and its compiled kernels
 * (cl_programs_emul.c). */

#ifndef COREG_CL_BACKEND_EMUL_H
#define COREG_CL_BACKEND_EMUL_H

#include <string.h>

#include <CL/cl.h>

#define EMUL_MAX_ARGS 40

/* A buffer: host memory. */
struct shim_cl_mem {
    void *host;
    size_t bytes;
};

/* A kernel by name, its work-item body and argument count. */
struct emul_kernel_entry {
    const char *name;
    void (*body)(void *);
    int nargs;
};

/* A kernel object: its entry and the bytes clSetKernelArg stored. */
struct shim_cl_kernel {
    const struct emul_kernel_entry *entry;
    unsigned char arg[EMUL_MAX_ARGS][16];
};

#ifdef __cplusplus
extern "C" {
#endif
extern const struct emul_kernel_entry emul_kernels[];
extern const int emul_nkernels;
#ifdef __cplusplus
}
#endif

static inline void *emul_arg_val(struct shim_cl_kernel *k, int i) { return k->arg[i]; }

/* A buffer argument: the host memory of the stored cl_mem. */
static inline void *emul_arg_ptr(struct shim_cl_kernel *k, int i)
{
    cl_mem m;

    memcpy(&m, k->arg[i], sizeof(m));
    return m ? m->host : NULL;
}

#ifdef __cplusplus
extern "C"
#endif
void emul_launch(void (*body)(void *), void *args, const size_t g[3], const size_t l[3]);

#endif /* COREG_CL_BACKEND_EMUL_H */
