/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the reference's eloftr.c, compiled where it lies
 * (the Makefile names it by path in REF_ELOFTR_C), with its static host
 * function rope_table (eloftr.c:267-291: the RoPE cos / sin table of the
 * aggregated grid, positions scaled by pos_scale) called directly; the
 * upload it ends with hands the table back here. Every other device,
 * ops.h, weight-file and progress entry point that eloftr.c names is a weak
 * symbol that is never reached. Built into _ref/libeloftr_host_ref.so by
 * oracle/Makefile. */

#include REF_ELOFTR_C

#include <stdlib.h>
#include <string.h>

static float *captured;
static size_t captured_bytes;

cl_mem ocl_upload(struct ocl_backend *ocl, const void *src, size_t n, const char *what)
{
    (void)ocl, (void)what;
    if (captured && n <= captured_bytes)
        memcpy(captured, src, n);
    return NULL;
}

#pragma weak clEnqueueCopyBuffer
#pragma weak clReleaseKernel
#pragma weak clSetKernelArg
#pragma weak ocl_alloc
#pragma weak ocl_check
#pragma weak ocl_kernel
#pragma weak ocl_read
#pragma weak ocl_release
#pragma weak ocl_write
#pragma weak ops_attention
#pragma weak ops_axpby
#pragma weak ops_conv1x1
#pragma weak ops_conv2d
#pragma weak ops_fold_bn
#pragma weak ops_gemm
#pragma weak ops_geom
#pragma weak ops_layernorm
#pragma weak ops_linear
#pragma weak ops_mat
#pragma weak ops_pool2d
#pragma weak ops_resize
#pragma weak ops_rope
#pragma weak ops_run
#pragma weak ops_transpose
#pragma weak progress_begin
#pragma weak progress_end
#pragma weak pth_bytes
#pragma weak pth_find
#pragma weak pth_read_f32
#pragma weak pth_require

/* The table of an ah x aw aggregated grid: (ah * aw, ELOFTR_DIM / 2, 2)
 * floats (cos, sin) into out. */
void ref_rope_table(int ah, int aw, float pos_scale, float *out)
{
    struct eloftr_model m;

    memset(&m, 0, sizeof(m));
    m.ah = ah;
    m.aw = aw;
    m.pos_scale = pos_scale;
    captured = out;
    captured_bytes = (size_t)ah * aw * ELOFTR_DIM * sizeof(float);
    rope_table(&m);
    captured = NULL;
}
