/* SPDX-License-Identifier: Unlicense */

/* Test infrastructure: the reference's roma.c, compiled where it lies (the
 * Makefile names it by path in REF_ROMA_C), with three of its static host
 * functions called directly: gp_solve (roma.c:772-836, the Gaussian
 * process's float64 Cholesky solve), prepare (:1159-1186, Pillow's
 * antialiased bicubic and the ImageNet normalization) and interp_pos
 * (:261-298, DINOv2's bicubic position-table interpolation). Every device,
 * ops.h, pth_loader.h and progress entry point that roma.c references is
 * declared weak below and never reached. Built into _ref/libroma_host_ref.so
 * by oracle/Makefile. */

#include REF_ROMA_C

#pragma weak clSetKernelArg
#pragma weak clReleaseKernel
#pragma weak clEnqueueCopyBuffer
#pragma weak clEnqueueCopyBufferRect
#pragma weak clEnqueueFillBuffer
#pragma weak ocl_alloc
#pragma weak ocl_check
#pragma weak ocl_kernel
#pragma weak ocl_read
#pragma weak ocl_release
#pragma weak ocl_upload
#pragma weak ocl_write
#pragma weak ops_axpby
#pragma weak ops_bmat
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
#pragma weak ops_run
#pragma weak ops_softmax_rows
#pragma weak ops_transpose
#pragma weak progress_begin
#pragma weak progress_end
#pragma weak pth_bytes
#pragma weak pth_find
#pragma weak pth_read_f32
#pragma weak pth_require
#pragma weak pth_strip_prefix

void ref_gp_solve(const float *K, int n, float *F, int d) { gp_solve(K, n, F, d); }

void ref_prepare(const float *in, int H, int W, float *out, int h, int w, int imagenet)
{
    prepare(in, H, W, out, h, w, imagenet);
}

/* The (1 + (ROMA_COARSE / 14)^2) x 1024 table, malloc'd. */
float *ref_interp_pos(const float *pos) { return interp_pos(pos); }

int ref_roma_coarse(void) { return ROMA_COARSE; }
