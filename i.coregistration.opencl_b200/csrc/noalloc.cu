// SPDX-License-Identifier: Unlicense
//
// ops_gemm_noalloc: ops_gemm with its bfloat16 operand staging in a fixed
// device array that belongs to the library, so that a call allocates no
// device memory.
//
// ops_gemm (ops.cu) packs the float32 operands of an OPS_BF16 product into
// o->scratch16 and grows that buffer with ocl_alloc (cudaMalloc) when a
// product needs more room. Some callers cannot allow that: a plug-in
// hosted by a framework whose caching allocator already holds the
// device's free memory (a cudaMalloc of its own may fail or fragment what
// the host keeps), and latency-bound pipelines that do all their
// allocation at start-up because cudaMalloc synchronises the whole device.
// This variant stages the packed operands in NOALLOC_SCRATCH_BYTES of file
// scope device memory instead, which the CUDA runtime reserves when it
// loads this file's module.
//
// Set-up: the first call on each device looks up the array's device
// address (cudaGetSymbolAddress, with that device current) and keeps it;
// the kernels receive that pointer. That look-up may load the module, so
// the first call on a device should come before any stream capture.
//
// Every call on a device shares the one array: calls that overlap in time
// (other streams, other host threads, other ops contexts on the device)
// overwrite each other's operands. Nothing in the array needs to start at
// zero: a call writes every element it reads afterwards (the tensor maps of
// the tensor-core tiles stop at the packed extents and zero-fill beyond).

#include <mutex>

#include "gemm.cuh"
#include "ops_b200.h"

using namespace coreg;

namespace {

const size_t NOALLOC_SCRATCH_BYTES = (size_t)16 << 20;
const int NOALLOC_MAX_DEVICES = 64;

__device__ __align__(256) unsigned char noalloc_scratch[NOALLOC_SCRATCH_BYTES];

std::mutex noalloc_mutex;
void *noalloc_ptr[NOALLOC_MAX_DEVICES];

// Device address of noalloc_scratch on `dev`, looked up once per device
// with that device current (the caller's current device is restored);
// NULL after recording an error.
void *scratch_of(int dev)
{
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES) {
        fail("ops_gemm_noalloc: device %d outside 0..%d", dev, NOALLOC_MAX_DEVICES - 1);
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(noalloc_mutex);
    if (noalloc_ptr[dev])
        return noalloc_ptr[dev];
    int cur = -1;
    if (!cuda_ok(cudaGetDevice(&cur), "cudaGetDevice"))
        return nullptr;
    if (cur != dev && !cuda_ok(cudaSetDevice(dev), "cudaSetDevice"))
        return nullptr;
    void *p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, noalloc_scratch);
    if (cur != dev)
        cudaSetDevice(cur);
    if (e != cudaSuccess || !p) {
        fail("ops_gemm_noalloc: cudaGetSymbolAddress of the scratch array on "
             "device %d: %s", dev, cudaGetErrorString(e));
        return nullptr;
    }
    noalloc_ptr[dev] = p;
    return p;
}

}  // namespace

extern "C" size_t ops_gemm_noalloc_max_bytes(void)
{
    return NOALLOC_SCRATCH_BYTES;
}

extern "C" void ops_gemm_noalloc(struct ops *o, int M, int N, int K, struct opnd A,
                                 struct opnd B, int transb, struct opnd C, int nb,
                                 int nb1, cl_mem bias, int biasrow, cl_mem R, long roff,
                                 float alpha, int act, float slope)
{
    if (pending())
        return;
    if (!o || !o->ocl || !A.buf || !B.buf || !C.buf) {
        fail("ops_gemm_noalloc: NULL context or operand");
        return;
    }
    if (nb < 1 || nb1 < 1 || M < 0 || N < 0 || K < 0) {
        fail("ops_gemm_noalloc: shape %d x %d x %d, batch %d / %d", M, N, K, nb, nb1);
        return;
    }
    GemmArgs g = gemm_args(M, N, K);
    g.A = fptr(A.buf, A.off);
    g.lda = A.ld;
    g.sa0 = A.s0;
    g.sa1 = A.s1;
    g.B = fptr(B.buf, B.off);
    g.ldb = B.ld;
    g.sb0 = B.s0;
    g.sb1 = B.s1;
    g.transb = transb;
    g.C = fptr(C.buf, C.off);
    g.ldc = C.ld;
    g.sc0 = C.s0;
    g.sc1 = C.s1;
    g.nb = nb;
    g.nb1 = nb1;
    g.bias = fptr(bias);
    g.biasrow = biasrow;
    g.R = R ? fptr(R, roff) : nullptr;
    g.alpha = alpha;
    g.act = act;
    g.slope = slope;
    g.ab = DT_F32;
    g.c = DT_F32;
    cudaStream_t st = stream_of(o->ocl);

    if (!gemm_packs_bf16(o->precision, M, N, K)) {
        // The float32 tiles stage nothing.
        gemm_simt(st, g);
        launch_ok("ops_gemm_noalloc");
        return;
    }
    const size_t ea = (size_t)nb * M * K, eb = (size_t)nb * N * K;
    const size_t a_bytes = (ea * 2 + 255) / 256 * 256;
    const size_t bytes = a_bytes + eb * 2;
    if (bytes > NOALLOC_SCRATCH_BYTES) {
        fail("ops_gemm_noalloc: the bfloat16 operands of %d x %d x %d (batch %d) "
             "take %zu bytes, more than the %zu-byte scratch array; use ops_gemm",
             M, N, K, nb, bytes, NOALLOC_SCRATCH_BYTES);
        return;
    }
    unsigned char *base = (unsigned char *)scratch_of(o->ocl->device);
    if (!base)
        return;
    __nv_bfloat16 *a16 = (__nv_bfloat16 *)base;
    __nv_bfloat16 *b16 = (__nv_bfloat16 *)(base + a_bytes);
    pack_bf16_rows(st, (const float *)g.A, g.lda, g.sa0, g.sa1, nb, nb1, M, K, a16);
    if (transb)
        pack_bf16_rows(st, (const float *)g.B, g.ldb, g.sb0, g.sb1, nb, nb1, N, K, b16);
    else
        pack_bf16_cols(st, (const float *)g.B, g.ldb, g.sb0, g.sb1, nb, nb1, K, N, b16);
    if (!launch_ok("ops_gemm_noalloc pack"))
        return;
    GemmArgs h = g;
    h.A = a16;
    h.lda = K;
    h.sa0 = (long)M * K * nb1;
    h.sa1 = (long)M * K;
    h.B = b16;
    h.ldb = K;
    h.sb0 = (long)N * K * nb1;
    h.sb1 = (long)N * K;
    h.transb = 1;
    h.ab = DT_BF16;
    if (!gemm_tc(st, h, o->ocl->sm_count))
        gemm_simt(st, h);
    launch_ok("ops_gemm_noalloc");
}
