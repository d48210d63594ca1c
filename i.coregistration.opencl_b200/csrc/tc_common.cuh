// SPDX-License-Identifier: Unlicense
//
// sm_100a building blocks of the tensor-core kernels (tc_gemm.cu,
// tc_attention.cu): mbarriers with bounded waits, TMA tensor loads,
// tcgen05 shared-memory matrix descriptors, MMA issue and commit, tensor
// memory loads and stores, and the host-side tensor-map encoder.

#pragma once

#include <cuda.h>
#include <stdint.h>

#include "gemm.cuh"

namespace coreg {
namespace tc {

// Error code of the first bounded wait that ran out (0: none); one copy
// per translation unit, read by that unit's status function.
static __device__ int g_error;

__device__ __forceinline__ uint32_t su32(const void *p)
{
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t gtime()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(count));
}

__device__ __forceinline__ void mbar_fence_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *b)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint64_t *b, uint32_t parity)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok)
                 : "r"(su32(b)), "r"(parity)
                 : "memory");
    return ok != 0;
}

// Wait for the phase of the given parity, at most about two seconds of
// global time; on time-out record code and return false.
__device__ __forceinline__ bool mbar_wait(uint64_t *b, uint32_t parity, int code)
{
    if (mbar_try(b, parity))
        return true;
    const uint64_t t0 = gtime();
    while (!mbar_try(b, parity)) {
        if (gtime() - t0 > 2000000000ull) {
            atomicCAS(&g_error, 0, code);
            return false;
        }
    }
    return true;
}

// The same for waiters that are not on the critical path (epilogue warps
// waiting for the whole main loop): back off between tries so that they
// leave the issue slots and the barrier unit to the producer and MMA warps.
__device__ __forceinline__ bool mbar_wait_backoff(uint64_t *b, uint32_t parity, int code)
{
    if (mbar_try(b, parity))
        return true;
    const uint64_t t0 = gtime();
    while (!mbar_try(b, parity)) {
        __nanosleep(256);
        if (gtime() - t0 > 2000000000ull) {
            atomicCAS(&g_error, 0, code);
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map,
                                            uint64_t *bar, int x, int y)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4}], [%2];" ::"r"(su32(dst)),
                 "l"((uint64_t)map), "r"(su32(bar)), "r"(x), "r"(y)
                 : "memory");
}

// Untiled bulk copy of bytes (a multiple of 16, both addresses 16-byte
// aligned) from global memory, completing on the mbarrier.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1], %2, [%3];" ::"r"(su32(dst)),
                 "l"(src), "r"(bytes), "r"(su32(bar))
                 : "memory");
}

// 3-D box (innermost coordinate x first); coordinates outside the tensor
// (negative ones included) read zeros.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map,
                                            uint64_t *bar, int x, int y, int z)
{
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(su32(dst)),
                 "l"((uint64_t)map), "r"(su32(bar)), "r"(x), "r"(y), "r"(z)
                 : "memory");
}

// TMA stores from shared memory (elements outside the tensor are not
// written), their bulk groups, and a named barrier of the epilogue warps.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x,
                                             int y)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                     (uint64_t)map),
                 "r"(su32(src)), "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int x,
                                             int y, int z)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
            (uint64_t)map),
        "r"(su32(src)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

__device__ __forceinline__ void bulk_commit()
{
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read()
{
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until every bulk group of this thread has completed (its global
// writes done).
__device__ __forceinline__ void bulk_wait_all()
{
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void named_bar(int id, int nthreads)
{
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2),
// version 1 (tcgen05). K-major tiles: rows of 128 bytes along K, 8-row
// groups sbo = 1024 bytes apart, lbo unused (1). MN-major tiles: rows of
// 128 bytes (64 elements) along M or N, one row per K index, 8-row K
// groups sbo = 1024 bytes apart, 64-element M/N groups lbo bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr, uint32_t lbo = 16,
                                               uint32_t sbo = 1024)
{
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFF) >> 4);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor of kind::f16: bfloat16 A and B, float32 D,
// M x N, A K-major, B K-major (b_mn 0) or MN-major (b_mn 1).
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int b_mn = 0)
{
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)b_mn << 16) |
           ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem, uint64_t da, uint64_t db,
                                         uint32_t idesc, uint32_t accum)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem),
                 "l"(da), "l"(db), "r"(idesc), "r"(accum));
}

__device__ __forceinline__ void mma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     su32(bar))
                 : "memory");
}

__device__ __forceinline__ void fence_before()
{
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void fence_after()
{
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Generic-proxy shared-memory writes made visible to the tensor cores.
__device__ __forceinline__ void fence_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t cols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     su32(dst)),
                 "r"(cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t tmem, uint32_t cols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(cols));
}

// 32 consecutive columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float v[32])
{
    uint32_t r[32];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                   "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
                   "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                   "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]),
                   "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++)
        v[i] = __uint_as_float(r[i]);
}

// 16 consecutive columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float v[16])
{
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                   "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; i++)
        v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float v[16])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
                 "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
                 "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])),
                 "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
                 "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
                 "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
                 "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])),
                 "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
                 "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
                 "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
                 : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float v[32])
{
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
                 "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
                 "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
                 "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])),
                 "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
                 "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
                 "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
                 "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])),
                 "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
                 "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
                 "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
                 "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
                 "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
                 "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])),
                 "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
                 "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
                 "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
                 "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
                 "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
                 : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Host: 2-D bfloat16 tensor map of a rows x cols row-major matrix
// (leading dimension ld elements), box box_rows x 64, 128-byte swizzle,
// zero fill outside.
bool make_map_2d(CUtensorMap *map, const void *base, long rows, long cols, long ld,
                 int box_rows);
// Host: 3-D bfloat16 tensor map of a channels-last (H, W, C) image, box
// TH x TW x 64.
bool make_map_conv(CUtensorMap *map, const void *base, int H, int W, int C, int TW,
                   int TH);
// Host: tensor map of the output of a GEMM for TMA stores: 2-D rows x cols
// (ld elements) or, with conv set, 3-D channels-last (H, W, cols); element
// size es (4 float, 2 bfloat16), box of 128 bytes of columns x box_rows
// (2-D) or TW x TH pixels (3-D), 128-byte swizzle.
bool make_map_out(CUtensorMap *map, void *base, int es, long rows, long cols, long ld,
                  int conv, int H, int W, int TW, int TH);
// Host: opt in to `bytes` of dynamic shared memory for kernel `fn` on the
// current device (once per device).
bool smem_opt_in(const void *fn, size_t bytes, unsigned *done_mask);

}  // namespace tc
}  // namespace coreg
