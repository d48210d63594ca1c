// SPDX-License-Identifier: Unlicense
//
// DISK on CUDA (disk.h): the U-Net on this build's ops.h kernels, the 5 x 5
// heatmap non-maxima suppression and the descriptor gather as CUDA kernels,
// and the device descriptor-distance stage (desc_nearest).
//
// Network (disk.c:23-31, kornia's Unet(in_features=3, size=5, down=[16, 32,
// 64, 64, 64], up=[64, 64, 64, 129])): down block 0 convolves the input;
// down blocks 1-4 average-pool, take instance-norm statistics (eps 1e-5)
// and convolve the normalized, PReLU-gated input; up blocks upsample the
// bottom input x2 (bilinear, scale factor) into the first 64 channels of a
// concatenation, append the skip connection, take statistics and
// convolve. All convolutions 5 x 5, padding 2.

#include <algorithm>
#include <stdlib.h>
#include <string.h>
#include <vector>

#include "common.cuh"
#include "disk.h"

using namespace coreg;

namespace {

const int layer_cin[DISK_LAYERS] = {3, 16, 32, 64, 64, 128, 128, 96, 80};
const int layer_cout[DISK_LAYERS] = {16, 32, 64, 64, 64, 64, 64, 64, DISK_DESC + 1};

}  // namespace

struct disk_impl {
    cl_mem w[DISK_LAYERS] = {}, b[DISK_LAYERS] = {}, alpha[DISK_LAYERS] = {};
    cl_mem input = nullptr, f[5] = {}, u[3] = {}, tmp = nullptr, cat = nullptr,
           out = nullptr, mean = nullptr, rstd = nullptr, mask = nullptr, xy = nullptr,
           desc = nullptr;
    // Keypoint selection on the device: the valid mask, per-block candidate
    // counts and offsets, the candidates (score, cell) in raster order, the
    // selected scores and the selection's count and cut.
    cl_mem valid = nullptr, counts = nullptr, cscore = nullptr, ccell = nullptr,
           score = nullptr, sel = nullptr;
};

namespace {

cl_mem upload_tensor(struct disk_model *m, struct pth_file *pf, const char *name, int ndim,
                     const long *shape)
{
    const struct pth_tensor *t = pth_require(pf, name, ndim, shape);
    if (!t)
        return nullptr;
    float *v = pth_read_f32(pf, t);
    if (!v)
        return nullptr;
    cl_mem buf = ocl_upload(m->ocl, v, pth_numel(t) * sizeof(float), name);
    free(v);
    return buf;
}

// disk_kernels.cl:10-35: cells of the h x w crop of the heatmap (element
// off, row pitch W) strictly above their 24 neighbours and thresh; the
// 2-cell border is never a candidate.
__global__ void nms5x5_k(const float *heat, int W, int h, int w, float thresh,
                         unsigned char *mask)
{
    const int x = blockIdx.x * blockDim.x + threadIdx.x, y = blockIdx.y;
    if (x >= w || y >= h)
        return;
    if (x < 2 || y < 2 || x >= w - 2 || y >= h - 2) {
        mask[(long)y * w + x] = 0;
        return;
    }
    const float v = heat[(long)y * W + x];
    bool keep = v > thresh;
    for (int dy = -2; dy <= 2 && keep; dy++)
        for (int dx = -2; dx <= 2; dx++)
            if ((dx || dy) && !(v > heat[(long)(y + dy) * W + x + dx])) {
                keep = false;
                break;
            }
    mask[(long)y * w + x] = keep;
}

// disk_kernels.cl:39-60: descriptor channels 0..D-1 at the keypoints,
// L2-normalized (eps 1e-12). One warp per keypoint.
__global__ void gather_desc_k(const float *feat, int H, int W, int D, const int *xy,
                              const int *count, float *desc)
{
    const int k = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x % 32;
    if (k >= *count)
        return;
    const long plane = (long)H * W, off = (long)xy[2 * k + 1] * W + xy[2 * k];
    float ss = 0.0f;
    for (int d = lane; d < D; d += 32) {
        const float v = feat[d * plane + off];
        ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    const float inv = 1.0f / fmaxf(sqrtf(ss), 1e-12f);
    for (int d = lane; d < D; d += 32)
        desc[(long)k * D + d] = feat[d * plane + off] * inv;
}

// ------------------------------------------- keypoint selection kernels
//
// The n-best rule of disk.c:236-266 (kornia heatmap_to_keypoints) on the
// device: the NMS candidates of the h x w crop (valid cells only) in raster
// order, the (n + 1)-th highest score as the cut (with n or fewer
// candidates the lowest), then the candidates strictly above the cut in
// raster order, at most n. Same values, same comparisons as the host
// rule, so the same keypoints.

constexpr int SEL_BLOCK = 1024;  // cells per block of the compaction

// Candidates per block of SEL_BLOCK cells.
__global__ void __launch_bounds__(SEL_BLOCK)
cand_count_k(const unsigned char *mask, const unsigned char *valid, long cells, int *counts)
{
    __shared__ int wsum[SEL_BLOCK / 32];
    const long i = (long)blockIdx.x * SEL_BLOCK + threadIdx.x;
    const bool c = i < cells && mask[i] && (!valid || valid[i]);
    const unsigned b = __ballot_sync(0xffffffffu, c);
    if (threadIdx.x % 32 == 0)
        wsum[threadIdx.x / 32] = __popc(b);
    __syncthreads();
    if (threadIdx.x < 32) {
        int v = wsum[threadIdx.x];
        for (int o = 16; o > 0; o /= 2)
            v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0)
            counts[blockIdx.x] = v;
    }
}

// Exclusive scan of nb counts in place (one block); the total into
// counts[nb].
__global__ void __launch_bounds__(SEL_BLOCK) cand_scan_k(int *counts, int nb)
{
    __shared__ int wsum[SEL_BLOCK / 32];
    __shared__ int carry;
    if (threadIdx.x == 0)
        carry = 0;
    __syncthreads();
    for (int base = 0; base < nb; base += SEL_BLOCK) {
        const int i = base + threadIdx.x, lane = threadIdx.x % 32, wp = threadIdx.x / 32;
        const int v = i < nb ? counts[i] : 0;
        int x = v;
        for (int o = 1; o < 32; o *= 2) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o)
                x += y;
        }
        if (lane == 31)
            wsum[wp] = x;
        __syncthreads();
        if (wp == 0) {
            int w = wsum[lane];
            for (int o = 1; o < 32; o *= 2) {
                const int y = __shfl_up_sync(0xffffffffu, w, o);
                if (lane >= o)
                    w += y;
            }
            wsum[lane] = w;
        }
        __syncthreads();
        const int excl = carry + (wp ? wsum[wp - 1] : 0) + x - v;
        __syncthreads();
        if (i < nb)
            counts[i] = excl;
        if (threadIdx.x == SEL_BLOCK - 1)
            carry = excl + v;
        __syncthreads();
    }
    if (threadIdx.x == 0)
        counts[nb] = carry;
}

// The candidates of each block, in raster order, at the block's offset:
// their score (heat at row pitch W) and cell (y w + x of the crop).
__global__ void __launch_bounds__(SEL_BLOCK)
cand_write_k(const unsigned char *mask, const unsigned char *valid, const float *heat, int W,
             int w, long cells, const int *offs, float *cscore, int *ccell)
{
    __shared__ int wsum[SEL_BLOCK / 32];
    const long i = (long)blockIdx.x * SEL_BLOCK + threadIdx.x;
    const int lane = threadIdx.x % 32, wp = threadIdx.x / 32;
    const bool c = i < cells && mask[i] && (!valid || valid[i]);
    const unsigned b = __ballot_sync(0xffffffffu, c);
    if (lane == 0)
        wsum[wp] = __popc(b);
    __syncthreads();
    if (wp == 0) {
        int x = wsum[lane];
        for (int o = 1; o < 32; o *= 2) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o)
                x += y;
        }
        wsum[lane] = x;
    }
    __syncthreads();
    if (c) {
        const int pos = offs[blockIdx.x] + (wp ? wsum[wp - 1] : 0) +
                        __popc(b & ((1u << lane) - 1u));
        const long y = i / w, x = i % w;
        cscore[pos] = heat[y * W + x];
        ccell[pos] = (int)i;
    }
}

// Order-preserving key of a float (larger float, larger key).
__device__ __forceinline__ unsigned fkey(float f)
{
    const unsigned u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : u | 0x80000000u;
}

__device__ __forceinline__ float fkey_inv(unsigned k)
{
    return __uint_as_float((k & 0x80000000u) ? k & 0x7fffffffu : ~k);
}

// The cut of the n-best rule over the C = *total candidate scores: the
// (n + 1)-th highest (0-based rank kk = min(n, C - 1) from the top) by a
// 4-round radix select on the keys, into sel[1] (as a float's bits); -inf
// without candidates. One block.
__global__ void __launch_bounds__(SEL_BLOCK)
select_cut_k(const float *cscore, const int *total, int n, int *sel)
{
    __shared__ unsigned hist[256];
    __shared__ unsigned prefix, pmask;
    __shared__ int rank;
    const int C = *total;
    if (C == 0) {
        if (threadIdx.x == 0)
            sel[1] = __float_as_int(-INFINITY);
        return;
    }
    if (threadIdx.x == 0) {
        prefix = 0;
        pmask = 0;
        // Rank from the bottom of the wanted key.
        rank = C - 1 - (C > n ? n : C - 1);
    }
    __syncthreads();
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int t = threadIdx.x; t < 256; t += SEL_BLOCK)
            hist[t] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < C; i += SEL_BLOCK) {
            const unsigned k = fkey(cscore[i]);
            if ((k & pmask) == prefix)
                atomicAdd(&hist[(k >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int r = rank;
            unsigned d = 0;
            for (; d < 256; d++) {
                if (r < (int)hist[d])
                    break;
                r -= hist[d];
            }
            rank = r;
            prefix |= d << shift;
            pmask |= 255u << shift;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0)
        sel[1] = __float_as_int(fkey_inv(prefix));
}

// The candidates strictly above the cut, in raster order, at most n: x, y
// into xy, scores into score, their count into sel[0]. One block walks
// the candidates SEL_BLOCK at a time.
__global__ void __launch_bounds__(SEL_BLOCK)
select_write_k(const float *cscore, const int *ccell, const int *total, int w, int n, int *sel,
               int *xy, float *score)
{
    __shared__ int wsum[SEL_BLOCK / 32];
    __shared__ int base;
    const int C = *total;
    const float cut = __int_as_float(sel[1]);
    const int lane = threadIdx.x % 32, wp = threadIdx.x / 32;
    if (threadIdx.x == 0)
        base = 0;
    __syncthreads();
    for (int c0 = 0; c0 < C; c0 += SEL_BLOCK) {
        if (base >= n)
            break;
        const int i = c0 + threadIdx.x;
        const bool keep = i < C && cscore[i] > cut;
        const unsigned b = __ballot_sync(0xffffffffu, keep);
        if (lane == 0)
            wsum[wp] = __popc(b);
        __syncthreads();
        if (wp == 0) {
            int x = wsum[lane];
            for (int o = 1; o < 32; o *= 2) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o)
                    x += y;
            }
            wsum[lane] = x;
        }
        __syncthreads();
        const int pos = base + (wp ? wsum[wp - 1] : 0) + __popc(b & ((1u << lane) - 1u));
        if (keep && pos < n) {
            xy[2 * pos] = ccell[i] % w;
            xy[2 * pos + 1] = ccell[i] / w;
            score[pos] = cscore[i];
        }
        __syncthreads();
        if (threadIdx.x == 0)
            base += wsum[SEL_BLOCK / 32 - 1];
        __syncthreads();
    }
    if (threadIdx.x == 0)
        sel[0] = base < n ? base : n;
}

void conv(struct disk_model *m, int l, cl_mem in, int H, int W, cl_mem out)
{
    struct conv_geom g = ops_geom(5, 1, 2);
    disk_impl *I = m->impl;
    if (l > 0)
        ops_conv2d(m->ops, in, layer_cin[l], H, W, I->w[l], I->b[l], layer_cout[l], &g,
                   I->mean, I->rstd, I->alpha[l], ACT_NONE, 0.0f, out);
    else
        ops_conv2d(m->ops, in, layer_cin[l], H, W, I->w[l], I->b[l], layer_cout[l], &g,
                   nullptr, nullptr, nullptr, ACT_NONE, 0.0f, out);
}

}  // namespace

extern "C" void disk_load(struct disk_model *m, struct ops *ops, struct pth_file *pf)
{
    memset(m, 0, sizeof(*m));
    if (pending())
        return;
    m->ocl = ops->ocl;
    m->ops = ops;
    m->impl = new disk_impl();
    char name[128];
    for (int l = 0; l < DISK_LAYERS; l++) {
        long wshape[4] = {layer_cout[l], layer_cin[l], 5, 5};
        long bshape[1] = {layer_cout[l]}, ashape[1] = {layer_cin[l]};
        const char *prefix = l < 5 ? "unet.path_down.%d.1.%d.%s" : "unet.path_up.%d.conv.%d.%s";
        const int idx = l < 5 ? l : l - 5;
        m->cin[l] = layer_cin[l];
        m->cout[l] = layer_cout[l];
        snprintf(name, sizeof(name), prefix, idx, 3, "weight");
        m->impl->w[l] = upload_tensor(m, pf, name, 4, wshape);
        snprintf(name, sizeof(name), prefix, idx, 3, "bias");
        m->impl->b[l] = upload_tensor(m, pf, name, 1, bshape);
        if (l > 0) {
            snprintf(name, sizeof(name), prefix, idx, 1, "weight");
            m->impl->alpha[l] = upload_tensor(m, pf, name, 1, ashape);
        }
    }
}

extern "C" void disk_alloc(struct disk_model *m, int H, int W, int nmax)
{
    if (pending())
        return;
    if (!m->impl) {
        fail("DISK: disk_alloc before disk_load");
        return;
    }
    if (H <= 0 || W <= 0 || H % DISK_MULTIPLE || W % DISK_MULTIPLE || nmax < 1) {
        fail("DISK tile %d x %d is not a multiple of %d (or %d keypoints)", H, W,
             DISK_MULTIPLE, nmax);
        return;
    }
    disk_impl *I = m->impl;
    const size_t px = (size_t)H * W;
    struct ocl_backend *ocl = m->ocl;
    m->H = H;
    m->W = W;
    m->nmax = nmax;
    I->input = ocl_alloc(ocl, 3 * px * 4, "input");
    for (int k = 0; k < 5; k++)
        I->f[k] = ocl_alloc(ocl, layer_cout[k] * (px >> (2 * k)) * 4, "down features");
    for (int k = 0; k < 3; k++)
        I->u[k] = ocl_alloc(ocl, 64 * (px >> (2 * (3 - k))) * 4, "up features");
    I->tmp = ocl_alloc(ocl, 16 * (px >> 2) * 4, "pooled");
    I->cat = ocl_alloc(ocl, 80 * px * 4, "concatenation");
    I->out = ocl_alloc(ocl, (DISK_DESC + 1) * px * 4, "output");
    I->mean = ocl_alloc(ocl, 128 * 4, "mean");
    I->rstd = ocl_alloc(ocl, 128 * 4, "rstd");
    I->mask = ocl_alloc(ocl, px, "nms mask");
    I->xy = ocl_alloc(ocl, 2 * (size_t)nmax * 4, "keypoints");
    I->desc = ocl_alloc(ocl, (size_t)nmax * DISK_DESC * 4, "descriptors");
    const long nblk = cdiv((long)px, SEL_BLOCK);
    I->valid = ocl_alloc(ocl, px, "valid mask");
    I->counts = ocl_alloc(ocl, (nblk + 1) * 4, "candidate counts");
    I->cscore = ocl_alloc(ocl, px * 4, "candidate scores");
    I->ccell = ocl_alloc(ocl, px * 4, "candidate cells");
    I->score = ocl_alloc(ocl, (size_t)nmax * 4, "keypoint scores");
    I->sel = ocl_alloc(ocl, 2 * 4, "selection");
}

extern "C" int disk_detect(struct disk_model *m, const float *img, int H, int W, int h,
                           int w, int n, float thresh, const unsigned char *valid, int *xy,
                           float *score, float *desc)
{
    if (pending())
        return 0;
    if (!m->impl || !m->impl->out) {
        fail("DISK: disk_detect before disk_alloc");
        return 0;
    }
    if (H > m->H || W > m->W || H % DISK_MULTIPLE || W % DISK_MULTIPLE || h < 1 || w < 1 ||
        h > H || w > W) {
        fail("DISK: tile %d x %d (content %d x %d) does not fit the %d x %d buffers", H, W, h,
             w, m->H, m->W);
        return 0;
    }
    disk_impl *I = m->impl;
    struct ocl_backend *ocl = m->ocl;
    cudaSetDevice(ocl->device);
    cudaStream_t st = stream_of(ocl);
    const size_t px = (size_t)H * W;
    if (n > m->nmax)
        n = m->nmax;
    ocl_write(ocl, I->input, 0, img, 3 * px * 4);

    // Down path.
    conv(m, 0, I->input, H, W, I->f[0]);
    for (int lev = 1; lev < 5; lev++) {
        const int c = layer_cout[lev - 1], hh = H >> lev, ww = W >> lev;
        cl_mem t = lev == 1 ? I->tmp : I->cat;
        ops_avgpool2(m->ops, I->f[lev - 1], c, H >> (lev - 1), W >> (lev - 1), t);
        ops_chan_stats(m->ops, t, c, hh * ww, 1e-5f, I->mean, I->rstd);
        conv(m, lev, t, hh, ww, I->f[lev]);
    }
    // Up path: the upsampled bottom input, then the skip connection.
    for (int j = 0; j < 4; j++) {
        const int l = 5 + j, lvl = 3 - j, hh = H >> lvl, ww = W >> lvl;
        cl_mem bot = j == 0 ? I->f[4] : I->u[j - 1];
        const int cb = 64, ch = layer_cout[lvl];
        const size_t plane = (size_t)hh * ww;
        ops_resize(m->ops, bot, cb, hh / 2, ww / 2, I->cat, hh, ww, 0, 0, 2.0f);
        cuda_ok(cudaMemcpyAsync((float *)I->cat->ptr + cb * plane, I->f[lvl]->ptr,
                                ch * plane * 4, cudaMemcpyDeviceToDevice, st),
                "DISK skip connection");
        ops_chan_stats(m->ops, I->cat, cb + ch, (int)plane, 1e-5f, I->mean, I->rstd);
        conv(m, l, I->cat, hh, ww, j < 3 ? I->u[j] : I->out);
    }
    // Heatmap NMS on the h x w crop, then the n-best selection and the
    // descriptor gather on the device; only the keypoints come back.
    const float *heat = (const float *)I->out->ptr + (size_t)DISK_DESC * px;
    nms5x5_k<<<dim3(cdiv(w, 128), h), 128, 0, st>>>(heat, W, h, w, thresh,
                                                    (unsigned char *)I->mask->ptr);
    const long cells = (long)h * w;
    const int nb = (int)cdiv(cells, SEL_BLOCK);
    const unsigned char *vd = nullptr;
    if (valid) {
        ocl_write(ocl, I->valid, 0, valid, (size_t)cells);
        vd = (const unsigned char *)I->valid->ptr;
    }
    int *counts = (int *)I->counts->ptr, *sel = (int *)I->sel->ptr;
    const unsigned char *mk = (const unsigned char *)I->mask->ptr;
    cand_count_k<<<nb, SEL_BLOCK, 0, st>>>(mk, vd, cells, counts);
    cand_scan_k<<<1, SEL_BLOCK, 0, st>>>(counts, nb);
    cand_write_k<<<nb, SEL_BLOCK, 0, st>>>(mk, vd, heat, W, w, cells, counts,
                                           (float *)I->cscore->ptr, (int *)I->ccell->ptr);
    select_cut_k<<<1, SEL_BLOCK, 0, st>>>((const float *)I->cscore->ptr, counts + nb, n, sel);
    select_write_k<<<1, SEL_BLOCK, 0, st>>>((const float *)I->cscore->ptr,
                                            (const int *)I->ccell->ptr, counts + nb, w, n, sel,
                                            (int *)I->xy->ptr, (float *)I->score->ptr);
    gather_desc_k<<<cdiv(n, 8), 256, 0, st>>>((const float *)I->out->ptr, H, W, DISK_DESC,
                                              (const int *)I->xy->ptr, sel,
                                              (float *)I->desc->ptr);
    if (!launch_ok("disk keypoint selection"))
        return 0;
    int nk = 0;
    ocl_read(ocl, I->sel, 0, &nk, sizeof(int));
    if (pending() || nk <= 0)
        return 0;
    ocl_read(ocl, I->xy, 0, xy, 2 * (size_t)nk * 4);
    ocl_read(ocl, I->score, 0, score, (size_t)nk * 4);
    ocl_read(ocl, I->desc, 0, desc, (size_t)nk * DISK_DESC * 4);
    return pending() ? 0 : nk;
}

extern "C" const float *disk_output_dev(const struct disk_model *m)
{
    return m && m->impl && m->impl->out ? (const float *)m->impl->out->ptr : nullptr;
}

extern "C" void disk_free(struct disk_model *m)
{
    disk_impl *I = m->impl;
    if (I) {
        for (int k = 0; k < DISK_LAYERS; k++) {
            ocl_release(&I->w[k]);
            ocl_release(&I->b[k]);
            ocl_release(&I->alpha[k]);
        }
        cl_mem *bufs[] = {&I->input, &I->tmp, &I->cat, &I->out, &I->mean, &I->rstd,
                          &I->mask, &I->xy, &I->desc, &I->valid, &I->counts, &I->cscore,
                          &I->ccell, &I->score, &I->sel};
        for (cl_mem *b : bufs)
            ocl_release(b);
        for (int k = 0; k < 5; k++)
            ocl_release(&I->f[k]);
        for (int k = 0; k < 3; k++)
            ocl_release(&I->u[k]);
        delete I;
    }
    memset(m, 0, sizeof(*m));
}

// ------------------------------------------------------- distance stage

namespace {

// Squared norms of n rows of dim floats.
__global__ void row_sq_k(const float *d, int n, int dim, float *q)
{
    const int i = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x % 32;
    if (i >= n)
        return;
    float s = 0.0f;
    for (int k = lane; k < dim; k += 32)
        s = fmaf(d[(long)i * dim + k], d[(long)i * dim + k], s);
    s = warp_sum(s);
    if (lane == 0)
        q[i] = s;
}

// Row i of the distance matrix dist = q1[i] + q2[j] - 2 dots[i][j]: the
// smallest (lowest index on ties) and the second smallest; one warp per
// row (adalam.c:62-82).
__global__ void row_best2_k(const float *dots, const float *q1, const float *q2, int n1, int n2,
                            int *nn12, float *score)
{
    const int i = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x % 32;
    if (i >= n1)
        return;
    float best = INFINITY, second = INFINITY;
    int bj = 0x7fffffff;
    for (int j = lane; j < n2; j += 32) {
        const float d = q1[i] + q2[j] - 2.0f * dots[(long)i * n2 + j];
        if (d < best) {
            second = best;
            best = d;
            bj = j;
        }
        else if (d < second)
            second = d;
    }
    for (int o = 16; o > 0; o /= 2) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const float os = __shfl_xor_sync(0xffffffffu, second, o);
        const int oj = __shfl_xor_sync(0xffffffffu, bj, o);
        if (ob < best || (ob == best && oj < bj)) {
            second = fminf(best, os);
            best = ob;
            bj = oj;
        }
        else
            second = fminf(second, ob);
    }
    if (lane == 0) {
        nn12[i] = bj;
        score[i] = best / (second > 1e-3f ? second : 1e-3f);
    }
}

// Column j: the row of the smallest distance (lowest index on ties); one
// thread per column, rows in order (adalam.c:84-94).
__global__ void col_best_k(const float *dots, const float *q1, const float *q2, int n1, int n2,
                           int *nn21)
{
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= n2)
        return;
    float best = INFINITY;
    int bi = 0;
    for (int i = 0; i < n1; i++) {
        const float d = q1[i] + q2[j] - 2.0f * dots[(long)i * n2 + j];
        if (d < best) {
            best = d;
            bi = i;
        }
    }
    nn21[j] = bi;
}

}  // namespace

extern "C" void desc_nearest(struct ops *o, const float *d1, int n1, const float *d2, int n2,
                             int dim, int *nn12, float *score, int *nn21)
{
    if (pending())
        return;
    if (n1 <= 0 || n2 <= 0 || dim <= 0) {
        fail("desc_nearest: %d x %d descriptors of %d", n1, n2, dim);
        return;
    }
    struct ocl_backend *ocl = o->ocl;
    cudaSetDevice(ocl->device);
    cudaStream_t st = stream_of(ocl);
    cl_mem A = ocl_upload(ocl, d1, (size_t)n1 * dim * 4, "descriptors 1");
    cl_mem B = ocl_upload(ocl, d2, (size_t)n2 * dim * 4, "descriptors 2");
    cl_mem D = ocl_alloc(ocl, (size_t)n1 * n2 * 4, "descriptor dots");
    cl_mem Q = ocl_alloc(ocl, ((size_t)n1 + n2) * 4, "descriptor norms");
    cl_mem R = ocl_alloc(ocl, ((size_t)2 * n1 + n2) * 4, "nearest");
    if (!pending()) {
        // The dot products as a float32 GEMM (A B^T), whatever ops' precision:
        // the indices are compared exactly.
        const int prec = o->precision;
        o->precision = OPS_FP32;
        ops_gemm(o, n1, n2, dim, ops_mat(A, 0, dim), ops_mat(B, 0, dim), 1, ops_mat(D, 0, n2), 1,
                 1, nullptr, 0, nullptr, 0, 1.0f, ACT_NONE, 0.0f);
        o->precision = prec;
        float *q1 = (float *)Q->ptr, *q2 = q1 + n1;
        int *r12 = (int *)R->ptr, *r21 = r12 + 2 * n1;
        float *rs = (float *)(r12 + n1);
        row_sq_k<<<cdiv(n1, 8), 256, 0, st>>>((const float *)A->ptr, n1, dim, q1);
        row_sq_k<<<cdiv(n2, 8), 256, 0, st>>>((const float *)B->ptr, n2, dim, q2);
        row_best2_k<<<cdiv(n1, 8), 256, 0, st>>>((const float *)D->ptr, q1, q2, n1, n2, r12, rs);
        if (nn21)
            col_best_k<<<cdiv(n2, 128), 128, 0, st>>>((const float *)D->ptr, q1, q2, n1, n2, r21);
        if (launch_ok("desc_nearest")) {
            ocl_read(ocl, R, 0, nn12, (size_t)n1 * 4);
            ocl_read(ocl, R, (size_t)n1 * 4, score, (size_t)n1 * 4);
            if (nn21)
                ocl_read(ocl, R, (size_t)2 * n1 * 4, nn21, (size_t)n2 * 4);
        }
    }
    ocl_release(&A);
    ocl_release(&B);
    ocl_release(&D);
    ocl_release(&Q);
    ocl_release(&R);
}
