// SPDX-License-Identifier: Unlicense
//
// Efficient LoFTR on CUDA (eloftr.h). The network runs on this build's ops.h
// kernels, channel-major float32 as the reference; the coarse matching (row
// log-sum-exp, running column statistics, dual-softmax confidences with
// first argmaxes, by blocks of rows) and the two-stage fine matching are
// this file's kernels, with the semantics of eloftr_kernels.cl.
//
// Model (eloftr.c:39-53, EfficientLoFTRConfig): RepVGG stages of 1, 2, 4, 14
// blocks (64, 64, 128, 256 channels, strides 2, 1, 2, 2), each block's 3 x 3,
// 1 x 1 and identity branches with their BatchNorms folded into one 3 x 3
// convolution + ReLU; 4 layers of aggregated self / self / cross / cross
// attention (depthwise 4 x 4 stride 4 query aggregation, 4 x 4 max-pooled
// keys and values, LayerNorm, 8 heads, 2-D RoPE on self attention, x4
// bilinear upsampling, MLP 512 with LeakyReLU 0.01, LayerNorm, residual);
// coarse dual softmax at temperature 0.1, threshold 0.2, border 2; fine
// fusion to 64 channels at full resolution; fine matching on 8 x 8 windows.

#include <algorithm>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <string>
#include <vector>

#include "common.cuh"
#include "eloftr.h"

using namespace coreg;

namespace {

const int stage_blocks[4] = {1, 2, 4, 14};
const int stage_out[4] = {64, 64, 128, 256};
const int stage_stride[4] = {2, 1, 2, 2};
constexpr int HEADS = 8, MLP = 512, BORDER = 2;
constexpr float EPS_BN = 1e-5f, EPS_LN = 1e-5f, LEAKY = 0.01f;
constexpr float COARSE_T = 0.1f, COARSE_THR = 0.2f, FINE_T = 10.0f;
constexpr double ROPE_BASE = 10000.0;
constexpr int ROPE_DIM = 128;  // head dim x partial rotary factor: 32 x 4

struct Attn {
    cl_mem q_agg = nullptr, norm_g = nullptr, norm_b = nullptr, wq = nullptr, wk = nullptr,
           wv = nullptr, wo = nullptr, fc1 = nullptr, fc2 = nullptr, mlp_g = nullptr,
           mlp_b = nullptr;
};

}  // namespace

struct eloftr_impl {
    cl_mem bw[ELOFTR_BLOCKS] = {}, bb[ELOFTR_BLOCKS] = {};
    int bcin[ELOFTR_BLOCKS] = {}, bcout[ELOFTR_BLOCKS] = {}, bstride[ELOFTR_BLOCKS] = {};
    Attn self_attn[ELOFTR_LAYERS], cross_attn[ELOFTR_LAYERS];
    cl_mem f_out = nullptr, f1_w[2] = {}, f2_w[2] = {}, f2_b[2] = {}, f3_w[2] = {};
    // Work buffers.
    cl_mem img = nullptr, s_a = nullptr, s_b = nullptr, f1[2] = {}, f2[2] = {}, x[2] = {},
           fine[2] = {};
    cl_mem t_q = nullptr, t_kv = nullptr, t_qn = nullptr, t_kvn = nullptr, t_Q = nullptr,
           t_K = nullptr, t_V = nullptr, t_O = nullptr, t_O2 = nullptr, t_cat = nullptr,
           t_tok = nullptr, t_h1 = nullptr, t_h2 = nullptr, rope = nullptr;
    cl_mem s_blk = nullptr, row_lse = nullptr, col_m = nullptr, col_s = nullptr,
           row_max = nullptr, row_arg = nullptr, col_max = nullptr, col_arg = nullptr;
    cl_mem fu_a = nullptr, fu_b = nullptr, fu_c = nullptr, m_idx = nullptr, m_out = nullptr;
    int blk_rows = 0;
    std::vector<cl_mem *> all()
    {
        std::vector<cl_mem *> v = {&f_out, &img, &s_a, &s_b, &t_q, &t_kv, &t_qn, &t_kvn, &t_Q,
                                   &t_K, &t_V, &t_O, &t_O2, &t_cat, &t_tok, &t_h1, &t_h2, &rope,
                                   &s_blk, &row_lse, &col_m, &col_s, &row_max, &row_arg,
                                   &col_max, &col_arg, &fu_a, &fu_b, &fu_c, &m_idx, &m_out};
        for (int i = 0; i < 2; i++) {
            v.push_back(&f1[i]);
            v.push_back(&f2[i]);
            v.push_back(&x[i]);
            v.push_back(&fine[i]);
            v.push_back(&f1_w[i]);
            v.push_back(&f2_w[i]);
            v.push_back(&f2_b[i]);
            v.push_back(&f3_w[i]);
        }
        for (int l = 0; l < ELOFTR_BLOCKS; l++) {
            v.push_back(&bw[l]);
            v.push_back(&bb[l]);
        }
        for (int l = 0; l < ELOFTR_LAYERS; l++)
            for (Attn *a : {&self_attn[l], &cross_attn[l]})
                for (cl_mem *p : {&a->q_agg, &a->norm_g, &a->norm_b, &a->wq, &a->wk, &a->wv,
                                  &a->wo, &a->fc1, &a->fc2, &a->mlp_g, &a->mlp_b})
                    v.push_back(p);
        return v;
    }
};

namespace {

std::vector<float> read_host(struct pth_file *pf, const std::string &name, int ndim,
                             const long *shape)
{
    std::vector<float> v;
    const struct pth_tensor *t = pth_require(pf, name.c_str(), ndim, shape);
    if (!t)
        return v;
    float *p = pth_read_f32(pf, t);
    if (p) {
        v.assign(p, p + pth_numel(t));
        free(p);
    }
    return v;
}

cl_mem upload(struct eloftr_model *m, const std::vector<float> &v, const char *what)
{
    if (v.empty())
        return nullptr;
    return ocl_upload(m->ocl, v.data(), v.size() * 4, what);
}

cl_mem load_dev(struct eloftr_model *m, struct pth_file *pf, const std::string &name, int ndim,
                const long *shape)
{
    return upload(m, read_host(pf, name, ndim, shape), name.c_str());
}

// BatchNorm <prefix>.{weight,bias,running_mean,running_var} folded into w
// (c x per) and b.
bool fold(struct pth_file *pf, const std::string &prefix, int c, long per, std::vector<float> &w,
          std::vector<float> &b)
{
    long s[1] = {c};
    std::vector<float> g = read_host(pf, prefix + ".weight", 1, s);
    std::vector<float> bt = read_host(pf, prefix + ".bias", 1, s);
    std::vector<float> mu = read_host(pf, prefix + ".running_mean", 1, s);
    std::vector<float> var = read_host(pf, prefix + ".running_var", 1, s);
    if (g.empty() || bt.empty() || mu.empty() || var.empty() || w.empty())
        return false;
    ops_fold_bn(w.data(), b.data(), c, per, g.data(), bt.data(), mu.data(), var.data(), EPS_BN);
    return true;
}

// RepVGG block l: conv1 (3 x 3) + conv2 (1 x 1) + identity, each with its
// BatchNorm, folded into one 3 x 3 convolution with bias (eloftr.c:110-162).
bool load_block(struct eloftr_model *m, struct pth_file *pf, int l, int stage, int blk)
{
    eloftr_impl *I = m->impl;
    const int ci = I->bcin[l], co = I->bcout[l];
    long s3[4] = {co, ci, 3, 3}, s1[4] = {co, ci, 1, 1};
    const std::string pre = "efficientloftr.backbone.stages." + std::to_string(stage) +
                            ".blocks." + std::to_string(blk);
    std::vector<float> w = read_host(pf, pre + ".conv1.conv.weight", 4, s3), b(co, 0.0f);
    if (!fold(pf, pre + ".conv1.norm", co, (long)ci * 9, w, b))
        return false;
    std::vector<float> w1 = read_host(pf, pre + ".conv2.conv.weight", 4, s1), b1(co, 0.0f);
    if (!fold(pf, pre + ".conv2.norm", co, ci, w1, b1))
        return false;
    for (int k = 0; k < co; k++) {
        for (int c = 0; c < ci; c++)
            w[((size_t)k * ci + c) * 9 + 4] += w1[(size_t)k * ci + c];
        b[k] += b1[k];
    }
    const bool ident = pth_find(pf, (pre + ".identity.weight").c_str()) != nullptr;
    if (ident) {
        if (ci != co || I->bstride[l] != 1) {
            fail("ELoFTR: unexpected identity branch in <%s>", pre.c_str());
            return false;
        }
        std::vector<float> wi((size_t)co * ci, 0.0f), bi(co, 0.0f);
        for (int k = 0; k < co; k++)
            wi[(size_t)k * ci + k] = 1.0f;
        if (!fold(pf, pre + ".identity", co, ci, wi, bi))
            return false;
        for (int k = 0; k < co; k++) {
            for (int c = 0; c < ci; c++)
                w[((size_t)k * ci + c) * 9 + 4] += wi[(size_t)k * ci + c];
            b[k] += bi[k];
        }
    }
    else if (ci == co && I->bstride[l] == 1) {
        fail("ELoFTR: identity branch missing in <%s>", pre.c_str());
        return false;
    }
    I->bw[l] = upload(m, w, "backbone weight");
    I->bb[l] = upload(m, b, "backbone bias");
    return !pending();
}

void load_attn(struct eloftr_model *m, struct pth_file *pf, int layer, const char *kind, Attn *a)
{
    const std::string pre = "efficientloftr.local_feature_transformer.layers." +
                            std::to_string(layer) + "." + kind + ".";
    long qa[4] = {ELOFTR_DIM, 1, 4, 4}, sq[2] = {ELOFTR_DIM, ELOFTR_DIM};
    long s1[2] = {MLP, 2 * ELOFTR_DIM}, s2[2] = {ELOFTR_DIM, MLP}, v1[1] = {ELOFTR_DIM};
    a->q_agg = load_dev(m, pf, pre + "aggregation.q_aggregation.weight", 4, qa);
    a->norm_g = load_dev(m, pf, pre + "aggregation.norm.weight", 1, v1);
    a->norm_b = load_dev(m, pf, pre + "aggregation.norm.bias", 1, v1);
    a->wq = load_dev(m, pf, pre + "attention.q_proj.weight", 2, sq);
    a->wk = load_dev(m, pf, pre + "attention.k_proj.weight", 2, sq);
    a->wv = load_dev(m, pf, pre + "attention.v_proj.weight", 2, sq);
    a->wo = load_dev(m, pf, pre + "attention.o_proj.weight", 2, sq);
    a->fc1 = load_dev(m, pf, pre + "mlp.fc1.weight", 2, s1);
    a->fc2 = load_dev(m, pf, pre + "mlp.fc2.weight", 2, s2);
    a->mlp_g = load_dev(m, pf, pre + "mlp.layer_norm.weight", 1, v1);
    a->mlp_b = load_dev(m, pf, pre + "mlp.layer_norm.bias", 1, v1);
}

// Fine fusion (eloftr.c:192-230): out_conv with the coarse features' 1 /
// sqrt(256) folded in, then per block out_conv1 (1 x 1), out_conv2 (3 x 3,
// BatchNorm folded) and out_conv3 (3 x 3).
void load_fusion(struct eloftr_model *m, struct pth_file *pf)
{
    eloftr_impl *I = m->impl;
    const int dims[3] = {256, 128, 64};
    long so[4] = {256, 256, 1, 1};
    std::vector<float> w = read_host(pf, "refinement_layer.out_conv.weight", 4, so);
    for (float &v : w)
        v /= 16.0f;
    I->f_out = upload(m, w, "out_conv");
    for (int i = 0; i < 2; i++) {
        const int hid = dims[i + 1], inter = dims[i];
        long s1[4] = {inter, hid, 1, 1}, s2[4] = {inter, inter, 3, 3}, s3[4] = {hid, inter, 3, 3};
        const std::string pre = "refinement_layer.out_conv_layers." + std::to_string(i) + ".";
        I->f1_w[i] = load_dev(m, pf, pre + "out_conv1.weight", 4, s1);
        std::vector<float> w2 = read_host(pf, pre + "out_conv2.weight", 4, s2), b2(inter, 0.0f);
        if (!fold(pf, pre + "batch_norm", inter, (long)inter * 9, w2, b2))
            return;
        I->f2_w[i] = upload(m, w2, "out_conv2");
        I->f2_b[i] = upload(m, b2, "out_conv2 bias");
        I->f3_w[i] = load_dev(m, pf, pre + "out_conv3.weight", 4, s3);
    }
}

cl_mem walloc(struct eloftr_model *m, size_t floats, const char *what)
{
    return ocl_alloc(m->ocl, floats * 4, what);
}

// RoPE angles of the aggregated grid (eloftr.c:262-291): position (i, j),
// 1-based, times pos_scale; pair p of the 256 channels: i f(p / 2) for even
// p, j f(p / 2) for odd p, f(k) = base^(-2k / ROPE_DIM); (cos, sin) pairs.
cl_mem rope_table(struct eloftr_model *m)
{
    const int np = ELOFTR_DIM / 2;
    std::vector<float> t((size_t)m->ah * m->aw * np * 2);
    for (int i = 0; i < m->ah; i++)
        for (int j = 0; j < m->aw; j++)
            for (int p = 0; p < np; p++) {
                const float f = (float)(1.0 / pow(ROPE_BASE, (double)(2 * (p / 2)) / ROPE_DIM));
                const float a = (p % 2 ? (float)(j + 1) : (float)(i + 1)) * m->pos_scale * f;
                float *q = &t[(((size_t)i * m->aw + j) * np + p) * 2];
                q[0] = cosf(a);
                q[1] = sinf(a);
            }
    return upload(m, t, "rope");
}

// --------------------------------------------------------- coarse matching

// Log-sum-exp of each row of a block S (R x N): one block of 256 per row,
// into lse[r0 + r] (eloftr_kernels.cl:12-43).
__global__ void __launch_bounds__(256) row_lse_k(const float *S, int N, int r0, float *lse)
{
    __shared__ float red[32];
    const float *s = S + (long)blockIdx.x * N;
    float m = -INFINITY;
    for (int j = threadIdx.x; j < N; j += 256)
        m = fmaxf(m, s[j]);
    m = block_max(m, red);
    float sum = 0.0f;
    for (int j = threadIdx.x; j < N; j += 256)
        sum += expf(s[j] - m);
    sum = block_sum(sum, red);
    if (threadIdx.x == 0)
        lse[r0 + blockIdx.x] = m + logf(sum);
}

// Running column maximum and sum of exponentials, merging this block's R
// rows (eloftr_kernels.cl:47-64).
__global__ void col_lse_k(const float *S, int R, int N, float *cm, float *cs)
{
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= N)
        return;
    float m = -INFINITY, s = 0.0f;
    for (int r = 0; r < R; r++)
        m = fmaxf(m, S[(long)r * N + j]);
    for (int r = 0; r < R; r++)
        s += expf(S[(long)r * N + j] - m);
    const float mo = cm[j], mn = fmaxf(mo, m);
    cs[j] = (mo == -INFINITY ? 0.0f : cs[j] * expf(mo - mn)) + s * expf(m - mn);
    cm[j] = mn;
}

// Dual-softmax confidence of one score (eloftr_kernels.cl:67-70).
__device__ __forceinline__ float dual_conf(float s, float lr, float cm, float cs)
{
    return expf(s - lr) * expf(s - (cm + logf(cs)));
}

// Row maximum and first argmax of the confidence, one block per row of the
// block (eloftr_kernels.cl:74-108).
__global__ void __launch_bounds__(256)
conf_row_k(const float *S, int N, int r0, const float *lse, const float *cm, const float *cs,
           float *rmax, int *rarg)
{
    __shared__ float vm[256];
    __shared__ int vi[256];
    const int l = threadIdx.x;
    const float *s = S + (long)blockIdx.x * N;
    const float lr = lse[r0 + blockIdx.x];
    float best = -1.0f;
    int bi = 0;
    for (int j = l; j < N; j += 256) {
        const float c = dual_conf(s[j], lr, cm[j], cs[j]);
        if (c > best) {
            best = c;
            bi = j;
        }
    }
    vm[l] = best;
    vi[l] = bi;
    __syncthreads();
    for (int h = 128; h > 0; h >>= 1) {
        if (l < h && (vm[l + h] > vm[l] || (vm[l + h] == vm[l] && vi[l + h] < vi[l]))) {
            vm[l] = vm[l + h];
            vi[l] = vi[l + h];
        }
        __syncthreads();
    }
    if (l == 0) {
        rmax[r0 + blockIdx.x] = vm[0];
        rarg[r0 + blockIdx.x] = vi[0];
    }
}

// Running column maximum and first argmax of the confidence over blocks of
// rows in increasing order (eloftr_kernels.cl:112-140).
__global__ void conf_col_k(const float *S, int R, int N, int r0, const float *lse,
                           const float *cm, const float *cs, float *cmax, int *carg)
{
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= N)
        return;
    float best = cmax[j];
    int bi = carg[j];
    const float m = cm[j], sm = cs[j];
    for (int r = 0; r < R; r++) {
        const float c = dual_conf(S[(long)r * N + j], lse[r0 + r], m, sm);
        if (c > best) {
            best = c;
            bi = r0 + r;
        }
    }
    cmax[j] = best;
    carg[j] = bi;
}

__global__ void fill_f_k(float *p, long n, float v)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < n)
        p[e] = v;
}

__global__ void fill_i_k(int *p, long n, int v)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e < n)
        p[e] = v;
}

// ----------------------------------------------------------- fine matching

constexpr int FW = 8, FW1 = FW + 2, FC = 64, FS = 8, NP = FW * FW, NQ = FW1 * FW1;
constexpr int F1C = FC - FS;  // first-stage channels

// Both fine stages for one coarse match per block of 256
// (eloftr_kernels.cl:146-295): the 8 x 8 window of image 0 at cell (x0, y0)
// against the 10 x 10 window of image 1 around cell (x1, y1); scores on the
// first 56 channels / 64; dual softmax; argmax over positions p of image 0
// and the inner 8 x 8 of image 1 (flattened p * 64 + i * 8 + j, first
// index on ties); the 3 x 3 scores on the last 8 channels / sqrt(8) / T
// around the chosen 10 x 10 index (-1 wrapping to 9, as the network was
// trained), softmax, expectation. The windows are staged in shared memory.
// Output per match: x0, y0, x1, y1 in the reference's convention.
struct FineSmem {
    float a[NP][F1C + 1];
    float b[NQ][F1C + 1];
    float sc[NP * NQ];
    float pm[NQ], ps[NQ], qm[NP], qs[NP];
    float vm[256];
    int vi[256];
    float s2[9];
};

__device__ __forceinline__ float fine_at(const float *f, int H, int W, int c, int x, int y)
{
    return x < 0 || y < 0 || x >= W || y >= H ? 0.0f : f[((long)c * H + y) * W + x];
}

__global__ void __launch_bounds__(256)
fine_k(const float *f0, const float *f1, int H, int W, const int4 *cells, int M, float T,
       float4 *out)
{
    extern __shared__ float fine_smem[];
    FineSmem &s = *reinterpret_cast<FineSmem *>(fine_smem);
    const int k = blockIdx.x, l = threadIdx.x;
    if (k >= M)
        return;
    const int4 cl = cells[k];
    for (int e = l; e < NP * F1C; e += 256) {
        const int c = e / NP, p = e % NP;
        s.a[p][c] = fine_at(f0, H, W, c, cl.x * FW + p % FW, cl.y * FW + p / FW);
    }
    for (int e = l; e < NQ * F1C; e += 256) {
        const int c = e / NQ, q = e % NQ;
        s.b[q][c] = fine_at(f1, H, W, c, cl.z * FW - 1 + q % FW1, cl.w * FW - 1 + q / FW1);
    }
    __syncthreads();
    for (int e = l; e < NP * NQ; e += 256) {
        const int p = e / NQ, q = e % NQ;
        float d = 0.0f;
#pragma unroll 8
        for (int c = 0; c < F1C; c++)
            d = fmaf(s.a[p][c], s.b[q][c], d);
        s.sc[e] = d * (1.0f / FC);
    }
    __syncthreads();
    for (int q = l; q < NQ; q += 256) {
        float m = -INFINITY, t = 0.0f;
        for (int p = 0; p < NP; p++)
            m = fmaxf(m, s.sc[p * NQ + q]);
        for (int p = 0; p < NP; p++)
            t += expf(s.sc[p * NQ + q] - m);
        s.pm[q] = m;
        s.ps[q] = t;
    }
    for (int p = l; p < NP; p += 256) {
        float m = -INFINITY, t = 0.0f;
        for (int q = 0; q < NQ; q++)
            m = fmaxf(m, s.sc[p * NQ + q]);
        for (int q = 0; q < NQ; q++)
            t += expf(s.sc[p * NQ + q] - m);
        s.qm[p] = m;
        s.qs[p] = t;
    }
    __syncthreads();
    float best = -1.0f;
    int bi = 0;
    for (int e = l; e < NP * FW * FW; e += 256) {
        const int pp = e / (FW * FW), ii = (e / FW) % FW, jj = e % FW;
        const int qq = (ii + 1) * FW1 + jj + 1;
        const float sv = s.sc[pp * NQ + qq];
        const float v = expf(sv - s.pm[qq]) / s.ps[qq] * (expf(sv - s.qm[pp]) / s.qs[pp]);
        if (v > best) {
            best = v;
            bi = e;
        }
    }
    s.vm[l] = best;
    s.vi[l] = bi;
    __syncthreads();
    for (int h = 128; h > 0; h >>= 1) {
        if (l < h && (s.vm[l + h] > s.vm[l] || (s.vm[l + h] == s.vm[l] && s.vi[l + h] < s.vi[l]))) {
            s.vm[l] = s.vm[l + h];
            s.vi[l] = s.vi[l + h];
        }
        __syncthreads();
    }
    const int bp = s.vi[0] / (FW * FW), bq = s.vi[0] % (FW * FW);
    const int qi = bq / FW, qj = bq % FW;
    if (l < 9) {
        const int ii = (qi + l / 3 - 1 + FW1) % FW1, jj = (qj + l % 3 - 1 + FW1) % FW1;
        const int ax = cl.x * FW + bp % FW, ay = cl.y * FW + bp / FW;
        const int bx = cl.z * FW - 1 + jj, by = cl.w * FW - 1 + ii;
        float d = 0.0f;
        for (int c = FC - FS; c < FC; c++)
            d = fmaf(fine_at(f0, H, W, c, ax, ay), fine_at(f1, H, W, c, bx, by), d);
        s.s2[l] = d * rsqrtf((float)FS) / T;
    }
    __syncthreads();
    if (l == 0) {
        float m = -INFINITY, t = 0.0f, ex = 0.0f, ey = 0.0f;
        for (int i = 0; i < 9; i++)
            m = fmaxf(m, s.s2[i]);
        for (int i = 0; i < 9; i++)
            t += expf(s.s2[i] - m);
        for (int i = 0; i < 9; i++) {
            const float w = expf(s.s2[i] - m) / t;
            ex += w * (i % 3 - 1);
            ey += w * (i / 3 - 1);
        }
        const float off = FW / 2 - 0.5f;
        out[k] = make_float4(cl.x * FW + bp % FW - off, cl.y * FW + bp / FW - off,
                             cl.z * FW + qj - off + ex, cl.w * FW + qi - off + ey);
    }
}

// ----------------------------------------------------------------- forward

void conv3x3(struct eloftr_model *m, cl_mem in, int C, int H, int W, cl_mem w, cl_mem b, int K,
             int stride, int act, cl_mem out)
{
    struct conv_geom g = ops_geom(3, stride, 1);
    ops_conv2d(m->ops, in, C, H, W, w, b, K, &g, nullptr, nullptr, nullptr, act, LEAKY, out);
}

// The RepVGG backbone on img (1 x H x W) of image k (eloftr.c:369-394).
void backbone(struct eloftr_model *m, int k)
{
    eloftr_impl *I = m->impl;
    cl_mem in = I->img;
    int Hc = m->H, Wc = m->W;
    for (int s = 0, l = 0; s < 4; s++)
        for (int b = 0; b < stage_blocks[s]; b++, l++) {
            const int st = I->bstride[l];
            const bool last = b == stage_blocks[s] - 1;
            cl_mem out = last && s == 1   ? I->f1[k]
                         : last && s == 2 ? I->f2[k]
                         : last && s == 3 ? I->x[k]
                                          : (in == I->s_a ? I->s_b : I->s_a);
            conv3x3(m, in, I->bcin[l], Hc, Wc, I->bw[l], I->bb[l], I->bcout[l], st, ACT_RELU, out);
            Hc /= st;
            Wc /= st;
            in = out;
        }
}

void dcopy(struct eloftr_model *m, cl_mem src, cl_mem dst, size_t floats)
{
    cuda_ok(cudaMemcpyAsync(dst->ptr, src->ptr, floats * 4, cudaMemcpyDeviceToDevice,
                            stream_of(m->ocl)),
            "ELoFTR copy");
}

// One aggregated attention block: X (256 x h x w) attends to Y, X updated
// in place (eloftr.c:407-449).
void agg_attn(struct eloftr_model *m, const Attn &a, cl_mem X, cl_mem Y, bool use_rope)
{
    eloftr_impl *I = m->impl;
    struct ops *o = m->ops;
    struct conv_geom g = {4, 4, 4, 4, 0, 0, 1, 1, ELOFTR_DIM};
    const int D = ELOFTR_DIM, n = m->h * m->w, na = m->ah * m->aw, hd = D / HEADS;
    ops_conv2d(o, X, D, m->h, m->w, a.q_agg, nullptr, D, &g, nullptr, nullptr, nullptr,
               ACT_NONE, 0.0f, I->t_q);
    ops_pool2d(o, Y, D, m->h, m->w, 4, 4, 0, 1, I->t_kv);
    ops_transpose(o, I->t_q, I->t_qn, 1, D, na);
    ops_transpose(o, I->t_kv, I->t_kvn, 1, D, na);
    ops_layernorm(o, na, D, I->t_qn, I->t_qn, a.norm_g, a.norm_b, EPS_LN, ACT_NONE, 0.0f);
    ops_layernorm(o, na, D, I->t_kvn, I->t_kvn, a.norm_g, a.norm_b, EPS_LN, ACT_NONE, 0.0f);
    ops_linear(o, na, D, D, I->t_qn, 0, a.wq, nullptr, I->t_Q, 0, ACT_NONE, 0.0f, 0);
    ops_linear(o, na, D, D, I->t_kvn, 0, a.wk, nullptr, I->t_K, 0, ACT_NONE, 0.0f, 0);
    ops_linear(o, na, D, D, I->t_kvn, 0, a.wv, nullptr, I->t_V, 0, ACT_NONE, 0.0f, 0);
    if (use_rope) {
        ops_rope(o, I->t_Q, 0, D, na, 1, D, na, I->rope, 1);
        ops_rope(o, I->t_K, 0, D, na, 1, D, na, I->rope, 1);
    }
    ops_attention(o, ops_mat(I->t_Q, 0, D), ops_mat(I->t_K, 0, D), ops_mat(I->t_V, 0, D),
                  ops_mat(I->t_O, 0, D), na, na, HEADS, hd, 1.0f / sqrtf((float)hd), nullptr);
    ops_linear(o, na, D, D, I->t_O, 0, a.wo, nullptr, I->t_Q, 0, ACT_NONE, 0.0f, 0);
    ops_transpose(o, I->t_Q, I->t_O2, 1, na, D);
    dcopy(m, X, I->t_cat, (size_t)D * n);
    ops_resize(o, I->t_O2, D, m->ah, m->aw, I->t_cat, m->h, m->w, D, 0, 4.0f);
    ops_transpose(o, I->t_cat, I->t_tok, 1, 2 * D, n);
    ops_linear(o, n, 2 * D, MLP, I->t_tok, 0, a.fc1, nullptr, I->t_h1, 0, ACT_LEAKY, LEAKY, 0);
    ops_linear(o, n, MLP, D, I->t_h1, 0, a.fc2, nullptr, I->t_h2, 0, ACT_NONE, 0.0f, 0);
    ops_layernorm(o, n, D, I->t_h2, I->t_h2, a.mlp_g, a.mlp_b, EPS_LN, ACT_NONE, 0.0f);
    ops_transpose(o, I->t_h2, I->t_cat, 1, n, D);
    ops_axpby(o, X, X, 1.0f, I->t_cat, 1.0f, (long)D * n, (long)D * n);
}

// Coarse dual-softmax matching by blocks of rows, then mutual maxima above
// the threshold away from the border (eloftr.c:473-571).
void coarse_match(struct eloftr_model *m)
{
    eloftr_impl *I = m->impl;
    struct ops *o = m->ops;
    cudaStream_t st = stream_of(m->ocl);
    const int D = ELOFTR_DIM, n = m->h * m->w, R = I->blk_rows;
    const float alpha = 1.0f / (D * COARSE_T);
    ops_transpose(o, I->x[0], I->t_tok, 1, D, n);
    ops_transpose(o, I->x[1], I->t_h1, 1, D, n);
    fill_f_k<<<cdiv(n, 256), 256, 0, st>>>((float *)I->col_m->ptr, n, -INFINITY);
    fill_f_k<<<cdiv(n, 256), 256, 0, st>>>((float *)I->col_s->ptr, n, 0.0f);
    fill_f_k<<<cdiv(n, 256), 256, 0, st>>>((float *)I->col_max->ptr, n, -1.0f);
    fill_i_k<<<cdiv(n, 256), 256, 0, st>>>((int *)I->col_arg->ptr, n, -1);
    // The scores in the context's precision: float32 contexts give the
    // reference's match indices exactly; bfloat16 contexts take the score
    // product on the tensor cores (bfloat16 features, float32 sums), which
    // can only move matches whose confidence or mutual test is a near-tie.
    for (int pass = 0; pass < 2; pass++)
        for (int r0 = 0; r0 < n; r0 += R) {
            const int rows = n - r0 < R ? n - r0 : R;
            ops_gemm(o, rows, n, D, ops_mat(I->t_tok, (long)r0 * D, D), ops_mat(I->t_h1, 0, D), 1,
                     ops_mat(I->s_blk, 0, n), 1, 1, nullptr, 0, nullptr, 0, alpha, ACT_NONE, 0.0f);
            const float *S = (const float *)I->s_blk->ptr;
            float *lse = (float *)I->row_lse->ptr, *cm = (float *)I->col_m->ptr,
                  *cs = (float *)I->col_s->ptr;
            if (pass == 0) {
                row_lse_k<<<rows, 256, 0, st>>>(S, n, r0, lse);
                col_lse_k<<<cdiv(n, 128), 128, 0, st>>>(S, rows, n, cm, cs);
            }
            else {
                conf_row_k<<<rows, 256, 0, st>>>(S, n, r0, lse, cm, cs, (float *)I->row_max->ptr,
                                                 (int *)I->row_arg->ptr);
                conf_col_k<<<cdiv(n, 128), 128, 0, st>>>(S, rows, n, r0, lse, cm, cs,
                                                         (float *)I->col_max->ptr,
                                                         (int *)I->col_arg->ptr);
            }
        }
    if (!launch_ok("eloftr coarse matching"))
        return;
    std::vector<float> rmax(n);
    std::vector<int> rarg(n), carg(n);
    ocl_read(m->ocl, I->row_max, 0, rmax.data(), (size_t)n * 4);
    ocl_read(m->ocl, I->row_arg, 0, rarg.data(), (size_t)n * 4);
    ocl_read(m->ocl, I->col_arg, 0, carg.data(), (size_t)n * 4);
    m->nm = 0;
    if (pending())
        return;
    for (int i = 0; i < n; i++) {
        const int j = rarg[i];
        const int xi = i % m->w, yi = i / m->w, xj = j % m->w, yj = j / m->w;
        if (!(rmax[i] > COARSE_THR) || carg[j] != i)
            continue;
        if (xi < BORDER || yi < BORDER || xi >= m->w - BORDER || yi >= m->h - BORDER ||
            xj < BORDER || yj < BORDER || xj >= m->w - BORDER || yj >= m->h - BORDER)
            continue;
        m->mi[m->nm] = i;
        m->mj[m->nm] = j;
        m->mconf[m->nm++] = rmax[i];
    }
}

// Fine fusion of image k into fine[k] (eloftr.c:575-604).
void fusion(struct eloftr_model *m, int k)
{
    eloftr_impl *I = m->impl;
    struct ops *o = m->ops;
    const int h = m->h, w = m->w, H4 = 2 * h, W4 = 2 * w, H2 = 4 * h, W2 = 4 * w;
    ops_conv1x1(o, I->x[k], 0, 256, h * w, I->f_out, nullptr, 256, I->fu_a, 0, ACT_NONE, 0.0f);
    ops_resize(o, I->fu_a, 256, h, w, I->fu_b, H4, W4, 0, 0, 2.0f);
    ops_conv1x1(o, I->f2[k], 0, 128, H4 * W4, I->f1_w[0], nullptr, 256, I->fu_c, 0, ACT_NONE,
                0.0f);
    ops_axpby(o, I->fu_c, I->fu_c, 1.0f, I->fu_b, 1.0f, 256L * H4 * W4, 256L * H4 * W4);
    conv3x3(m, I->fu_c, 256, H4, W4, I->f2_w[0], I->f2_b[0], 256, 1, ACT_LEAKY, I->fu_a);
    conv3x3(m, I->fu_a, 256, H4, W4, I->f3_w[0], nullptr, 128, 1, ACT_NONE, I->fu_b);
    ops_resize(o, I->fu_b, 128, H4, W4, I->fu_c, H2, W2, 0, 0, 2.0f);
    ops_conv1x1(o, I->f1[k], 0, 64, H2 * W2, I->f1_w[1], nullptr, 128, I->fu_a, 0, ACT_NONE,
                0.0f);
    ops_axpby(o, I->fu_a, I->fu_a, 1.0f, I->fu_c, 1.0f, 128L * H2 * W2, 128L * H2 * W2);
    conv3x3(m, I->fu_a, 128, H2, W2, I->f2_w[1], I->f2_b[1], 128, 1, ACT_LEAKY, I->fu_b);
    conv3x3(m, I->fu_b, 128, H2, W2, I->f3_w[1], nullptr, 64, 1, ACT_NONE, I->fu_c);
    ops_resize(o, I->fu_c, 64, H2, W2, I->fine[k], m->H, m->W, 0, 0, 2.0f);
}

void fine_match(struct eloftr_model *m)
{
    eloftr_impl *I = m->impl;
    if (m->nm == 0)
        return;
    std::vector<int> cells((size_t)m->nm * 4);
    for (int i = 0; i < m->nm; i++) {
        cells[4 * i] = m->mi[i] % m->w;
        cells[4 * i + 1] = m->mi[i] / m->w;
        cells[4 * i + 2] = m->mj[i] % m->w;
        cells[4 * i + 3] = m->mj[i] / m->w;
    }
    ocl_write(m->ocl, I->m_idx, 0, cells.data(), cells.size() * 4);
    fine_k<<<m->nm, 256, sizeof(FineSmem), stream_of(m->ocl)>>>(
        (const float *)I->fine[0]->ptr, (const float *)I->fine[1]->ptr, m->H, m->W,
        (const int4 *)I->m_idx->ptr, m->nm, FINE_T, (float4 *)I->m_out->ptr);
    if (launch_ok("eloftr fine matching"))
        ocl_read(m->ocl, I->m_out, 0, m->kp, (size_t)m->nm * 4 * 4);
}

void dump_dev(struct eloftr_model *m, const char *dir, int tile, const char *what, cl_mem b,
              size_t floats)
{
    std::vector<float> v(floats);
    ocl_read(m->ocl, b, 0, v.data(), floats * 4);
    if (pending())
        return;
    char path[4096];
    snprintf(path, sizeof(path), "%s/tile%03d_eloftr_%s.f32", dir, tile, what);
    FILE *fp = fopen(path, "wb");
    if (!fp || fwrite(v.data(), 4, floats, fp) != floats)
        fail("Unable to write debug dump <%s>", path);
    if (fp)
        fclose(fp);
}

}  // namespace

extern "C" void eloftr_load(struct eloftr_model *m, struct ops *ops, struct pth_file *pf)
{
    memset(m, 0, sizeof(*m));
    if (pending())
        return;
    m->ops = ops;
    m->ocl = ops->ocl;
    m->pos_scale = 1.0f;
    m->impl = new eloftr_impl();
    eloftr_impl *I = m->impl;
    cudaSetDevice(m->ocl->device);
    for (int s = 0, l = 0, cin = 1; s < 4; s++)
        for (int b = 0; b < stage_blocks[s]; b++, l++) {
            I->bcin[l] = cin;
            I->bcout[l] = stage_out[s];
            I->bstride[l] = b == 0 ? stage_stride[s] : 1;
            if (!load_block(m, pf, l, s, b))
                return;
            cin = stage_out[s];
        }
    for (int i = 0; i < ELOFTR_LAYERS; i++) {
        load_attn(m, pf, i, "self_attention", &I->self_attn[i]);
        load_attn(m, pf, i, "cross_attention", &I->cross_attn[i]);
    }
    load_fusion(m, pf);
    static unsigned opted = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(opted >> (dev & 31) & 1)) {
        if (!cuda_ok(cudaFuncSetAttribute(fine_k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)sizeof(FineSmem)),
                     "eloftr fine kernel"))
            return;
        opted |= 1u << (dev & 31);
    }
}

extern "C" void eloftr_alloc(struct eloftr_model *m, int H, int W)
{
    if (pending())
        return;
    if (!m->impl) {
        fail("ELoFTR: eloftr_alloc before eloftr_load");
        return;
    }
    if (H <= 0 || W <= 0 || H % ELOFTR_MULTIPLE || W % ELOFTR_MULTIPLE) {
        fail("ELoFTR tile %d x %d is not a multiple of %d", H, W, ELOFTR_MULTIPLE);
        return;
    }
    eloftr_impl *I = m->impl;
    cudaSetDevice(m->ocl->device);
    const size_t hw = (size_t)H * W;
    m->H = H;
    m->W = W;
    m->h = H / 8;
    m->w = W / 8;
    m->ah = m->h / 4;
    m->aw = m->w / 4;
    const size_t n = (size_t)m->h * m->w, na = (size_t)m->ah * m->aw;
    I->img = walloc(m, hw, "image");
    I->s_a = walloc(m, 16 * hw, "backbone");
    I->s_b = walloc(m, 16 * hw, "backbone");
    for (int k = 0; k < 2; k++) {
        I->f1[k] = walloc(m, 16 * hw, "1/2 features");
        I->f2[k] = walloc(m, 8 * hw, "1/4 features");
        I->x[k] = walloc(m, ELOFTR_DIM * n, "1/8 features");
        I->fine[k] = walloc(m, ELOFTR_FINE_DIM * hw, "fine features");
    }
    I->t_q = walloc(m, ELOFTR_DIM * na, "aggregated");
    I->t_kv = walloc(m, ELOFTR_DIM * na, "aggregated");
    I->t_qn = walloc(m, ELOFTR_DIM * na, "tokens");
    I->t_kvn = walloc(m, ELOFTR_DIM * na, "tokens");
    I->t_Q = walloc(m, ELOFTR_DIM * na, "queries");
    I->t_K = walloc(m, ELOFTR_DIM * na, "keys");
    I->t_V = walloc(m, ELOFTR_DIM * na, "values");
    I->t_O = walloc(m, ELOFTR_DIM * na, "attention");
    I->t_O2 = walloc(m, ELOFTR_DIM * na, "attention");
    I->t_cat = walloc(m, 2 * ELOFTR_DIM * n, "concatenation");
    I->t_tok = walloc(m, 2 * ELOFTR_DIM * n, "tokens");
    I->t_h1 = walloc(m, MLP * n, "mlp");
    I->t_h2 = walloc(m, ELOFTR_DIM * n, "mlp");
    I->rope = rope_table(m);
    // Score blocks of at most 64 Mi floats.
    I->blk_rows = (int)std::max<size_t>(1, std::min<size_t>(n, (size_t)64 * 1048576 / n));
    I->s_blk = walloc(m, (size_t)I->blk_rows * n, "scores");
    I->row_lse = walloc(m, n, "row lse");
    I->col_m = walloc(m, n, "column max");
    I->col_s = walloc(m, n, "column sum");
    I->row_max = walloc(m, n, "row max");
    I->col_max = walloc(m, n, "column max");
    I->row_arg = walloc(m, n, "row argmax");
    I->col_arg = walloc(m, n, "column argmax");
    I->fu_a = walloc(m, 32 * hw, "fusion");
    I->fu_b = walloc(m, 32 * hw, "fusion");
    I->fu_c = walloc(m, 32 * hw, "fusion");
    m->nmax = (int)n;
    I->m_idx = walloc(m, n * 4, "match cells");
    I->m_out = walloc(m, n * 4, "fine matches");
    m->mi = (int *)calloc(n, sizeof(int));
    m->mj = (int *)calloc(n, sizeof(int));
    m->mconf = (float *)calloc(n, sizeof(float));
    m->kp = (float *)calloc(n * 4, sizeof(float));
}

extern "C" void eloftr_match(struct eloftr_model *m, const float *grey0, const float *grey1,
                             const char *dump, int tile)
{
    if (pending())
        return;
    if (!m->impl || !m->impl->img) {
        fail("ELoFTR: eloftr_match before eloftr_alloc");
        return;
    }
    eloftr_impl *I = m->impl;
    cudaSetDevice(m->ocl->device);
    const size_t n = (size_t)m->h * m->w, hw = (size_t)m->H * m->W;
    const bool d = dump && *dump;
    m->nm = 0;
    for (int k = 0; k < 2; k++) {
        ocl_write(m->ocl, I->img, 0, k ? grey1 : grey0, hw * 4);
        backbone(m, k);
    }
    if (d) {
        dump_dev(m, dump, tile, "backbone_0", I->x[0], ELOFTR_DIM * n);
        dump_dev(m, dump, tile, "backbone_1", I->x[1], ELOFTR_DIM * n);
    }
    for (int l = 0; l < ELOFTR_LAYERS; l++) {
        agg_attn(m, I->self_attn[l], I->x[0], I->x[0], true);
        agg_attn(m, I->self_attn[l], I->x[1], I->x[1], true);
        // As the reference: image 1 attends to image 0's features already
        // updated by this layer's cross attention.
        agg_attn(m, I->cross_attn[l], I->x[0], I->x[1], false);
        agg_attn(m, I->cross_attn[l], I->x[1], I->x[0], false);
    }
    if (d) {
        dump_dev(m, dump, tile, "coarse_0", I->x[0], ELOFTR_DIM * n);
        dump_dev(m, dump, tile, "coarse_1", I->x[1], ELOFTR_DIM * n);
    }
    coarse_match(m);
    for (int k = 0; k < 2; k++)
        fusion(m, k);
    if (d) {
        dump_dev(m, dump, tile, "fine_0", I->fine[0], ELOFTR_FINE_DIM * hw);
        dump_dev(m, dump, tile, "fine_1", I->fine[1], ELOFTR_FINE_DIM * hw);
    }
    fine_match(m);
    launch_ok("eloftr_match");
}

extern "C" void eloftr_free(struct eloftr_model *m)
{
    if (m->impl) {
        for (cl_mem *p : m->impl->all())
            ocl_release(p);
        delete m->impl;
    }
    free(m->mi);
    free(m->mj);
    free(m->mconf);
    free(m->kp);
    memset(m, 0, sizeof(*m));
}
