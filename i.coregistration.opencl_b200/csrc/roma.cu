// SPDX-License-Identifier: Unlicense
//
// RoMa's device stage (roma.h) on a B200: weight loading and folding,
// work buffers, and the per-tile sequence of the reference's roma_match
// (roma.c:1357-1435), every step on the device.
//
// Layouts: feature maps are token-major (cells x channels, channels
// contiguous), so that every 1 x 1 convolution and linear layer is a GEMM
// whose operands are both K-major and every 3 x 3 convolution an implicit
// GEMM over the channels-last map; warps, certainties and confidences are
// planar (k, n) as the reference's. Precision: with OPS_FP32 all
// arithmetic is float32 (the reference's); with OPS_BF16 the matrix
// products take bfloat16 operands (weights converted at load, activations
// written in bfloat16 by their producers) with float32 accumulation,
// while the residual streams, the Gaussian process, the anchor logits and
// the warps stay float32.

#include <math.h>
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>
#include <string>
#include <vector>

#include "roma.h"
#include "roma_kernels.cuh"

using namespace coreg;

namespace {

const float EPS_BN = 1e-5f;
const float EPS_LN_VIT = 1e-6f;
const float EPS_LN_DEC = 1e-5f;
const int VIT_HEADS = 16, DEC_HEADS = 8, MLP_RATIO = 4, GP_DIM = 512;
const float GP_T = 0.2f, COS_EPS = 1e-6f;
const double GP_NOISE = 0.1;
const int VIT_GRID = 37;
const int NCLS = ROMA_CLS_RES * ROMA_CLS_RES;

// roma_model() of the outdoor model (roma.c:60-64).
const int ref_scale[ROMA_SCALES] = {16, 8, 4, 2, 1};
const int ref_feat[ROMA_SCALES] = {512, 512, 256, 64, 9};
const int ref_emb[ROMA_SCALES] = {128, 64, 32, 16, 6};
const int ref_radius[ROMA_SCALES] = {7, 3, 2, 0, 0};
const int proj_in_ch[ROMA_SCALES] = {1024, 512, 256, 128, 64};
// RoMa v2's refiners (roma.c:454-458).
const int ref2_scale[ROMA2_SCALES] = {4, 2, 1};
const int ref2_in[ROMA2_SCALES] = {256, 128, 64};
const int ref2_feat[ROMA2_SCALES] = {192, 48, 12};
const int ref2_emb[ROMA2_SCALES] = {79, 23, 8};
const int ref2_radius[ROMA2_SCALES] = {3, 1, 0};
// VGG19-BN features[:40] (roma.c:68-69).
const int vgg_blocks[4] = {2, 2, 4, 4};
const int vgg_width[4] = {64, 128, 256, 512};

struct Block {
    float *n1g, *n1b, *qkv_b, *proj_b, *n2g, *n2b, *fc1_b, *fc2_b;
    void *qkv_w, *proj_w, *fc1_w, *fc2_w;
};

struct Refiner {
    int scale, feat, emb, radius, cin, nout;
    int cinp; // cin padded (row stride of the refiner maps)
    int fpitch; // row stride of the input feature maps (feat, padded to 8 for RoMa v2's)
    float *dw_w[ROMA_HIDDEN + 1], *dw_b[ROMA_HIDDEN + 1];
    void *pw_w[ROMA_HIDDEN + 1];
    float *pw_b[ROMA_HIDDEN + 1];
    void *out_w;
    float *out_b, *emb_w, *emb_b;
};

struct PilDev {
    int *start = nullptr;
    double *weight = nullptr;
    PilAxis ax{};
};

}  // namespace

// Row pitch (floats) of the refiners' output d_c (3 or 6 values a cell):
// 32-byte rows, which the tensor-core GEMM writes with TMA stores.
constexpr int DC_PITCH = 8;

struct roma_impl {
    DType wt = DT_F32; // GEMM weights
    DType at = DT_F32; // activations that feed GEMMs
    std::vector<void *> allocs;
    // Weights.
    void *vgg_w[16];
    float *vgg_b[16];
    // kp > 0: a few-channel layer stored as (cout, kp) rows for the
    // explicit-im2col tensor-core path (bfloat16 mode).
    int vgg_cin[16], vgg_cout[16], vgg_kp[16];
    void *patch_w;
    float *patch_b, *cls;
    // bfloat16 mode: patch weights as (1024, patch_kp) rows (zero padded),
    // the patches gathered into patch_col (n16 x patch_kp) for the tensor
    // cores.
    int patch_kp = 0;
    __nv_bfloat16 *patch_col = nullptr;
    std::vector<float> pos_raw; // (1 + 37 * 37) x 1024, host
    Block vit[ROMA_VIT_DEPTH], dec[ROMA_DEC_DEPTH];
    float *norm_g, *norm_b;
    void *proj_w[ROMA_SCALES];
    float *proj_b[ROMA_SCALES];
    std::vector<float> gp_w, gp_bias; // pos_conv (512 x 2), (512), host
    void *to_out_w;
    float *to_out_b;
    Refiner ref[ROMA_SCALES], ref2[ROMA2_SCALES];
    void *vgg2_w[8];
    float *vgg2_b[8];
    int vgg2_cin[8], vgg2_cout[8], vgg2_kp[8];
    void *proj2_w[ROMA2_SCALES];
    float *proj2_b[ROMA2_SCALES];
    // Geometry of the passes.
    int Cs = ROMA_COARSE, c16, n16, ntok;
    int hm, wm;
    // Work buffers.
    float *pos = nullptr, *gp_basis = nullptr;
    float *in_dev[2] = {};
    void *img = nullptr, *v_a = nullptr, *v_b = nullptr;
    float *pil_tmp = nullptr;
    void *P[ROMA_SCALES][2] = {}, *P2[ROMA2_SCALES][2] = {};
    float *t_x = nullptr, *t_out = nullptr;
    void *t_n = nullptr, *t_qkv = nullptr, *t_o = nullptr, *t_h = nullptr;
    size_t t_qkv_bytes = 0;
    float *g_nx, *g_ny, *g_kyy, *g_kxy, *g_x;
    // bfloat16 mode: the GP features split into bfloat16 parts for the
    // kernel matrices on the tensor cores (A3 forms of A's and B's
    // features, B3 form of B's; n16 x 3 GP_DIM each).
    __nv_bfloat16 *g_s3[3];
    double *gp_work;
    int *gp_flag;
    void *d_a = nullptr, *d_b = nullptr;
    float *d_c = nullptr;
    float *fl[2], *ce[2], *cf[2], *cert16, *lowres;
    float *o_flow, *o_cert, *o_sd;
    PilDev pil_cx, pil_cy, pil_fx, pil_fy;
    bool alloc_done = false;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
    // roma_match's own graph of the tile over in_dev, built on its first
    // call without dumps or profiling.
    cudaGraph_t match_graph = nullptr;
    cudaGraphExec_t match_exec = nullptr;
    int match_imagenet = -1;  // m->imagenet when match_graph was captured
};

// ------------------------------------------------------------- utilities

namespace {

size_t dsize(DType t) { return t == DT_BF16 ? 2 : 4; }

void *dmalloc(roma_impl *I, size_t bytes, const char *what)
{
    void *p = nullptr;
    if (pending())
        return nullptr;
    if (bytes == 0)
        bytes = 16;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail("CUDA: allocating %zu MiB for <%s> failed: %s", bytes >> 20, what,
             cudaGetErrorString(e));
        return nullptr;
    }
    I->allocs.push_back(p);
    return p;
}

// Upload n floats as dtype t (float32 or bfloat16).
void *upload(roma_impl *I, const float *v, size_t n, DType t, const char *what)
{
    void *d = dmalloc(I, n * dsize(t), what);
    if (!d)
        return nullptr;
    if (t == DT_F32) {
        cuda_ok(cudaMemcpy(d, v, n * 4, cudaMemcpyHostToDevice), what);
        return d;
    }
    std::vector<__nv_bfloat16> h(n);
    for (size_t i = 0; i < n; i++)
        h[i] = __float2bfloat16_rn(v[i]);
    cuda_ok(cudaMemcpy(d, h.data(), n * 2, cudaMemcpyHostToDevice), what);
    return d;
}

float *upload_f(roma_impl *I, const float *v, size_t n, const char *what)
{
    return (float *)upload(I, v, n, DT_F32, what);
}

struct HostT {
    float *v = nullptr;
    long n = 0;
    ~HostT() { free(v); }
};

bool read_host(struct pth_file *pf, const char *name, int ndim,
               const long *shape, HostT &out)
{
    const struct pth_tensor *t = pth_require(pf, name, ndim, shape);
    if (!t)
        return false;
    out.v = pth_read_f32(pf, t);
    out.n = pth_numel(t);
    return out.v != nullptr;
}

std::string fmt(const char *f, ...) __attribute__((format(printf, 1, 2)));
std::string fmt(const char *f, ...)
{
    char b[256];
    va_list ap;
    va_start(ap, f);
    vsnprintf(b, sizeof(b), f, ap);
    va_end(ap);
    return b;
}

// BatchNorm <bn> of c channels folded into w (c x per) and b
// (roma.c:103-123, with ops_fold_bn).
bool fold(struct pth_file *pf, const std::string &bn, int c, long per, float *w,
          float *b)
{
    long s1[1] = {c};
    HostT g, bt, mu, var;
    if (!read_host(pf, (bn + ".weight").c_str(), 1, s1, g) ||
        !read_host(pf, (bn + ".bias").c_str(), 1, s1, bt) ||
        !read_host(pf, (bn + ".running_mean").c_str(), 1, s1, mu) ||
        !read_host(pf, (bn + ".running_var").c_str(), 1, s1, var))
        return false;
    ops_fold_bn(w, b, c, per, g.v, bt.v, mu.v, var.v, EPS_BN);
    return true;
}

// Convolution <conv> (co x per, optional bias) with BatchNorm <bn> folded
// (roma.c:127-150), on the host.
bool conv_bn_host(struct pth_file *pf, const std::string &conv,
                  const std::string &bn, int co, int ndim, const long *shape,
                  std::vector<float> &w, std::vector<float> &b)
{
    long per = 1, bs[1] = {co};
    for (int d = 1; d < ndim; d++)
        per *= shape[d];
    HostT tw;
    if (!read_host(pf, (conv + ".weight").c_str(), ndim, shape, tw))
        return false;
    w.assign(tw.v, tw.v + (size_t)co * per);
    b.assign(co, 0.0f);
    if (pth_find(pf, (conv + ".bias").c_str())) {
        HostT tb;
        if (!read_host(pf, (conv + ".bias").c_str(), 1, bs, tb))
            return false;
        b.assign(tb.v, tb.v + co);
    }
    return fold(pf, bn, co, per, w.data(), b.data());
}

// (co, ci, 3, 3) -> (co, 3, 3, ci): the implicit-GEMM order of the
// token-major 3 x 3 convolution.
std::vector<float> conv3_reorder(const std::vector<float> &w, int co, int ci)
{
    std::vector<float> r(w.size());
    for (int o = 0; o < co; o++)
        for (int c = 0; c < ci; c++)
            for (int k = 0; k < 9; k++)
                r[((size_t)o * 9 + k) * ci + c] = w[((size_t)o * ci + c) * 9 + k];
    return r;
}

// The first nblk blocks of VGG19-BN under <pre>.<index> (roma.c:217-239).
bool load_vgg(roma_impl *I, struct pth_file *pf, const char *pre, int nblk,
              void **w, float **b, int *cin_out, int *cout_out, int *kp_out)
{
    int l = 0, idx = 0, cin = 3;
    for (int blk = 0; blk < nblk; blk++) {
        for (int j = 0; j < vgg_blocks[blk]; j++, l++) {
            const int co = vgg_width[blk];
            long shape[4] = {co, cin, 3, 3};
            std::vector<float> wv, bv;
            if (!conv_bn_host(pf, fmt("%s.%d", pre, idx), fmt("%s.%d", pre, idx + 1),
                              co, 4, shape, wv, bv))
                return false;
            std::vector<float> r = conv3_reorder(wv, co, cin);
            kp_out[l] = 0;
            if (I->wt == DT_BF16 && 9 * cin <= 64) {
                // Few input channels (the RGB layer): rows of kp columns,
                // zero beyond 9 cin.
                const int kp = (9 * cin + 15) / 16 * 16;
                std::vector<float> rp((size_t)co * kp, 0.0f);
                for (int o = 0; o < co; o++)
                    for (int j = 0; j < 9 * cin; j++)
                        rp[(size_t)o * kp + j] = r[(size_t)o * 9 * cin + j];
                r.swap(rp);
                kp_out[l] = kp;
            }
            w[l] = upload(I, r.data(), r.size(), I->wt, "vgg");
            b[l] = upload_f(I, bv.data(), co, "vgg");
            cin_out[l] = cin;
            cout_out[l] = co;
            cin = co;
            idx += 3; // Convolution, BatchNorm, ReLU.
        }
        idx++; // MaxPool.
    }
    return !pending();
}

void *load_dev(roma_impl *I, struct pth_file *pf, const std::string &name,
               int ndim, const long *shape, DType t)
{
    HostT h;
    if (!read_host(pf, name.c_str(), ndim, shape, h))
        return nullptr;
    return upload(I, h.v, h.n, t, name.c_str());
}

// One transformer block <pre>: LayerScales folded into proj and fc2
// (roma.c:155-214).
bool load_block(roma_impl *I, struct pth_file *pf, const std::string &pre,
                int D, int qkv_bias, int ls, Block *b)
{
    long v1[1] = {D}, sqkv[2] = {3 * D, D}, s3[1] = {3 * D};
    long sp[2] = {D, D}, s1[2] = {MLP_RATIO * D, D}, sb1[1] = {MLP_RATIO * D};
    long s2[2] = {D, MLP_RATIO * D};
    b->n1g = (float *)load_dev(I, pf, pre + ".norm1.weight", 1, v1, DT_F32);
    b->n1b = (float *)load_dev(I, pf, pre + ".norm1.bias", 1, v1, DT_F32);
    b->qkv_w = load_dev(I, pf, pre + ".attn.qkv.weight", 2, sqkv, I->wt);
    b->qkv_b = qkv_bias ? (float *)load_dev(I, pf, pre + ".attn.qkv.bias", 1, s3,
                                            DT_F32)
                        : nullptr;
    b->n2g = (float *)load_dev(I, pf, pre + ".norm2.weight", 1, v1, DT_F32);
    b->n2b = (float *)load_dev(I, pf, pre + ".norm2.bias", 1, v1, DT_F32);
    b->fc1_w = load_dev(I, pf, pre + ".mlp.fc1.weight", 2, s1, I->wt);
    b->fc1_b = (float *)load_dev(I, pf, pre + ".mlp.fc1.bias", 1, sb1, DT_F32);
    for (int j = 0; j < 2; j++) {
        const std::string wn = j ? ".mlp.fc2" : ".attn.proj";
        const int in = j ? MLP_RATIO * D : D;
        HostT w, bias;
        if (!read_host(pf, (pre + wn + ".weight").c_str(), 2, j ? s2 : sp, w) ||
            !read_host(pf, (pre + wn + ".bias").c_str(), 1, v1, bias))
            return false;
        if (ls) {
            HostT g;
            if (!read_host(pf, (pre + fmt(".ls%d.gamma", j + 1)).c_str(), 1, v1, g))
                return false;
            for (int i = 0; i < D; i++) {
                for (int c = 0; c < in; c++)
                    w.v[(size_t)i * in + c] *= g.v[i];
                bias.v[i] *= g.v[i];
            }
        }
        void *dw = upload(I, w.v, (size_t)D * in, I->wt, "block");
        float *db = upload_f(I, bias.v, D, "block");
        if (j) {
            b->fc2_w = dw;
            b->fc2_b = db;
        }
        else {
            b->proj_w = dw;
            b->proj_b = db;
        }
    }
    return !pending();
}

// rows x cols row-major into prows x pcols, zero padded.
std::vector<float> pad_matrix(const float *v, int rows, int cols, int prows,
                              int pcols)
{
    std::vector<float> out((size_t)prows * pcols, 0.0f);
    for (int r = 0; r < rows; r++)
        memcpy(&out[(size_t)r * pcols], v + (size_t)r * cols, cols * sizeof(float));
    return out;
}

// Refiner input width padded to a multiple of 16 channels (16-byte rows
// of bfloat16 for the tensor-memory-access loads of the 1 x 1 GEMMs).
int pad16(int c) { return (c + 15) / 16 * 16; }

// ConvRefiner blocks: depthwise 5 x 5 with its BatchNorm folded, 1 x 1.
bool load_ref_blocks(roma_impl *I, struct pth_file *pf, Refiner *r,
                     const std::string &pre, bool v2)
{
    for (int b = 0; b <= ROMA_HIDDEN; b++) {
        long sdw[4] = {r->cin, 1, 5, 5}, spw[4] = {r->cin, r->cin, 1, 1};
        long sb[1] = {r->cin};
        const std::string blk =
            b == 0 ? pre + ".block1" : pre + fmt(".hidden_blocks.%d", b - 1);
        const std::string conv = v2 ? blk + ".conv_depthwise" : blk + ".0";
        const std::string bn = v2 ? blk + ".norm" : blk + ".1";
        const std::string pw = v2 ? blk + ".conv_pointwise" : blk + ".3";
        std::vector<float> w, bias;
        if (!conv_bn_host(pf, conv, bn, r->cin, 4, sdw, w, bias))
            return false;
        // Channels padded to cinp with zero weights and biases: the padded
        // channels of every block stay 0.
        w.resize((size_t)r->cinp * 25, 0.0f);
        bias.resize(r->cinp, 0.0f);
        r->dw_w[b] = upload_f(I, w.data(), w.size(), "dw");
        r->dw_b[b] = upload_f(I, bias.data(), bias.size(), "dw");
        HostT pw_w, pw_b;
        if (!read_host(pf, (pw + ".weight").c_str(), 4, spw, pw_w) ||
            !read_host(pf, (pw + ".bias").c_str(), 1, sb, pw_b))
            return false;
        std::vector<float> pwp = pad_matrix(pw_w.v, r->cin, r->cin, r->cinp, r->cinp);
        std::vector<float> pbp(pw_b.v, pw_b.v + r->cin);
        pbp.resize(r->cinp, 0.0f);
        r->pw_w[b] = upload(I, pwp.data(), pwp.size(), I->wt, "pw");
        r->pw_b[b] = upload_f(I, pbp.data(), pbp.size(), "pw");
    }
    return !pending();
}

// roma.c:352-396.
bool load_refiner(roma_impl *I, struct pth_file *pf, int s)
{
    Refiner *r = &I->ref[s];
    r->scale = ref_scale[s];
    r->feat = ref_feat[s];
    r->emb = ref_emb[s];
    r->radius = ref_radius[s];
    const int corr = r->radius ? (2 * r->radius + 1) * (2 * r->radius + 1) : 0;
    r->cin = 2 * r->feat + r->emb + corr;
    r->cinp = pad16(r->cin);
    r->fpitch = r->feat;
    r->nout = 3;
    const std::string pre = fmt("decoder.conv_refiner.%d", r->scale);
    if (!load_ref_blocks(I, pf, r, pre, false))
        return false;
    long so[4] = {3, r->cin, 1, 1}, sob[1] = {3};
    long se[4] = {r->emb, 2, 1, 1}, seb[1] = {r->emb};
    {
        HostT ow;
        if (!read_host(pf, (pre + ".out_conv.weight").c_str(), 4, so, ow))
            return false;
        std::vector<float> p = pad_matrix(ow.v, 3, r->cin, 3, r->cinp);
        r->out_w = upload(I, p.data(), p.size(), I->wt, "out_conv");
    }
    r->out_b = (float *)load_dev(I, pf, pre + ".out_conv.bias", 1, sob, DT_F32);
    r->emb_w = (float *)load_dev(I, pf, pre + ".disp_emb.weight", 4, se, DT_F32);
    r->emb_b = (float *)load_dev(I, pf, pre + ".disp_emb.bias", 1, seb, DT_F32);
    return !pending();
}

// roma.c:460-531: input projection, blocks, warp and confidence heads
// concatenated into 6 outputs.
bool load_refiner2(roma_impl *I, struct pth_file *pf, int j)
{
    Refiner *r = &I->ref2[j];
    r->scale = ref2_scale[j];
    r->feat = ref2_feat[j];
    r->emb = ref2_emb[j];
    r->radius = ref2_radius[j];
    const int corr = r->radius ? (2 * r->radius + 1) * (2 * r->radius + 1) : 0;
    r->cin = 2 * r->feat + r->emb + corr;
    r->cinp = pad16(r->cin);
    // 16-byte rows (bfloat16) for the projection's TMA-store epilogue.
    r->fpitch = (r->feat + 7) / 8 * 8;
    r->nout = 6;
    const std::string pre = fmt("refiners.%d", r->scale);
    long sp[2] = {ref2_feat[j], ref2_in[j]}, spb[1] = {ref2_feat[j]};
    I->proj2_w[j] = load_dev(I, pf, pre + ".proj.weight", 2, sp, I->wt);
    I->proj2_b[j] = (float *)load_dev(I, pf, pre + ".proj.bias", 1, spb, DT_F32);
    if (!load_ref_blocks(I, pf, r, pre, true))
        return false;
    long se[4] = {r->emb, 2, 1, 1}, seb[1] = {r->emb};
    long sw[4] = {2, r->cin, 1, 1}, swb[1] = {2};
    long sc[4] = {4, r->cin, 1, 1}, scb[1] = {4};
    r->emb_w = (float *)load_dev(I, pf, pre + ".disp_emb.weight", 4, se, DT_F32);
    r->emb_b = (float *)load_dev(I, pf, pre + ".disp_emb.bias", 1, seb, DT_F32);
    HostT ww, cw, wb, cb;
    if (!read_host(pf, (pre + ".warp_head.weight").c_str(), 4, sw, ww) ||
        !read_host(pf, (pre + ".confidence_head.weight").c_str(), 4, sc, cw) ||
        !read_host(pf, (pre + ".warp_head.bias").c_str(), 1, swb, wb) ||
        !read_host(pf, (pre + ".confidence_head.bias").c_str(), 1, scb, cb))
        return false;
    std::vector<float> w(6 * (size_t)r->cin), bias(6);
    memcpy(w.data(), ww.v, 2 * (size_t)r->cin * 4);
    memcpy(w.data() + 2 * (size_t)r->cin, cw.v, 4 * (size_t)r->cin * 4);
    for (int k = 0; k < 2; k++)
        bias[k] = wb.v[k];
    for (int k = 0; k < 4; k++)
        bias[2 + k] = cb.v[k];
    w = pad_matrix(w.data(), 6, r->cin, 6, r->cinp);
    r->out_w = upload(I, w.data(), w.size(), I->wt, "heads");
    r->out_b = upload_f(I, bias.data(), 6, "heads");
    return !pending();
}

// PyTorch's bicubic convolution weights (A = -0.75) at fraction t.
void cubic_weights(double t, double w[4])
{
    const double A = -0.75;
    double x = t + 1;
    w[0] = ((A * x - 5 * A) * x + 8 * A) * x - 4 * A;
    x = t;
    w[1] = ((A + 2) * x - (A + 3)) * x * x + 1;
    x = 1 - t;
    w[2] = ((A + 2) * x - (A + 3)) * x * x + 1;
    x = 2 - t;
    w[3] = ((A * x - 5 * A) * x + 8 * A) * x - 4 * A;
}

// DINOv2's interpolate_pos_encoding for a c16 x c16 grid: the 37 x 37
// patch embeddings resized by F.interpolate(mode="bicubic", scale_factor=
// (c16 + 0.1) / 37), source coordinates from that factor; the class
// embedding first (roma.c:257-298).
std::vector<float> interp_pos(const float *pos, int c16)
{
    const int D = ROMA_VIT_DIM;
    std::vector<float> out((size_t)(1 + c16 * c16) * D);
    const double inv = VIT_GRID / (c16 + 0.1);
    memcpy(out.data(), pos, D * sizeof(float));
    for (int oy = 0; oy < c16; oy++)
        for (int ox = 0; ox < c16; ox++) {
            const double ry = inv * (oy + 0.5) - 0.5, rx = inv * (ox + 0.5) - 0.5;
            const int iy = (int)floor(ry), ix = (int)floor(rx);
            double wy[4], wx[4];
            float *o = out.data() + (size_t)(1 + oy * c16 + ox) * D;
            cubic_weights(ry - iy, wy);
            cubic_weights(rx - ix, wx);
            for (int c = 0; c < D; c++) {
                double s = 0;
                for (int i = 0; i < 4; i++) {
                    int yy = iy - 1 + i;
                    yy = yy < 0 ? 0 : yy > VIT_GRID - 1 ? VIT_GRID - 1 : yy;
                    for (int j = 0; j < 4; j++) {
                        int xx = ix - 1 + j;
                        xx = xx < 0 ? 0 : xx > VIT_GRID - 1 ? VIT_GRID - 1 : xx;
                        s += wy[i] * wx[j] *
                             pos[(size_t)(1 + yy * VIT_GRID + xx) * D + c];
                    }
                }
                o[c] = (float)s;
            }
        }
    return out;
}

// GP basis of the coarse grid: cos(8 pi pos_conv(x, y)) at the c16 x c16
// cell centres, token-major (roma.c:328-350).
std::vector<float> gp_basis(const std::vector<float> &w,
                            const std::vector<float> &b, int c16)
{
    std::vector<float> out((size_t)c16 * c16 * GP_DIM);
    for (int i = 0; i < c16 * c16; i++) {
        const float x = -1.0f + 1.0f / c16 + (i % c16) * (2.0f - 2.0f / c16) / (c16 - 1);
        const float y = -1.0f + 1.0f / c16 + (i / c16) * (2.0f - 2.0f / c16) / (c16 - 1);
        for (int d = 0; d < GP_DIM; d++) {
            const float v = w[2 * d] * x + w[2 * d + 1] * y + b[d];
            out[(size_t)i * GP_DIM + d] = cosf(8.0f * (float)M_PI * v);
        }
    }
    return out;
}

// Pillow's bicubic taps (a = -0.5, support 2 scaled by the reduction) of
// every output index, normalized (roma.c:1106-1155).
double pil_cubic(double x)
{
    const double a = -0.5;
    x = fabs(x);
    if (x < 1)
        return ((a + 2) * x - (a + 3)) * x * x + 1;
    if (x < 2)
        return (((x - 5) * x + 8) * x - 4) * a;
    return 0;
}

bool pil_axis(roma_impl *I, int n_in, int n_out, PilDev *d)
{
    const double scale = (double)n_in / n_out, fs = scale > 1 ? scale : 1;
    const double support = 2 * fs;
    std::vector<int> start(n_out), count(n_out);
    std::vector<std::vector<double>> k(n_out);
    int taps = 1;
    for (int o = 0; o < n_out; o++) {
        const double center = (o + 0.5) * scale;
        int xmin = (int)(center - support + 0.5);
        if (xmin < 0)
            xmin = 0;
        int xmax = (int)(center + support + 0.5);
        if (xmax > n_in)
            xmax = n_in;
        xmax -= xmin;
        if (xmax > 64) {
            fail("RoMa: resampling ratio too large");
            return false;
        }
        double ww = 0;
        k[o].resize(xmax);
        for (int x = 0; x < xmax; x++) {
            k[o][x] = pil_cubic((x + xmin - center + 0.5) / fs);
            ww += k[o][x];
        }
        for (int x = 0; x < xmax; x++)
            k[o][x] = ww != 0 ? k[o][x] / ww : 0;
        start[o] = xmin;
        count[o] = xmax;
        if (xmax > taps)
            taps = xmax;
    }
    // Pad every row to taps (zero weights), keeping the reads inside the
    // input: the start moves left where needed.
    std::vector<double> wt((size_t)n_out * taps, 0.0);
    for (int o = 0; o < n_out; o++) {
        int s = start[o];
        if (s + taps > n_in)
            s = n_in - taps;
        if (s < 0)
            s = 0;
        for (int x = 0; x < count[o]; x++)
            wt[(size_t)o * taps + (start[o] - s) + x] = k[o][x];
        start[o] = s;
    }
    if (taps > n_in) {
        fail("RoMa: resampling %d -> %d needs %d taps", n_in, n_out, taps);
        return false;
    }
    d->start = (int *)dmalloc(I, n_out * sizeof(int), "pil");
    d->weight = (double *)dmalloc(I, wt.size() * sizeof(double), "pil");
    if (pending())
        return false;
    if (!cuda_ok(cudaMemcpy(d->start, start.data(), n_out * sizeof(int),
                            cudaMemcpyHostToDevice),
                 "RoMa resampling taps") ||
        !cuda_ok(cudaMemcpy(d->weight, wt.data(), wt.size() * sizeof(double),
                            cudaMemcpyHostToDevice),
                 "RoMa resampling weights"))
        return false;
    d->ax.n_out = n_out;
    d->ax.taps = taps;
    d->ax.start = d->start;
    d->ax.weight = d->weight;
    return true;
}

int side(const roma_impl *I, int n, int s)
{
    (void)I;
    return s == 0 ? n / ROMA_PATCH : n / ref_scale[s];
}

}  // namespace

// ------------------------------------------------------------ load / free

extern "C" void roma_load(struct roma_model *m, struct ops *ops,
                          struct pth_file *pf, struct pth_file *dino)
{
    memset(m, 0, sizeof(*m));
    if (pending())
        return;
    m->ops = ops;
    m->ocl = ops->ocl;
    m->imagenet = 1;
    m->coarse = ROMA_COARSE;
    m->precision = ops->precision;
    cudaSetDevice(m->ocl->device);
    roma_impl *I = new roma_impl();
    m->impl = I;
    if (m->precision == OPS_BF16) {
        I->wt = DT_BF16;
        I->at = DT_BF16;
    }
    // MatchAnything's Lightning checkpoint.
    pth_strip_prefix(pf, "matcher.model.");
    if (!load_vgg(I, pf, "encoder.cnn.layers", 4, I->vgg_w, I->vgg_b, I->vgg_cin,
                  I->vgg_cout, I->vgg_kp))
        return;
    // DINOv2 (roma.c:300-324).
    {
        long sw[2] = {ROMA_VIT_DIM, 3 * ROMA_PATCH * ROMA_PATCH};
        long sw4[4] = {ROMA_VIT_DIM, 3, ROMA_PATCH, ROMA_PATCH};
        long v1[1] = {ROMA_VIT_DIM}, sc[3] = {1, 1, ROMA_VIT_DIM};
        long sp[3] = {1, VIT_GRID * VIT_GRID + 1, ROMA_VIT_DIM};
        (void)sw;
        if (I->wt == DT_BF16) {
            const int K = 3 * ROMA_PATCH * ROMA_PATCH, kp = (K + 15) / 16 * 16;
            HostT hw;
            if (!read_host(dino, "patch_embed.proj.weight", 4, sw4, hw))
                return;
            std::vector<float> pad((size_t)ROMA_VIT_DIM * kp, 0.0f);
            for (int o = 0; o < ROMA_VIT_DIM; o++)
                for (int k = 0; k < K; k++)
                    pad[(size_t)o * kp + k] = hw.v[(size_t)o * K + k];
            I->patch_w = upload(I, pad.data(), pad.size(), DT_BF16, "patch_embed");
            I->patch_kp = kp;
        }
        else
            I->patch_w = load_dev(I, dino, "patch_embed.proj.weight", 4, sw4, I->wt);
        I->patch_b = (float *)load_dev(I, dino, "patch_embed.proj.bias", 1, v1, DT_F32);
        I->cls = (float *)load_dev(I, dino, "cls_token", 3, sc, DT_F32);
        HostT pos;
        if (!read_host(dino, "pos_embed", 3, sp, pos))
            return;
        I->pos_raw.assign(pos.v, pos.v + pos.n);
        for (int i = 0; i < ROMA_VIT_DEPTH; i++)
            if (!load_block(I, dino, fmt("blocks.%d", i), ROMA_VIT_DIM, 1, 1,
                            &I->vit[i]))
                return;
        I->norm_g = (float *)load_dev(I, dino, "norm.weight", 1, v1, DT_F32);
        I->norm_b = (float *)load_dev(I, dino, "norm.bias", 1, v1, DT_F32);
    }
    for (int s = 0; s < ROMA_SCALES; s++) {
        long shape[4] = {ref_feat[s], proj_in_ch[s], 1, 1};
        std::vector<float> w, b;
        if (!conv_bn_host(pf, fmt("decoder.proj.%d.0", ref_scale[s]),
                          fmt("decoder.proj.%d.1", ref_scale[s]), ref_feat[s], 4,
                          shape, w, b))
            return;
        I->proj_w[s] = upload(I, w.data(), w.size(), I->wt, "proj");
        I->proj_b[s] = upload_f(I, b.data(), b.size(), "proj");
    }
    {
        long sw[4] = {GP_DIM, 2, 1, 1}, sb[1] = {GP_DIM};
        HostT w, b;
        if (!read_host(pf, "decoder.gps.16.pos_conv.weight", 4, sw, w) ||
            !read_host(pf, "decoder.gps.16.pos_conv.bias", 1, sb, b))
            return;
        I->gp_w.assign(w.v, w.v + w.n);
        I->gp_bias.assign(b.v, b.v + b.n);
    }
    for (int i = 0; i < ROMA_DEC_DEPTH; i++)
        if (!load_block(I, pf, fmt("decoder.embedding_decoder.blocks.%d", i),
                        ROMA_DEC_DIM, 0, 0, &I->dec[i]))
            return;
    {
        long so[2] = {NCLS + 1, ROMA_DEC_DIM}, sob[1] = {NCLS + 1};
        I->to_out_w = load_dev(I, pf, "decoder.embedding_decoder.to_out.weight", 2,
                               so, I->wt);
        I->to_out_b = (float *)load_dev(I, pf, "decoder.embedding_decoder.to_out.bias",
                                        1, sob, DT_F32);
    }
    for (int s = 0; s < ROMA_SCALES; s++)
        if (!load_refiner(I, pf, s))
            return;
}

extern "C" void roma_load_v2(struct roma_model *m, struct pth_file *pf)
{
    roma_impl *I = m->impl;
    if (pending() || !I)
        return;
    cudaSetDevice(m->ocl->device);
    if (!load_vgg(I, pf, "refiner_features.layers", 3, I->vgg2_w, I->vgg2_b,
                  I->vgg2_cin, I->vgg2_cout, I->vgg2_kp))
        return;
    for (int j = 0; j < ROMA2_SCALES; j++)
        if (!load_refiner2(I, pf, j))
            return;
    m->v2 = 1;
}

extern "C" void roma_set_coarse(struct roma_model *m, int side_px)
{
    if (pending())
        return;
    if (side_px < 56 || side_px % 56) {
        fail("RoMa: coarse side %d is not a positive multiple of 56", side_px);
        return;
    }
    if (m->impl && m->impl->alloc_done) {
        fail("RoMa: roma_set_coarse after roma_alloc");
        return;
    }
    m->coarse = side_px;
}

extern "C" void roma_free(struct roma_model *m)
{
    roma_impl *I = m->impl;
    if (I) {
        cudaSetDevice(m->ocl->device);
        cudaStreamSynchronize(stream_of(m->ocl));
        if (I->graph_exec)
            cudaGraphExecDestroy(I->graph_exec);
        if (I->graph)
            cudaGraphDestroy(I->graph);
        if (I->match_exec)
            cudaGraphExecDestroy(I->match_exec);
        if (I->match_graph)
            cudaGraphDestroy(I->match_graph);
        for (void *p : I->allocs)
            cudaFree(p);
        delete I;
    }
    if (m->flow)
        cudaFreeHost(m->flow);
    if (m->cert)
        cudaFreeHost(m->cert);
    if (m->sd)
        cudaFreeHost(m->sd);
    memset(m, 0, sizeof(*m));
}

// ------------------------------------------------------------------ alloc

extern "C" void roma_alloc(struct roma_model *m, int H, int W)
{
    roma_impl *I = m->impl;
    if (pending() || !I)
        return;
    if (H % ROMA_MULTIPLE || W % ROMA_MULTIPLE || H <= 0 || W <= 0) {
        fail("RoMa tile %d x %d is not a multiple of %d", H, W, ROMA_MULTIPLE);
        return;
    }
    if (I->alloc_done) {
        fail("RoMa: roma_alloc called twice");
        return;
    }
    cudaSetDevice(m->ocl->device);
    m->H = H;
    m->W = W;
    I->Cs = m->coarse;
    I->c16 = I->Cs / ROMA_PATCH;
    I->n16 = I->c16 * I->c16;
    I->ntok = I->n16 + 1;
    I->hm = H > I->Cs ? H : I->Cs;
    I->wm = W > I->Cs ? W : I->Cs;
    const size_t hm = (size_t)I->hm * I->wm, n16 = I->n16, ntok = I->ntok;
    const size_t as = dsize(I->at);
    const int D = ROMA_VIT_DIM;

    {
        std::vector<float> ip = interp_pos(I->pos_raw.data(), I->c16);
        I->pos = upload_f(I, ip.data(), ip.size(), "pos_embed");
        std::vector<float> gb = gp_basis(I->gp_w, I->gp_bias, I->c16);
        I->gp_basis = upload_f(I, gb.data(), gb.size(), "GP basis");
    }
    for (int k = 0; k < 2; k++)
        I->in_dev[k] = (float *)dmalloc(I, 3 * (size_t)H * W * 4, "input");
    I->img = dmalloc(I, 3 * hm * as, "image");
    I->pil_tmp = (float *)dmalloc(I, 3 * (size_t)H * I->Cs * 4, "resample");
    I->v_a = dmalloc(I, 64 * hm * as, "VGG");
    I->v_b = dmalloc(I, 64 * hm * as, "VGG");
    for (int k = 0; k < 2; k++) {
        I->P[0][k] = dmalloc(I, n16 * GP_DIM * 4, "1/16 features");
        for (int s = 1; s < ROMA_SCALES; s++)
            I->P[s][k] = dmalloc(I,
                                 (size_t)ref_feat[s] * (I->hm / ref_scale[s]) *
                                     (I->wm / ref_scale[s]) * as,
                                 "projected features");
    }
    // Token buffers for both images' DINOv2 tokens.
    I->t_x = (float *)dmalloc(I, 2 * ntok * D * 4, "tokens");
    I->t_n = dmalloc(I, 2 * ntok * D * as, "tokens");
    I->t_qkv_bytes = (size_t)2 * ntok * 3 * D * as;
    I->t_qkv = dmalloc(I, I->t_qkv_bytes, "qkv");
    I->t_o = dmalloc(I, 2 * ntok * D * as, "attention");
    I->t_h = dmalloc(I, 2 * ntok * MLP_RATIO * D * as, "mlp");
    I->t_out = (float *)dmalloc(I, n16 * (NCLS + 1) * 4, "anchor logits");
    I->g_nx = (float *)dmalloc(I, n16 * 4, "norms");
    I->g_ny = (float *)dmalloc(I, n16 * 4, "norms");
    if (I->at == DT_BF16)
        for (int k = 0; k < 3; k++)
            I->g_s3[k] = (__nv_bfloat16 *)dmalloc(I, n16 * 3 * GP_DIM * 2, "GP split features");
    I->g_kyy = (float *)dmalloc(I, n16 * n16 * 4, "GP kernel");
    I->g_kxy = (float *)dmalloc(I, n16 * n16 * 4, "GP kernel");
    I->g_x = (float *)dmalloc(I, n16 * GP_DIM * 4, "GP solve");
    if (I->patch_kp)
        I->patch_col = (__nv_bfloat16 *)dmalloc(I, n16 * I->patch_kp * 2, "patches");
    I->gp_work = (double *)dmalloc(I, gp_work_doubles((int)n16, GP_DIM) * 8, "GP work");
    I->gp_flag = (int *)dmalloc(I, sizeof(int), "GP flag");
    size_t dmax = 0;
    for (int p = 0; p < 2; p++)
        for (int s = p; s < ROMA_SCALES; s++) {
            const int ph = p ? H : I->Cs, pw = p ? W : I->Cs;
            const size_t n = (size_t)side(I, ph, s) * side(I, pw, s);
            dmax = std::max(dmax, (size_t)I->ref[s].cinp * n);
        }
    if (m->v2)
        for (int p = 0; p < 2; p++)
            for (int s = 0; s < ROMA2_SCALES; s++) {
                const int ph = p ? H : I->Cs, pw = p ? W : I->Cs;
                const size_t n = (size_t)(ph / ref2_scale[s]) * (pw / ref2_scale[s]);
                dmax = std::max(dmax, (size_t)I->ref2[s].cinp * n);
            }
    I->d_a = dmalloc(I, dmax * as, "refiner");
    I->d_b = dmalloc(I, dmax * as, "refiner");
    I->d_c = (float *)dmalloc(I, (size_t)DC_PITCH * hm * 4, "refiner");
    for (int k = 0; k < 2; k++) {
        I->fl[k] = (float *)dmalloc(I, 2 * hm * 4, "warp");
        I->ce[k] = (float *)dmalloc(I, hm * 4, "certainty");
        I->cf[k] = (float *)dmalloc(I, 4 * hm * 4, "confidence");
    }
    if (m->v2)
        for (int k = 0; k < 2; k++)
            for (int s = 0; s < ROMA2_SCALES; s++)
                I->P2[s][k] = dmalloc(I,
                                      (size_t)I->ref2[s].fpitch * (I->hm / ref2_scale[s]) *
                                          (I->wm / ref2_scale[s]) * as,
                                      "projected features");
    I->cert16 = (float *)dmalloc(I, n16 * 4, "coarse certainty");
    I->lowres = (float *)dmalloc(I, (size_t)H * W * 4, "coarse certainty");
    I->o_flow = (float *)dmalloc(I, 2 * (size_t)H * W * 4, "flow");
    I->o_cert = (float *)dmalloc(I, (size_t)H * W * 4, "cert");
    I->o_sd = (float *)dmalloc(I, (size_t)H * W * 4, "sd");
    if (pending())
        return;
    cudaMemset(I->gp_flag, 0, sizeof(int));
    if (!pil_axis(I, W, I->Cs, &I->pil_cx) || !pil_axis(I, H, I->Cs, &I->pil_cy) ||
        !pil_axis(I, W, W, &I->pil_fx) || !pil_axis(I, H, H, &I->pil_fy))
        return;
    if (!cuda_ok(cudaMallocHost((void **)&m->flow, 2 * (size_t)H * W * 4), "host") ||
        !cuda_ok(cudaMallocHost((void **)&m->cert, (size_t)H * W * 4), "host"))
        return;
    if (m->v2 && !cuda_ok(cudaMallocHost((void **)&m->sd, (size_t)H * W * 4), "host"))
        return;
    I->alloc_done = true;
}

// -------------------------------------------------------------- the tile

namespace {

struct Ctx {
    struct roma_model *m;
    roma_impl *I;
    cudaStream_t st;
    const char *dump;
    int tile;
};

void gemm_nt(Ctx &c, const char *what, int M, int N, int K, const void *A,
             long lda, DType ta, const void *B, const float *bias, void *C,
             long ldc, DType tc, int act, bool residual)
{
    GemmArgs g = gemm_args(M, N, K);
    g.A = A;
    g.lda = lda;
    g.B = B;
    g.ldb = K;
    g.transb = 1;
    g.C = C;
    g.ldc = ldc;
    g.bias = bias;
    g.R = residual ? C : nullptr;
    g.act = act;
    g.ab = ta;
    g.c = tc;
    gemm_run(c.m->ocl, g, what);
}

void dump_host(Ctx &c, const char *what, const float *v, size_t n)
{
    char path[4096];
    snprintf(path, sizeof(path), "%s/tile%03d_roma_%s.f32", c.dump, c.tile, what);
    FILE *fp = fopen(path, "wb");
    if (!fp || fwrite(v, sizeof(float), n, fp) != n)
        fail("Unable to write debug dump <%s>", path);
    if (fp)
        fclose(fp);
}

// Device buffer of n elements of type t into a float dump; with
// rows / cols set, a token-major (rows x cols) buffer written
// channel-major (cols x rows), the reference's layout.
void dump_dev(Ctx &c, const char *what, const void *p, DType t, size_t n,
              long rows = 0, long cols = 0)
{
    if (!c.dump || pending())
        return;
    cudaStreamSynchronize(c.st);
    std::vector<float> v(n);
    if (t == DT_F32)
        cudaMemcpy(v.data(), p, n * 4, cudaMemcpyDeviceToHost);
    else {
        std::vector<__nv_bfloat16> h(n);
        cudaMemcpy(h.data(), p, n * 2, cudaMemcpyDeviceToHost);
        for (size_t i = 0; i < n; i++)
            v[i] = __bfloat162float(h[i]);
    }
    if (rows) {
        std::vector<float> tr(n);
        for (long r = 0; r < rows; r++)
            for (long k = 0; k < cols; k++)
                tr[(size_t)k * rows + r] = v[(size_t)r * cols + k];
        v.swap(tr);
    }
    dump_host(c, what, v.data(), n);
}

// Pillow resampling of image k (device (3, H, W)) to h x w, normalized,
// into img (channels-last).
void prepare(Ctx &c, const float *in, int H, int W, const PilDev &ax,
             const PilDev &ay)
{
    roma_impl *I = c.I;
    Prof p(c.m->ocl, "roma_prepare");
    pil_resize_norm(c.st, in, H, W, I->pil_tmp, ax.ax, ay.ax, c.m->imagenet,
                    I->img, I->at);
    launch_ok("roma_prepare");
}

// kp > 0: the few-channel path, with col (h w x kp elements) as its
// im2col buffer.
void conv3(Ctx &c, const void *in, int cin, int h, int w, const void *wt,
           const float *b, int cout, void *out, int kp, void *col)
{
    if (kp) {
        Prof p(c.m->ocl, "vgg_conv3x3");
        conv3x3_im2col_tc(c.st, (const __nv_bfloat16 *)in, h, w, cin, kp,
                          (const __nv_bfloat16 *)wt, b, cout, ACTF_RELU, 0.0f, out,
                          c.I->at, (__nv_bfloat16 *)col, c.m->ocl->sm_count);
        launch_ok("vgg_conv3x3");
        return;
    }
    GemmArgs g = gemm_args(h * w, cout, 9 * cin);
    g.A = in;
    g.amode = 1;
    g.cH = h;
    g.cW = w;
    g.cC = cin;
    g.B = wt;
    g.ldb = 9 * cin;
    g.transb = 1;
    g.C = out;
    g.ldc = cout;
    g.bias = b;
    g.act = ACTF_RELU;
    g.ab = c.I->at;
    g.c = c.I->at;
    gemm_run(c.m->ocl, g, "vgg_conv3x3");
}

// VGG19-BN on img (h x w, channels-last) of image k: the projected
// features before each pooling into P[4] (1/1) .. P[1] (1/8)
// (roma.c:742-768); only the scales listed in need are projected.
void vgg(Ctx &c, int H, int W, int k, const bool need[ROMA_SCALES])
{
    roma_impl *I = c.I;
    const void *in = I->img;
    int l = 0, h = H, w = W;
    for (int blk = 0; blk < 4; blk++) {
        const int s = 4 - blk;
        for (int j = 0; j < vgg_blocks[blk]; j++, l++) {
            void *out = in == I->v_a ? I->v_b : I->v_a;
            conv3(c, in, I->vgg_cin[l], h, w, I->vgg_w[l], I->vgg_b[l],
                  I->vgg_cout[l], out, I->vgg_kp[l], out == I->v_a ? I->v_b : I->v_a);
            in = out;
        }
        if (need[s])
            gemm_nt(c, "vgg_proj", h * w, ref_feat[s], proj_in_ch[s], in,
                    proj_in_ch[s], I->at, I->proj_w[s], I->proj_b[s], I->P[s][k],
                    ref_feat[s], I->at, ACTF_NONE, false);
        if (blk < 3) {
            void *out = in == I->v_a ? I->v_b : I->v_a;
            Prof p(c.m->ocl, "maxpool");
            maxpool2_tm(c.st, in, I->at, h, w, vgg_width[blk], out);
            in = out;
            h /= 2;
            w /= 2;
        }
    }
}

// RoMa v2's VGG19-BN (three blocks) through each refiner's input
// projection into P2 (roma.c:1000-1027).
void vgg2(Ctx &c, int H, int W, int k)
{
    roma_impl *I = c.I;
    const void *in = I->img;
    int l = 0, h = H, w = W;
    for (int blk = 0; blk < 3; blk++) {
        const int r = 2 - blk;
        for (int j = 0; j < vgg_blocks[blk]; j++, l++) {
            void *out = in == I->v_a ? I->v_b : I->v_a;
            conv3(c, in, I->vgg2_cin[l], h, w, I->vgg2_w[l], I->vgg2_b[l],
                  I->vgg2_cout[l], out, I->vgg2_kp[l], out == I->v_a ? I->v_b : I->v_a);
            in = out;
        }
        gemm_nt(c, "vgg2_proj", h * w, I->ref2[r].feat, ref2_in[r], in, ref2_in[r],
                I->at, I->proj2_w[r], I->proj2_b[r], I->P2[r][k], I->ref2[r].fpitch,
                I->at, ACTF_NONE, false);
        if (blk < 2) {
            void *out = in == I->v_a ? I->v_b : I->v_a;
            Prof p(c.m->ocl, "maxpool");
            maxpool2_tm(c.st, in, I->at, h, w, vgg_width[blk], out);
            in = out;
            h /= 2;
            w /= 2;
        }
    }
}

__global__ void cls_pos_k(float *x, const float *cls, const float *pos, int D)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < D)
        x[i] = cls[i] + pos[i];
}

// Pre-norm transformer block on t_x (N x D) in place (roma.c:697-713),
// attention without the score matrix.
// One pre-norm transformer block over nimg images of N tokens each, stored
// one after the other in the token buffers: every linear layer runs once
// over all nimg N rows, attention per image.
void block(Ctx &c, const Block &b, int N, int nimg, int D, int heads, float eps)
{
    roma_impl *I = c.I;
    const DType at = I->at;
    const int rows = N * nimg;
    {
        Prof p(c.m->ocl, "layernorm");
        layernorm_rows(c.st, I->t_x, I->t_n, at, b.n1g, b.n1b, rows, D, eps,
                       ACTF_NONE, 0.0f);
    }
    gemm_nt(c, "qkv", rows, 3 * D, D, I->t_n, D, at, b.qkv_w, b.qkv_b, I->t_qkv,
            3 * D, at, ACTF_NONE, false);
    {
        const int hd = D / heads;
        const size_t es = dsize(at);
        const float scale = 1.0f / sqrtf((float)hd);
        Prof p(c.m->ocl, "attention");
        if (at != DT_BF16 || !attention_tc(c.st, I->t_qkv, N, D, heads, I->t_o, D, scale,
                                           nimg))
            for (int k = 0; k < nimg; k++) {
                const char *q = (const char *)I->t_qkv + (size_t)k * N * 3 * D * es;
                attention_l(c.st, q, 3 * D, q + D * es, 3 * D, q + 2 * D * es, 3 * D,
                            (char *)I->t_o + (size_t)k * N * D * es, D, N, N, heads, hd,
                            scale, nullptr, at);
            }
        launch_ok("attention");
    }
    gemm_nt(c, "proj", rows, D, D, I->t_o, D, at, b.proj_w, b.proj_b, I->t_x, D,
            DT_F32, ACTF_NONE, true);
    {
        Prof p(c.m->ocl, "layernorm");
        layernorm_rows(c.st, I->t_x, I->t_n, at, b.n2g, b.n2b, rows, D, eps,
                       ACTF_NONE, 0.0f);
    }
    gemm_nt(c, "fc1", rows, MLP_RATIO * D, D, I->t_n, D, at, b.fc1_w, b.fc1_b,
            I->t_h, MLP_RATIO * D, at, ACTF_GELU, false);
    gemm_nt(c, "fc2", rows, D, MLP_RATIO * D, I->t_h, MLP_RATIO * D, at, b.fc2_w,
            b.fc2_b, I->t_x, D, DT_F32, ACTF_NONE, true);
}

// DINOv2 on img (Cs x Cs, channels-last): the normalized patch tokens,
// projected (decoder.proj.16), into P[0][k] (roma.c:717-738).
// The 14 x 14 patches of a channels-last (H, W, 3) bfloat16 image as rows
// of kp columns, column k = (c, ky, kx) (the PyTorch weight order), zero
// from 588 on. One thread per 8 columns: one 16-byte store.
__global__ void patch_rows_k(const __nv_bfloat16 *img, int H, int W, int kp,
                             __nv_bfloat16 *rows)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    const int chunks = kp / 8, pw = W / ROMA_PATCH;
    const long np = (long)(H / ROMA_PATCH) * pw;
    if (e >= np * chunks)
        return;
    const long m = e / chunks;
    const int j0 = (int)(e % chunks) * 8;
    const int py = (int)(m / pw), px = (int)(m % pw);
    constexpr int PP = ROMA_PATCH * ROMA_PATCH;
    __align__(16) __nv_bfloat16 v[8];
#pragma unroll
    for (int q = 0; q < 8; q++) {
        const int k = j0 + q;
        __nv_bfloat16 x = __float2bfloat16_rn(0.0f);
        if (k < 3 * PP) {
            const int ch = k / PP, r = k % PP;
            const int yy = py * ROMA_PATCH + r / ROMA_PATCH, xx = px * ROMA_PATCH + r % ROMA_PATCH;
            x = img[((long)yy * W + xx) * 3 + ch];
        }
        v[q] = x;
    }
    *(uint4 *)(rows + m * kp + j0) = *(const uint4 *)v;
}

// Patch and position embedding of image k's prepared input (img) into
// token rows k ntok .. of t_x: class token, then the 14 x 14 patches.
void dino_embed(Ctx &c, int k)
{
    roma_impl *I = c.I;
    const int D = ROMA_VIT_DIM, N16 = I->n16;
    float *x = I->t_x + (size_t)k * I->ntok * D;
    if (I->patch_kp) {
        // bfloat16: the patches gathered into rows, then the tensor cores.
        const int kp = I->patch_kp;
        patch_rows_k<<<cdiv((long)N16 * (kp / 8), 256), 256, 0, c.st>>>(
            (const __nv_bfloat16 *)I->img, I->Cs, I->Cs, kp, I->patch_col);
        GemmArgs g = gemm_args(N16, D, kp);
        g.A = I->patch_col;
        g.lda = kp;
        g.B = I->patch_w;
        g.ldb = kp;
        g.transb = 1;
        g.C = x + D;
        g.ldc = D;
        g.bias = I->patch_b;
        g.R = I->pos + D;
        g.ab = DT_BF16;
        g.c = DT_F32;
        gemm_run(c.m->ocl, g, "patch_embed");
        cls_pos_k<<<cdiv(D, 256), 256, 0, c.st>>>(x, I->cls, I->pos, D);
        return;
    }
    GemmArgs g = gemm_args(N16, D, 3 * ROMA_PATCH * ROMA_PATCH);
    g.A = I->img;
    g.amode = 2;
    g.cH = I->Cs;
    g.cW = I->Cs;
    g.cC = 3;
    g.cP = ROMA_PATCH;
    g.B = I->patch_w;
    g.ldb = 3 * ROMA_PATCH * ROMA_PATCH;
    g.transb = 1;
    g.C = x + D;
    g.ldc = D;
    g.bias = I->patch_b;
    g.R = I->pos + D;
    g.ab = I->at;
    g.c = DT_F32;
    gemm_run(c.m->ocl, g, "patch_embed");
    cls_pos_k<<<cdiv(D, 256), 256, 0, c.st>>>(x, I->cls, I->pos, D);
}

// DINOv2's 24 blocks over both images' tokens at once, the final norm, and
// per image the dump point and the projection into P[0] (roma.c:717-738).
void dino(Ctx &c)
{
    roma_impl *I = c.I;
    const int D = ROMA_VIT_DIM, N16 = I->n16, NT = I->ntok;
    for (int i = 0; i < ROMA_VIT_DEPTH; i++)
        block(c, I->vit[i], NT, 2, D, VIT_HEADS, EPS_LN_VIT);
    {
        Prof p(c.m->ocl, "layernorm");
        layernorm_rows(c.st, I->t_x, I->t_n, I->at, I->norm_g, I->norm_b, 2 * NT, D,
                       EPS_LN_VIT, ACTF_NONE, 0.0f);
    }
    for (int k = 0; k < 2; k++) {
        const void *tok = (const char *)I->t_n + ((size_t)k * NT + 1) * D * dsize(I->at);
        dump_dev(c, k ? "dino_1" : "dino_0", tok, I->at, (size_t)N16 * D, N16, D);
        gemm_nt(c, "proj16", N16, GP_DIM, D, tok, D, I->at, I->proj_w[0], I->proj_b[0],
                I->P[0][k], GP_DIM, DT_F32, ACTF_NONE, false);
    }
}

// x = hi + lo with hi, lo bfloat16 (hi = x rounded, lo = the rest
// rounded): the A form [hi | hi | lo] and the B form [hi | lo | hi] of an n x
// d float matrix, so that A3 B3^T = hi hi' + hi lo' + lo hi', the float
// product up to the lo lo' term and the rounding of lo (relative 2^-16).
__global__ void split3_k(const float *x, long n, int d, __nv_bfloat16 *a3, __nv_bfloat16 *b3)
{
    const long e = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n * d)
        return;
    const long r = e / d;
    const int c = (int)(e % d);
    const float v = x[e];
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
    __nv_bfloat16 *ra = a3 + r * 3 * d, *rb = b3 ? b3 + r * 3 * d : nullptr;
    ra[c] = hi;
    ra[d + c] = hi;
    ra[2 * d + c] = lo;
    if (rb) {
        rb[c] = hi;
        rb[d + c] = lo;
        rb[2 * d + c] = hi;
    }
}

// The same split of the transpose of a float n x d matrix x (row k, column
// j): row j of b3 is [hi, lo, hi] of column j of x, so that a3 b3^T with
// a3 = split3_k's [hi, hi, lo] rows of another matrix is that matrix times
// x. 32 x 32 tiles through shared memory: coalesced reads along j, writes
// along k.
__global__ void split3t_k(const float *x, int n, int d, __nv_bfloat16 *b3)
{
    __shared__ float t[32][33];
    const int k0 = blockIdx.y * 32, j0 = blockIdx.x * 32;
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int k = k0 + r, j = j0 + threadIdx.x;
        t[r][threadIdx.x] = k < n && j < d ? x[(long)k * d + j] : 0.0f;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += 8) {
        const int j = j0 + r, k = k0 + threadIdx.x;
        if (j >= d || k >= n)
            continue;
        const float v = t[threadIdx.x][r];
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
        __nv_bfloat16 *rb = b3 + (long)j * 3 * n;
        rb[k] = hi;
        rb[n + k] = lo;
        rb[2 * n + k] = hi;
    }
}

// Gaussian-process posterior of A's 1/16 features given B's and the
// position basis, into t_x columns 0..511, A's features in 512..1023
// (roma.c:873-896), the solve on the device in double. In bfloat16 mode the
// two kernel matrices' products (cosines of normalized features) and the
// posterior product K_xy X run on the tensor cores as three-term bfloat16
// splits (K = 3 x 512 and 3 n; the split K_xy is staged in the qkv buffer,
// free between the encoder and the decoder); float32 mode keeps the float32
// products.
void gp(Ctx &c)
{
    roma_impl *I = c.I;
    const int n = I->n16;
    const float *ya = (const float *)I->P[0][0], *yb = (const float *)I->P[0][1];
    {
        Prof p(c.m->ocl, "gp_kernel");
        roma_row_norm_l(c.st, ya, n, GP_DIM, I->g_nx);
        roma_row_norm_l(c.st, yb, n, GP_DIM, I->g_ny);
    }
    if (I->at == DT_BF16) {
        {
            Prof p(c.m->ocl, "gp_kernel");
            const long e = (long)n * GP_DIM;
            split3_k<<<cdiv(e, 256), 256, 0, c.st>>>(yb, n, GP_DIM, I->g_s3[1], I->g_s3[2]);
            split3_k<<<cdiv(e, 256), 256, 0, c.st>>>(ya, n, GP_DIM, I->g_s3[0], nullptr);
            launch_ok("gp_kernel");
        }
        gemm_nt(c, "gp_gemm", n, n, 3 * GP_DIM, I->g_s3[1], 3 * GP_DIM, DT_BF16, I->g_s3[2],
                nullptr, I->g_kyy, n, DT_F32, ACTF_NONE, false);
        gemm_nt(c, "gp_gemm", n, n, 3 * GP_DIM, I->g_s3[0], 3 * GP_DIM, DT_BF16, I->g_s3[2],
                nullptr, I->g_kxy, n, DT_F32, ACTF_NONE, false);
    }
    else {
        gemm_nt(c, "gp_gemm", n, n, GP_DIM, yb, GP_DIM, DT_F32, yb, nullptr, I->g_kyy,
                n, DT_F32, ACTF_NONE, false);
        gemm_nt(c, "gp_gemm", n, n, GP_DIM, ya, GP_DIM, DT_F32, yb, nullptr, I->g_kxy,
                n, DT_F32, ACTF_NONE, false);
    }
    {
        Prof p(c.m->ocl, "gp_kernel");
        roma_cos_exp_l(c.st, I->g_kyy, I->g_ny, I->g_ny, n, n, GP_T, COS_EPS);
        roma_cos_exp_l(c.st, I->g_kxy, I->g_nx, I->g_ny, n, n, GP_T, COS_EPS);
    }
    {
        Prof p(c.m->ocl, "gp_cholesky");
        gp_solve_dev(c.st, I->g_kyy, n, I->gp_basis, GP_DIM, GP_NOISE, I->g_x,
                     I->gp_work, I->gp_flag);
        launch_ok("gp_cholesky");
    }
    if (I->at == DT_BF16 && (size_t)6 * n * n <= I->t_qkv_bytes && n % 8 == 0) {
        __nv_bfloat16 *a3 = (__nv_bfloat16 *)I->t_qkv, *b3 = I->g_s3[0];
        {
            Prof p(c.m->ocl, "gp_kernel");
            const long e = (long)n * n;
            split3_k<<<cdiv(e, 256), 256, 0, c.st>>>(I->g_kxy, n, n, a3, nullptr);
            split3t_k<<<dim3(cdiv(GP_DIM, 32), cdiv(n, 32)), dim3(32, 8), 0, c.st>>>(
                (const float *)I->g_x, n, GP_DIM, b3);
            launch_ok("gp_kernel");
        }
        gemm_nt(c, "gp_gemm", n, GP_DIM, 3 * n, a3, 3 * n, DT_BF16, b3, nullptr, I->t_x,
                ROMA_DEC_DIM, DT_F32, ACTF_NONE, false);
    }
    else {
        GemmArgs g = gemm_args(n, GP_DIM, n);
        g.A = I->g_kxy;
        g.lda = n;
        g.B = I->g_x;
        g.ldb = GP_DIM;
        g.transb = 0;
        g.C = I->t_x;
        g.ldc = ROMA_DEC_DIM;
        g.ab = DT_F32;
        g.c = DT_F32;
        gemm_run(c.m->ocl, g, "gp_gemm");
    }
    copy2d(c.st, ya, DT_F32, GP_DIM, I->t_x + GP_DIM, DT_F32, ROMA_DEC_DIM, n,
           GP_DIM);
    if (c.dump) {
        std::vector<float> mu((size_t)n * GP_DIM);
        cudaStreamSynchronize(c.st);
        cudaMemcpy2D(mu.data(), GP_DIM * 4, I->t_x, ROMA_DEC_DIM * 4, GP_DIM * 4, n,
                     cudaMemcpyDeviceToHost);
        dump_host(c, "gp", mu.data(), mu.size());
    }
}

// Coordinate decoder on t_x: coarse warp and certainty logit into fl[0],
// ce[0] (roma.c:900-919).
void decoder(Ctx &c)
{
    roma_impl *I = c.I;
    const int n = I->n16, D = ROMA_DEC_DIM;
    for (int i = 0; i < ROMA_DEC_DEPTH; i++)
        block(c, I->dec[i], n, 1, D, DEC_HEADS, EPS_LN_DEC);
    const void *x = I->t_x;
    if (I->at != DT_F32) {
        copy2d(c.st, I->t_x, DT_F32, D, I->t_n, I->at, D, n, D);
        x = I->t_n;
    }
    gemm_nt(c, "to_out", n, NCLS + 1, D, x, D, I->at, I->to_out_w, I->to_out_b,
            I->t_out, NCLS + 1, DT_F32, ACTF_NONE, false);
    // The anchor logits and the certainty logit, token-major (n x 4097):
    // an extra dump point, so that a check can tell the tokens whose
    // first-index argmax is a near-tie from kernel error.
    dump_dev(c, "cls_logits", I->t_out, DT_F32, (size_t)n * (NCLS + 1));
    Prof p(c.m->ocl, "roma_cls_to_flow");
    roma_cls_to_flow_l(c.st, I->t_out, NCLS + 1, NCLS, ROMA_CLS_RES, n, I->fl[0],
                       I->ce[0]);
    launch_ok("roma_cls_to_flow");
}

// Refiner input d = (f_A, f_B at the warp, displacement embedding, local
// correlation) on an hs x ws grid, then the 9 blocks and the output
// convolution into d_c (n x nout).
void refiner_body(Ctx &c, const Refiner &r, const void *fa, const void *fb,
                  DType tf, int hs, int ws, float dfx, float dfy,
                  const float *flow)
{
    roma_impl *I = c.I;
    const long n = (long)hs * ws;
    const DType at = I->at;
    {
        Prof p(c.m->ocl, "refiner_input");
        if (r.cinp != r.cin) {
            const size_t es = dsize(at);
            cudaMemset2DAsync((char *)I->d_a + r.cin * es, r.cinp * es, 0,
                              (r.cinp - r.cin) * es, n, c.st);
        }
        copy2d(c.st, fa, tf, r.fpitch, I->d_a, at, r.cinp, n, r.feat);
        roma_warp_sample_l(c.st, {fb, 1, r.fpitch, tf}, r.feat, hs, ws, flow,
                           {I->d_a, 1, r.cinp, at}, r.feat);
        roma_disp_emb_l(c.st, flow, hs, ws, dfx, dfy, r.emb_w, r.emb_b, r.emb,
                        {I->d_a, 1, r.cinp, at}, 2 * r.feat);
        launch_ok("refiner_input");
    }
    if (r.radius) {
        Prof p(c.m->ocl, "roma_local_corr");
        roma_local_corr_l(c.st, {fa, 1, r.fpitch, tf}, {fb, 1, r.fpitch, tf}, r.feat, hs,
                          ws, r.radius, flow, {I->d_a, 1, r.cinp, at},
                          2 * r.feat + r.emb);
        launch_ok("roma_local_corr");
    }
    // Blocks: in bfloat16 mode at the widths the fused tensor-core kernel
    // takes, one kernel per block ping-ponging between d_a and d_b;
    // otherwise the depthwise kernel into d_b and the product back into d_a.
    void *x = I->d_a, *y = I->d_b;
    const bool fused = at == DT_BF16 && (r.cinp == 32 || r.cinp == 64 || r.cinp == 128);
    for (int b = 0; b <= ROMA_HIDDEN; b++) {
        if (fused) {
            Prof p(c.m->ocl, "refiner_block");
            if (!dwpw_tc(c.st, x, hs, ws, r.cinp, r.dw_w[b], r.dw_b[b], r.pw_w[b], r.pw_b[b],
                         y, c.m->ocl->sm_count)) {
                fail("refiner block: the fused kernel could not be launched");
                return;
            }
            launch_ok("refiner_block");
            std::swap(x, y);
            continue;
        }
        {
            Prof p(c.m->ocl, "roma_dwconv5");
            roma_dwconv5_l(c.st, {x, 1, r.cinp, at}, r.cinp, hs, ws, r.dw_w[b], r.dw_b[b],
                           {y, 1, r.cinp, at});
            launch_ok("roma_dwconv5");
        }
        gemm_nt(c, "refiner_pw", (int)n, r.cinp, r.cinp, y, r.cinp, at, r.pw_w[b], r.pw_b[b],
                x, r.cinp, at, ACTF_NONE, false);
    }
    gemm_nt(c, "refiner_out", (int)n, r.nout, r.cinp, x, r.cinp, at, r.out_w, r.out_b,
            I->d_c, DC_PITCH, DT_F32, ACTF_NONE, false);
}

// ConvRefiner s on an hs x ws grid of a pass of size Hf x Wf (scale
// factor sf): updates the warp fl and certainty ce (roma.c:923-995).
void refine(Ctx &c, int s, int hs, int ws, int Hf, int Wf, float sf, float *fl,
            float *ce)
{
    roma_impl *I = c.I;
    const Refiner &r = I->ref[s];
    const float fac = 40.0f / 32.0f * sf;
    const DType tf = s == 0 ? DT_F32 : I->at;
    refiner_body(c, r, I->P[s][0], I->P[s][1], tf, hs, ws, fac, fac, fl);
    Prof p(c.m->ocl, "roma_update");
    roma_update_l(c.st, fl, ce, {I->d_c, 1, DC_PITCH, DT_F32}, hs * ws,
                  (float)r.scale, (float)Wf, (float)Hf);
    launch_ok("roma_update");
}

// RoMa v2's refiner j (roma.c:1033-1104).
void refine2(Ctx &c, int j, int hs, int ws, int Hp, int Wp, float *fl, float *cf)
{
    roma_impl *I = c.I;
    const Refiner &r = I->ref2[j];
    refiner_body(c, r, I->P2[j][0], I->P2[j][1], I->at, hs, ws,
                 (float)Wp / ROMA2_ANCHOR, (float)Hp / ROMA2_ANCHOR, fl);
    Prof p(c.m->ocl, "roma2_update");
    roma2_update_l(c.st, fl, cf, {I->d_c, 1, DC_PITCH, DT_F32}, hs * ws, (float)ws,
                   (float)hs);
    launch_ok("roma2_update");
}

void resize(Ctx &c, const float *in, int C, int h, int w, float *out, int H,
            int W)
{
    Prof p(c.m->ocl, "resize_bilinear");
    resize_planes(c.st, in, C, h, w, out, H, W, 0, 0, 0.0f);
    launch_ok("resize_bilinear");
}

// RoMa's refiners s0 .. s1 - 1 of pass p (size Hp x Wp), resized between
// scales (roma.c:1232-1256).
void refiners(Ctx &c, int p, int s0, int s1, int Hp, int Wp, float sf, int *cur)
{
    roma_impl *I = c.I;
    for (int s = s0; s < s1; s++) {
        const int hs = side(I, Hp, s), ws = side(I, Wp, s);
        refine(c, s, hs, ws, Hp, Wp, sf, I->fl[*cur], I->ce[*cur]);
        if (p == 0 && s == 0)
            cudaMemcpyAsync(I->cert16, I->ce[*cur], (size_t)hs * ws * 4,
                            cudaMemcpyDeviceToDevice, c.st);
        if (c.dump) {
            char what[64];
            snprintf(what, sizeof(what), "p%d_s%d_flow", p, ref_scale[s]);
            dump_dev(c, what, I->fl[*cur], DT_F32, 2 * (size_t)hs * ws);
            snprintf(what, sizeof(what), "p%d_s%d_cert", p, ref_scale[s]);
            dump_dev(c, what, I->ce[*cur], DT_F32, (size_t)hs * ws);
        }
        if (s < s1 - 1) {
            const int hn = side(I, Hp, s + 1), wn = side(I, Wp, s + 1);
            resize(c, I->fl[*cur], 2, hs, ws, I->fl[!*cur], hn, wn);
            resize(c, I->ce[*cur], 1, hs, ws, I->ce[!*cur], hn, wn);
            *cur = !*cur;
        }
    }
}

// RoMa v2's refiners of pass p from the warp and confidence on the
// current h x w grid; zero_prec clears the precision first
// (roma.c:1272-1301).
void refiners2(Ctx &c, int p, int Hp, int Wp, int *h, int *w, int *cur,
               int zero_prec)
{
    roma_impl *I = c.I;
    for (int j = 0; j < ROMA2_SCALES; j++) {
        const int hs = Hp / ref2_scale[j], ws = Wp / ref2_scale[j];
        const size_t n = (size_t)*h * *w;
        if (zero_prec && j == 0)
            cudaMemsetAsync(I->cf[*cur] + n, 0, 3 * n * 4, c.st);
        resize(c, I->fl[*cur], 2, *h, *w, I->fl[!*cur], hs, ws);
        resize(c, I->cf[*cur], 4, *h, *w, I->cf[!*cur], hs, ws);
        *cur = !*cur;
        refine2(c, j, hs, ws, Hp, Wp, I->fl[*cur], I->cf[*cur]);
        if (c.dump) {
            char what[64];
            snprintf(what, sizeof(what), "p%d_v2s%d_flow", p, ref2_scale[j]);
            dump_dev(c, what, I->fl[*cur], DT_F32, 2 * (size_t)hs * ws);
            snprintf(what, sizeof(what), "p%d_v2s%d_conf", p, ref2_scale[j]);
            dump_dev(c, what, I->cf[*cur], DT_F32, 4 * (size_t)hs * ws);
        }
        *h = hs;
        *w = ws;
    }
}

void dump_input(Ctx &c, const char *what, int h, int w)
{
    // img is channels-last (h, w, 3): the reference dumps (3, h, w).
    dump_dev(c, what, c.I->img, c.I->at, 3 * (size_t)h * w, (long)h * w, 3);
}

void run_tile(Ctx &c, const float *inA, const float *inB)
{
    struct roma_model *m = c.m;
    roma_impl *I = c.I;
    const int H = m->H, W = m->W, Cs = I->Cs;
    const size_t hw = (size_t)H * W;
    const float *in[2] = {inA, inB};
    int cur = 0;
    bool need[ROMA_SCALES] = {false, false, false, false, false};
    for (int s = 1; s < ROMA_SCALES; s++)
        need[s] = !m->v2 || s == 1;

    // Coarse pass.
    for (int k = 0; k < 2; k++) {
        prepare(c, in[k], H, W, I->pil_cx, I->pil_cy);
        dump_input(c, k ? "in_c_1" : "in_c_0", Cs, Cs);
        vgg(c, Cs, Cs, k, need);
        if (m->v2)
            vgg2(c, Cs, Cs, k);
        dino_embed(c, k);
    }
    dino(c);
    gp(c);
    decoder(c);
    if (c.dump) {
        dump_dev(c, "cls_flow", I->fl[0], DT_F32, 2 * (size_t)I->n16);
        dump_dev(c, "cls_cert", I->ce[0], DT_F32, I->n16);
    }
    refiners(c, 0, 0, m->v2 ? 2 : ROMA_SCALES, Cs, Cs, 1.0f, &cur);

    if (m->v2) {
        // match_v2 (roma.c:1308-1355).
        int h = side(I, Cs, 1), w = side(I, Cs, 1);
        const size_t n = (size_t)h * w;
        cudaMemsetAsync(I->cf[cur], 0, 4 * n * 4, c.st);
        cudaMemcpyAsync(I->cf[cur], I->ce[cur], n * 4, cudaMemcpyDeviceToDevice,
                        c.st);
        refiners2(c, 0, Cs, Cs, &h, &w, &cur, 0);
        for (int k = 0; k < 2; k++) {
            prepare(c, in[k], H, W, I->pil_fx, I->pil_fy);
            dump_input(c, k ? "in_f_1" : "in_f_0", H, W);
            vgg2(c, H, W, k);
        }
        refiners2(c, 1, H, W, &h, &w, &cur, 1);
        cudaMemcpyAsync(I->o_flow, I->fl[cur], 2 * hw * 4, cudaMemcpyDeviceToDevice,
                        c.st);
        cudaMemcpyAsync(I->o_cert, I->cf[cur], hw * 4, cudaMemcpyDeviceToDevice,
                        c.st);
        Prof p(m->ocl, "roma_finish");
        roma_finish_l(c.st, I->o_flow, I->o_cert, I->cf[cur] + hw, nullptr, I->o_sd,
                      (long)hw);
        launch_ok("roma_finish");
        return;
    }
    // Fine pass at the tile's size from the coarse pass's finest warp
    // (roma.c:1395-1434).
    bool needf[ROMA_SCALES] = {false, true, true, true, true};
    for (int k = 0; k < 2; k++) {
        prepare(c, in[k], H, W, I->pil_fx, I->pil_fy);
        dump_input(c, k ? "in_f_1" : "in_f_0", H, W);
        vgg(c, H, W, k, needf);
    }
    resize(c, I->fl[cur], 2, Cs, Cs, I->fl[!cur], side(I, H, 1), side(I, W, 1));
    resize(c, I->ce[cur], 1, Cs, Cs, I->ce[!cur], side(I, H, 1), side(I, W, 1));
    cur = !cur;
    refiners(c, 1, 1, ROMA_SCALES, H, W, sqrtf((float)H * W) / Cs, &cur);
    resize(c, I->cert16, 1, I->c16, I->c16, I->lowres, H, W);
    cudaMemcpyAsync(I->o_flow, I->fl[cur], 2 * hw * 4, cudaMemcpyDeviceToDevice,
                    c.st);
    cudaMemcpyAsync(I->o_cert, I->ce[cur], hw * 4, cudaMemcpyDeviceToDevice, c.st);
    Prof p(m->ocl, "roma_finish");
    roma_finish_l(c.st, I->o_flow, I->o_cert, nullptr, I->lowres, nullptr, (long)hw);
    launch_ok("roma_finish");
}

bool ready(struct roma_model *m)
{
    if (pending())
        return false;
    if (!m->impl || !m->impl->alloc_done) {
        fail("RoMa: roma_match before roma_alloc");
        return false;
    }
    return true;
}

}  // namespace

namespace {

// The tile over the device images inA, inB captured into *graph and
// instantiated into *exec (both replaced); the kernel count, or -1 after
// recording an error.
int capture_tile(struct roma_model *m, const float *inA, const float *inB, cudaGraph_t *graph,
                 cudaGraphExec_t *exec)
{
    roma_impl *I = m->impl;
    cudaStream_t st = stream_of(m->ocl);
    if (*exec) {
        cudaGraphExecDestroy(*exec);
        *exec = nullptr;
    }
    if (*graph) {
        cudaGraphDestroy(*graph);
        *graph = nullptr;
    }
    if (!cuda_ok(cudaStreamSynchronize(st), "RoMa graph capture") ||
        !cuda_ok(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal),
                 "cudaStreamBeginCapture"))
        return -1;
    Ctx c{m, I, st, nullptr, 0};
    run_tile(c, inA, inB);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(st, &g);
    if (pending() || !cuda_ok(e, "cudaStreamEndCapture")) {
        if (g)
            cudaGraphDestroy(g);
        return -1;
    }
    *graph = g;
    if (!cuda_ok(cudaGraphInstantiate(exec, g, 0), "cudaGraphInstantiate"))
        return -1;
    size_t n = 0;
    cudaGraphGetNodes(g, nullptr, &n);
    std::vector<cudaGraphNode_t> nodes(n);
    cudaGraphGetNodes(g, nodes.data(), &n);
    int kernels = 0;
    for (auto nd : nodes) {
        cudaGraphNodeType t;
        cudaGraphNodeGetType(nd, &t);
        kernels += t == cudaGraphNodeTypeKernel;
    }
    return kernels;
}

}  // namespace

extern "C" void roma_match_dev(struct roma_model *m, const float *imgA,
                               const float *imgB)
{
    if (!ready(m))
        return;
    cudaSetDevice(m->ocl->device);
    Ctx c{m, m->impl, stream_of(m->ocl), nullptr, 0};
    run_tile(c, imgA, imgB);
}

extern "C" void roma_results_dev(struct roma_model *m, float **flow,
                                 float **cert, float **sd)
{
    roma_impl *I = m->impl;
    if (flow)
        *flow = I ? I->o_flow : nullptr;
    if (cert)
        *cert = I ? I->o_cert : nullptr;
    if (sd)
        *sd = I && m->v2 ? I->o_sd : nullptr;
}

extern "C" int roma_sync(struct roma_model *m)
{
    int flag = 0;
    if (!ready(m))
        return -1;
    cudaSetDevice(m->ocl->device);
    if (!cuda_ok(cudaStreamSynchronize(stream_of(m->ocl)), "roma_sync"))
        return -1;
    cudaMemcpy(&flag, m->impl->gp_flag, sizeof(int), cudaMemcpyDeviceToHost);
    if (flag) {
        cudaMemset(m->impl->gp_flag, 0, sizeof(int));
        fail("RoMa: Gaussian process kernel not positive definite");
        return 1;
    }
    return 0;
}

extern "C" void roma_match(struct roma_model *m, const float *imgA,
                           const float *imgB, const char *dump, int tile)
{
    if (!ready(m))
        return;
    cudaSetDevice(m->ocl->device);
    roma_impl *I = m->impl;
    cudaStream_t st = stream_of(m->ocl);
    const size_t hw = (size_t)m->H * m->W;
    if (!cuda_ok(cudaMemcpyAsync(I->in_dev[0], imgA, 3 * hw * 4,
                                 cudaMemcpyHostToDevice, st),
                 "roma_match input") ||
        !cuda_ok(cudaMemcpyAsync(I->in_dev[1], imgB, 3 * hw * 4,
                                 cudaMemcpyHostToDevice, st),
                 "roma_match input"))
        return;
    Ctx c{m, I, st, dump && *dump ? dump : nullptr, tile};
    if (c.dump || m->ocl->profile) {
        // Dumps read back between stages, and profiling times each
        // launch: the tile runs launch by launch.
        run_tile(c, I->in_dev[0], I->in_dev[1]);
    }
    else {
        // Otherwise one launch of the tile's graph over in_dev (captured on
        // the first such call, again if m->imagenet changed): the host
        // issues one launch instead of the tile's several hundred.
        if (!I->match_exec || I->match_imagenet != m->imagenet) {
            if (capture_tile(m, I->in_dev[0], I->in_dev[1], &I->match_graph, &I->match_exec) <
                0)
                return;
            I->match_imagenet = m->imagenet;
        }
        if (!cuda_ok(cudaGraphLaunch(I->match_exec, st), "cudaGraphLaunch"))
            return;
    }
    cudaMemcpyAsync(m->flow, I->o_flow, 2 * hw * 4, cudaMemcpyDeviceToHost, st);
    cudaMemcpyAsync(m->cert, I->o_cert, hw * 4, cudaMemcpyDeviceToHost, st);
    if (m->v2)
        cudaMemcpyAsync(m->sd, I->o_sd, hw * 4, cudaMemcpyDeviceToHost, st);
    if (roma_sync(m) != 0)
        return;
    if (c.dump) {
        dump_host(c, "flow", m->flow, 2 * hw);
        dump_host(c, "cert", m->cert, hw);
        if (m->v2)
            dump_host(c, "sd", m->sd, hw);
    }
}

extern "C" int roma_graph_build(struct roma_model *m, const float *imgA,
                                const float *imgB)
{
    if (!ready(m))
        return -1;
    cudaSetDevice(m->ocl->device);
    return capture_tile(m, imgA, imgB, &m->impl->graph, &m->impl->graph_exec);
}

extern "C" void roma_graph_launch(struct roma_model *m)
{
    if (!ready(m))
        return;
    if (!m->impl->graph_exec) {
        fail("RoMa: roma_graph_launch before roma_graph_build");
        return;
    }
    cudaSetDevice(m->ocl->device);
    cuda_ok(cudaGraphLaunch(m->impl->graph_exec, stream_of(m->ocl)),
            "cudaGraphLaunch");
}

extern "C" void *coreg_host_alloc(size_t bytes)
{
    void *p = nullptr;
    if (pending())
        return nullptr;
    if (!cuda_ok(cudaMallocHost(&p, bytes ? bytes : 16), "cudaMallocHost"))
        return nullptr;
    return p;
}

extern "C" void coreg_host_free(void *p)
{
    if (p)
        cudaFreeHost(p);
}
