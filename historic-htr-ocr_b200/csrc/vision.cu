// vision.cu — the host side of the vision encoder + projector behind ocr_cuda.h: the seeded synthetic q8_0 weights
// (with the tensor cores' tile-major copies), the bake's plan, and the encode: patch gather → patch embedding →
// pre_ln → n_layer × [ln1 → qkv → 2D RoPE (+ K / V f16 head-major) → full attention → o (+ residual) → ln2 →
// gate|up with SwiGLU → down (+ residual)] → input_norm + 2x2 unfold → merger → mm.1 → GELU → mm.2.
//
// Every matrix product runs on the tensor-core contraction (k_bgemm.cu) over the rows in groups of 32 (two groups per
// CTA), with the operand split exactly into f16 hi + lo; the attention is the full-attention form of the tcgen05
// attention (k_attn_prefill_tc.cu). One stream, no host round trip between kernels.
//
// Reference (b-straub/historic-htr-ocr): Vision (app/crates/ocr-wgpu/src/vision.rs:37-450): VisionConfig 37-88,
// pixel_lut 152-155, rope_table 159-175, grid 241-249, run 266-317, project 405-423; the bake's plan
// (app/crates/ocr-core/src/imageops.rs:275-316).
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>
#include <string>
#include <vector>

#include "ctx.h"
#include "kernels.cuh"

using namespace ocr;

namespace {

struct VLayer {
    QMat qkv, o, gu, down;  // qkv rows [q | k | v]; gu rows interleaved (gate 0, up 0, gate 1, …)
    BgMaps bq_qkv, bq_o, bq_gu, bq_down;
    float *ln1 = nullptr, *ln2 = nullptr;
};

// tensor kinds of one layer in the synthetic generator's numbering (sub-stream 200000 + layer * 16 + kind)
enum { VK_LN1 = 0, VK_Q, VK_K, VK_V, VK_O, VK_LN2, VK_GATE, VK_UP, VK_DOWN };
constexpr uint64_t V_LAYER_STREAM = 200000, V_PATCH_STREAM = 300000, V_PRE_LN_STREAM = 300001,
                   V_INPUT_NORM_STREAM = 300002, V_MERGER_STREAM = 300003, V_MM1_STREAM = 300004,
                   V_MM2_STREAM = 300005;

uint64_t substream(uint64_t seed, uint64_t k) {
    uint64_t z = (seed ^ 0x6F63722D62323030ull) + (k + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

int patch_cols(const ocr_vision_cfg& c) { return (3 * c.patch * c.patch + 255) / 256 * 256; }

}  // namespace

struct ocr_vision {
    ocr_ctx* ctx = nullptr;
    ocr_vision_cfg cfg{};
    int pcols = 0;
    void* mem = nullptr;  // the weights, their tile-major copies, the norms, the pixel LUT
    size_t mem_bytes = 0;
    std::vector<VLayer> layers;
    QMat patch, merger, mm1, mm2;
    BgMaps bq_patch, bq_merger, bq_mm1, bq_mm2;
    float *pre_ln = nullptr, *input_norm = nullptr, *lut = nullptr;
    void* work = nullptr;  // the encode's buffers, grown for the largest image seen
    size_t work_bytes = 0;
};

namespace {

ocr_status check_vcfg(const ocr_vision_cfg& c) {
    if (c.n_layer < 0 || c.dim <= 0 || c.n_head <= 0 || c.n_ff <= 0 || c.patch <= 0 || c.proj_dim <= 0)
        return fail(OCR_ERR_ARG, "vision config: sizes must be positive");
    if (c.dim % c.n_head != 0 || c.dim / c.n_head != 64)
        return fail(OCR_ERR_ARG, "head dim " + std::to_string(c.dim) + "/" + std::to_string(c.n_head) +
                                     ": the attention kernel is written for 64");
    if (c.merge != 2 || c.n_ff < 4 * c.dim) return fail(OCR_ERR_ARG, "merge / n_ff: the unfold is 2x2 (n_ff >= 4 dim)");
    if (3 * c.patch * c.patch > 4096) return fail(OCR_ERR_ARG, "patch too large");
    if (!bgemm_shape_ok(3 * c.dim, c.dim) || !bgemm_shape_ok(c.dim, c.n_ff) || !bgemm_shape_ok(2 * c.n_ff, c.dim) ||
        !bgemm_shape_ok(c.dim, 4 * c.dim) || !bgemm_shape_ok(c.proj_dim, c.proj_dim))
        return fail(OCR_ERR_ARG, "vision config: the contraction takes widths that are multiples of 256, at most 4096");
    if (!(c.eps > 0.0f) || !(c.rope_theta > 0.0f)) return fail(OCR_ERR_ARG, "vision config: eps and rope_theta > 0");
    for (int i = 0; i < 3; i++)
        if (!(c.std[i] != 0.0f)) return fail(OCR_ERR_ARG, "vision config: std must be non-zero");
    return OCR_OK;
}

// a bump allocator over one device allocation: 256-B aligned offsets
struct Plan {
    size_t off = 0;
    size_t take(size_t n) {
        const size_t o = off;
        off += (n + 255) / 256 * 256;
        return o;
    }
};

// the encode's buffers for n patches (n_out merged tokens) and the image's bytes
struct Work {
    float *x, *h, *qkv, *rope, *out;
    __half *kh, *vh;
    uint8_t *x16a, *x16o, *x16g, *rgb;
    int n_pad;
};

size_t work_layout(const ocr_vision_cfg& c, int pcols, int n, int max_pos, size_t rgb_bytes, Work* w,
                   uint8_t* base) {
    Plan p;
    const int groups = (n + BG_SLOTS - 1) / BG_SLOTS, n_pad = (n + 63) / 64 * 64;
    const size_t gr = (size_t)groups * BG_SLOTS;
    const size_t o_x = p.take(gr * c.dim * 4), o_h = p.take(gr * std::max(c.dim, c.proj_dim) * 4);
    const size_t o_qkv = p.take(gr * 3 * c.dim * 4);
    const size_t o_rope = p.take((size_t)2 * max_pos * (c.dim / c.n_head / 4) * 2 * 4);
    const size_t o_out = p.take(gr * std::max(c.dim, c.proj_dim) * 4);
    const size_t o_kh = p.take((size_t)c.n_head * n_pad * (c.dim / c.n_head) * 2);
    const size_t o_vh = p.take((size_t)c.n_head * n_pad * (c.dim / c.n_head) * 2);
    const size_t o_a = p.take((size_t)groups * x16_group_bytes(std::max(pcols, c.dim)));
    const size_t o_o = p.take((size_t)groups * x16_group_bytes(c.dim));
    const size_t o_g = p.take((size_t)groups * x16_group_bytes(std::max(c.n_ff, 4 * c.dim)));
    const size_t o_rgb = p.take(rgb_bytes);
    if (w && base) {
        w->x = (float*)(base + o_x);
        w->h = (float*)(base + o_h);
        w->qkv = (float*)(base + o_qkv);
        w->rope = (float*)(base + o_rope);
        w->out = (float*)(base + o_out);
        w->kh = (__half*)(base + o_kh);
        w->vh = (__half*)(base + o_vh);
        w->x16a = base + o_a;
        w->x16o = base + o_o;
        w->x16g = base + o_g;
        w->rgb = base + o_rgb;
        w->n_pad = n_pad;
    }
    return p.off;
}

// vision.rs:159-175: [half][pos][k] (cos, sin), the angle multiplied up step by step in f32
std::vector<float> rope2d_table(float theta, int d_head, int max_pos) {
    const int n_dims = d_head / 2;
    const float theta_scale = powf(theta, -2.0f / (float)n_dims);
    std::vector<float> out;
    out.reserve((size_t)2 * max_pos * (n_dims / 2) * 2);
    for (int half = 0; half < 2; half++) {
        const float freq_scale = half == 0 ? 1.0f : powf(theta, -2.0f / (float)d_head);
        for (int pos = 0; pos < max_pos; pos++) {
            float t = (float)pos;
            for (int k = 0; k < n_dims / 2; k++) {
                const float a = freq_scale * t;
                out.push_back(cosf(a));
                out.push_back(sinf(a));
                t *= theta_scale;
            }
        }
    }
    return out;
}

bool is_device_ptr(const void* p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// the encode of an image placed in its (baked) canvas: layers < 0 → embeddings, else the residual after `layers`
ocr_status encode(ocr_vision* v, const uint8_t* rgb, const Placement& pl, int layers, float* out, size_t cap,
                  int* n_rows, int* row_width) {
    const ocr_vision_cfg& c = v->cfg;
    ocr_ctx* ctx = v->ctx;
    const int grid = c.patch * c.merge;
    if (pl.width <= 0 || pl.height <= 0 || pl.width % grid || pl.height % grid ||
        std::max(pl.width, pl.height) > c.image_size)
        return fail(OCR_ERR_ARG, "image " + std::to_string(pl.width) + "x" + std::to_string(pl.height) +
                                     " is not baked (both sides on the " + std::to_string(grid) +
                                     " px grid, longest <= " + std::to_string(c.image_size) + ")");
    if (layers > c.n_layer)
        return fail(OCR_ERR_ARG, std::to_string(layers) + " layers asked, the encoder has " + std::to_string(c.n_layer));
    if (!rgb || !out) return fail(OCR_ERR_ARG, "null image or output");
    const int px = pl.width / c.patch, py = pl.height / c.patch, n = px * py, max_pos = std::max(px, py);
    const int n_out = n / (c.merge * c.merge), d_head = c.dim / c.n_head;
    const int rows = layers >= 0 ? n : n_out, width = layers >= 0 ? c.dim : c.proj_dim;
    if ((size_t)rows * width > cap)
        return fail(OCR_ERR_ARG, "output holds " + std::to_string(cap) + " floats, the encode writes " +
                                     std::to_string((size_t)rows * width));
    OCR_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    const size_t rgb_bytes = (size_t)pl.img_w * pl.img_h * 3;
    const bool rgb_dev = is_device_ptr(rgb);
    const size_t need = work_layout(c, v->pcols, n, max_pos, rgb_dev ? 16 : rgb_bytes, nullptr, nullptr);
    if (v->work_bytes < need) {
        OCR_CUDA(cudaStreamSynchronize(st));
        if (v->work) dfree(v->work, v->work_bytes, &ctx->mem_work);
        v->work = nullptr;
        v->work_bytes = 0;
        OCR_CUDA(dalloc(&v->work, need, &ctx->mem_work));
        v->work_bytes = need;
    }
    Work w{};
    work_layout(c, v->pcols, n, max_pos, rgb_dev ? 16 : rgb_bytes, &w, (uint8_t*)v->work);
    const std::vector<float> cs = rope2d_table(c.rope_theta, d_head, max_pos);
    OCR_CUDA(cudaMemcpyAsync(w.rope, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, st));
    const uint8_t* d_rgb = rgb;
    if (!rgb_dev) {
        OCR_CUDA(cudaMemcpyAsync(w.rgb, rgb, rgb_bytes, cudaMemcpyHostToDevice, st));
        d_rgb = w.rgb;
    }
    auto gemm = [&](const QMat& m, const BgMaps& bq, const uint8_t* x16, int mode, float* y, int y_stride,
                    uint8_t* y16, int nb) {
        BgArgs g;
        g.w = m;
        g.x16 = x16;
        g.mode = mode;
        g.y = y;
        g.y_stride = y_stride;
        g.y16 = y16;
        g.nb = nb;
        g.wide = 1;
        g.err = ctx->d_err;
        launch_bgemm(st, g, bq, ctx->num_sms, false);
    };
    auto norm_prep = [&](const float* x, const float* nw, uint8_t* x16) {
        PrepArgs p;
        p.x = x;
        p.x_stride = c.dim;
        p.nw = nw;
        p.eps = c.eps;
        p.K = c.dim;
        p.nb = n;
        p.x16 = x16;
        p.err = ctx->d_err;
        launch_xprep(st, p, false);
    };
    // patches → patch embedding → pre_ln
    launch_patchify(st, d_rgb, pl, c.patch, v->lut, v->pcols, w.x16a);
    gemm(v->patch, v->bq_patch, w.x16a, MV_STORE, w.h, c.dim, nullptr, n);
    launch_rmsnorm_rows(st, w.h, v->pre_ln, w.x, n, c.dim, c.eps);
    const int n_layers = layers >= 0 ? layers : c.n_layer;
    TcAttnArgs at;
    at.q = w.qkv;
    at.q_stride = 3 * c.dim;
    at.L = n;
    at.n_head = c.n_head;
    at.group = 1;
    at.k = w.kh;
    at.v = w.vh;
    at.kv_head_stride = (size_t)w.n_pad * d_head;
    at.n_keys = n;
    at.scale = 1.0f / sqrtf((float)d_head);
    at.out16 = w.x16o;
    at.out16_K = c.dim;
    at.err = ctx->d_err;
    for (int l = 0; l < n_layers; l++) {
        const VLayer& L = v->layers[l];
        norm_prep(w.x, L.ln1, w.x16a);
        gemm(L.qkv, L.bq_qkv, w.x16a, MV_STORE, w.qkv, 3 * c.dim, nullptr, n);
        launch_rope2d_heads(st, w.qkv, n, c.n_head, d_head, px, w.rope, max_pos, w.kh, w.vh, w.n_pad);
        launch_attention_full_tc(st, at);
        gemm(L.o, L.bq_o, w.x16o, MV_ADD, w.x, c.dim, nullptr, n);
        norm_prep(w.x, L.ln2, w.x16a);
        gemm(L.gu, L.bq_gu, w.x16a, MV_SWIGLU, nullptr, 0, w.x16g, n);
        gemm(L.down, L.bq_down, w.x16g, MV_ADD, w.x, c.dim, nullptr, n);
    }
    const float* result = w.x;
    if (layers < 0) {
        // the projector: input_norm + 2x2 unfold → merger → mm.1 → GELU → mm.2
        launch_unfold_prep(st, w.x, v->input_norm, c.eps, px, py, c.dim, w.x16g);
        gemm(v->merger, v->bq_merger, w.x16g, MV_STORE, w.h, c.dim, nullptr, n_out);
        launch_act_prep(st, w.h, n_out, c.dim, 0, w.x16a);
        gemm(v->mm1, v->bq_mm1, w.x16a, MV_STORE, w.qkv, c.proj_dim, nullptr, n_out);
        launch_act_prep(st, w.qkv, n_out, c.proj_dim, 1, w.x16a);
        gemm(v->mm2, v->bq_mm2, w.x16a, MV_STORE, w.out, c.proj_dim, nullptr, n_out);
        result = w.out;
    }
    OCR_CUDA(cudaGetLastError());
    OCR_CUDA(cudaMemcpyAsync(out, result, (size_t)rows * width * 4, cudaMemcpyDefault, st));
    OCR_CUDA(cudaStreamSynchronize(st));
    OCR_TRY(check_device_error(ctx));
    if (n_rows) *n_rows = rows;
    if (row_width) *row_width = width;
    return OCR_OK;
}

// the Lanczos-3 taps of a resize from n_in to n_out samples (imageops::resize, FilterType::Lanczos3, of the `image`
// crate 0.25): for output o, ratio = in / out, sratio = max(ratio, 1), the centre (o + 0.5) ratio, taps [floor(centre
// - 3 sratio), ceil(centre + 3 sratio)) clamped to the input, weights lanczos3((i - (centre - 0.5)) / sratio) divided
// by their sum — all in f32 as the crate computes them. One row of max_n weights per output.
struct Taps {
    std::vector<int32_t> left, n;
    std::vector<float> w;
    int max_n = 0;
};
float sinc_f(float t) {
    const float a = t * 3.14159265358979323846f;
    return t == 0.0f ? 1.0f : sinf(a) / a;
}
float lanczos3(float x) { return fabsf(x) < 3.0f ? sinc_f(x) * sinc_f(x / 3.0f) : 0.0f; }
Taps taps_for(int n_in, int n_out) {
    Taps t;
    const float ratio = (float)n_in / (float)n_out;
    const float sratio = ratio < 1.0f ? 1.0f : ratio;
    const float support = 3.0f * sratio;
    std::vector<std::vector<float>> rows(n_out);
    for (int o = 0; o < n_out; o++) {
        float centre = ((float)o + 0.5f) * ratio;
        long l = (long)floorf(centre - support), r = (long)ceilf(centre + support);
        l = std::min(std::max(l, 0L), (long)n_in - 1);
        r = std::min(std::max(r, l + 1), (long)n_in);
        centre -= 0.5f;
        std::vector<float>& w = rows[o];
        float sum = 0.0f;
        for (long i = l; i < r; i++) {
            w.push_back(lanczos3(((float)i - centre) / sratio));
            sum += w.back();
        }
        for (float& x : w) x /= sum;
        t.left.push_back((int32_t)l);
        t.n.push_back((int32_t)w.size());
        t.max_n = std::max(t.max_n, (int)w.size());
    }
    t.w.assign((size_t)n_out * t.max_n, 0.0f);
    for (int o = 0; o < n_out; o++) std::copy(rows[o].begin(), rows[o].end(), t.w.begin() + (size_t)o * t.max_n);
    return t;
}

// The bake on the device (imageops.rs:318-323): rgb (host or device) [h0][w0][3] → the scaled image in `scaled`
// (device, [p.scaled_h][p.scaled_w][3]; the input itself, copied, when the plan does not scale). Temporaries are
// allocated for the call and freed before it returns (synchronous).
ocr_status bake_scaled(ocr_ctx* ctx, const uint8_t* rgb, int w0, int h0, const ocr_bake_plan& p, uint8_t* scaled,
                       bool rgb_dev) {
    cudaStream_t st = ctx->stream;
    const size_t in_bytes = (size_t)w0 * h0 * 3;
    if (p.scaled_w == w0 && p.scaled_h == h0)
        return cudaMemcpyAsync(scaled, rgb, in_bytes, cudaMemcpyDefault, st) == cudaSuccess
                   ? OCR_OK
                   : cuda_fail(cudaGetLastError(), "bake: copy");
    const int w = p.scaled_w, h = p.scaled_h;
    const Taps tv = taps_for(h0, h), th = taps_for(w0, w);
    Plan pl;
    const size_t o_in = pl.take(rgb_dev ? 16 : in_bytes), o_tmp = pl.take((size_t)h * w0 * 3 * 4);
    const size_t o_vl = pl.take((size_t)h * 4), o_vn = pl.take((size_t)h * 4), o_vw = pl.take(tv.w.size() * 4);
    const size_t o_hl = pl.take((size_t)w * 4), o_hn = pl.take((size_t)w * 4), o_hw = pl.take(th.w.size() * 4);
    void* buf = nullptr;
    OCR_CUDA(dalloc(&buf, pl.off, &ctx->mem_work));
    uint8_t* b = (uint8_t*)buf;
    cudaError_t e = cudaSuccess;
    const uint8_t* d_rgb = rgb;
    if (!rgb_dev) {
        e = cudaMemcpyAsync(b + o_in, rgb, in_bytes, cudaMemcpyHostToDevice, st);
        d_rgb = b + o_in;
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(b + o_vl, tv.left.data(), (size_t)h * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(b + o_vn, tv.n.data(), (size_t)h * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(b + o_vw, tv.w.data(), tv.w.size() * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(b + o_hl, th.left.data(), (size_t)w * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(b + o_hn, th.n.data(), (size_t)w * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(b + o_hw, th.w.data(), th.w.size() * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) {
        launch_resize(st, d_rgb, w0, h0, w, h, (const int*)(b + o_vl), (const int*)(b + o_vn),
                      (const float*)(b + o_vw), tv.max_n, (const int*)(b + o_hl), (const int*)(b + o_hn),
                      (const float*)(b + o_hw), th.max_n, (float*)(b + o_tmp), scaled);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    dfree(buf, pl.off, &ctx->mem_work);
    if (e != cudaSuccess) return cuda_fail(e, "bake: resize");
    return OCR_OK;
}

void plan_for(int longest, int grid, int w0, int h0, ocr_bake_plan* p) {
    double w = w0, h = h0;
    const double l = std::max(w, h);
    if (l > longest) {
        const double s = (double)longest / l;
        w = std::max(1.0, std::round(w * s));
        h = std::max(1.0, std::round(h * s));
    }
    p->scaled_w = (int)w;
    p->scaled_h = (int)h;
    p->left = p->top = p->right = p->bottom = 0;
    auto pad = [&](double nw, double nh) {
        const int pw = (int)(nw - w), ph = (int)(nh - h);
        p->left += pw / 2;
        p->right += pw - pw / 2;
        p->top += ph / 2;
        p->bottom += ph - ph / 2;
        w = nw;
        h = nh;
    };
    const double min_short = 56.0;
    if (std::min(w, h) < min_short) {
        if (w <= h) pad(min_short, h);
        else pad(w, min_short);
    }
    const double sw = std::ceil(w / grid) * grid, sh = std::ceil(h / grid) * grid;
    if (sw != w || sh != h) pad(sw, sh);
}

}  // namespace

extern "C" {

ocr_status ocr_bake_plan_for(int longest, int grid, int w0, int h0, ocr_bake_plan* out) {
    if (!out) return fail(OCR_ERR_ARG, "null argument");
    if (longest <= 0 || grid <= 0 || w0 <= 0 || h0 <= 0) return fail(OCR_ERR_ARG, "sizes must be positive");
    plan_for(longest, grid, w0, h0, out);
    return OCR_OK;
}

ocr_status ocr_vision_synthetic(ocr_ctx* ctx, const ocr_vision_cfg* cfg, uint64_t seed, float sigma_w,
                                ocr_vision** out) {
    if (!ctx || !cfg || !out) return fail(OCR_ERR_ARG, "null argument");
    OCR_TRY(check_vcfg(*cfg));
    const ocr_vision_cfg& c = *cfg;
    OCR_CUDA(cudaSetDevice(ctx->device));
    auto* v = new ocr_vision();
    v->ctx = ctx;
    v->cfg = c;
    v->pcols = patch_cols(c);
    const int d = c.dim, f = c.n_ff;
    // the layout: per layer qkv, o, gu, down (row layout + tile-major copy), ln1, ln2; then the patch embedding,
    // merger, mm.1, mm.2 likewise, pre_ln, input_norm, the LUT
    Plan p;
    struct M {
        size_t w, t;
        int rows, cols;
    };
    auto mat = [&](int rows, int cols) {
        M m;
        m.rows = rows;
        m.cols = cols;
        m.w = p.take((size_t)rows * q8_stride(cols));
        m.t = p.take(bgemm_tiled_bytes(rows, cols));
        return m;
    };
    struct LO {
        M qkv, o, gu, down;
        size_t ln1, ln2;
    };
    std::vector<LO> lo(c.n_layer);
    for (auto& L : lo) {
        L.qkv = mat(3 * d, d);
        L.o = mat(d, d);
        L.gu = mat(2 * f, d);
        L.down = mat(d, f);
        L.ln1 = p.take((size_t)d * 4);
        L.ln2 = p.take((size_t)d * 4);
    }
    const M mp = mat(d, v->pcols), mg = mat(d, 4 * d), m1 = mat(c.proj_dim, d), m2 = mat(c.proj_dim, c.proj_dim);
    const size_t o_pre = p.take((size_t)d * 4), o_in = p.take((size_t)d * 4), o_lut = p.take(768 * 4);
    cudaError_t e = dalloc(&v->mem, p.off, &ctx->mem_weights);
    if (e != cudaSuccess) {
        delete v;
        return cuda_fail(e, "ocr_vision_synthetic: the weights");
    }
    v->mem_bytes = p.off;
    ctx->refs++;
    uint8_t* base = (uint8_t*)v->mem;
    auto qm = [&](const M& m, QMat& q, BgMaps& b) {
        q.w = base + m.w;
        q.rows = m.rows;
        q.cols = m.cols;
        q.stride = q8_stride(m.cols);
        b.tiles = base + m.t;
    };
    cudaStream_t st = ctx->stream;
    v->layers.resize(c.n_layer);
    for (int l = 0; l < c.n_layer; l++) {
        VLayer& L = v->layers[l];
        qm(lo[l].qkv, L.qkv, L.bq_qkv);
        qm(lo[l].o, L.o, L.bq_o);
        qm(lo[l].gu, L.gu, L.bq_gu);
        qm(lo[l].down, L.down, L.bq_down);
        L.ln1 = (float*)(base + lo[l].ln1);
        L.ln2 = (float*)(base + lo[l].ln2);
        auto sub = [&](int kind) { return substream(seed, V_LAYER_STREAM + (uint64_t)l * 16 + kind); };
        launch_synth_norm(st, sub(VK_LN1), d, L.ln1);
        launch_synth_norm(st, sub(VK_LN2), d, L.ln2);
        uint8_t* wq = const_cast<uint8_t*>(L.qkv.w);
        launch_synth_q8_0(st, sub(VK_Q), sigma_w, d, d, wq, 1, 0);
        launch_synth_q8_0(st, sub(VK_K), sigma_w, d, d, wq, 1, d);
        launch_synth_q8_0(st, sub(VK_V), sigma_w, d, d, wq, 1, 2 * d);
        launch_synth_q8_0(st, sub(VK_O), sigma_w, d, d, const_cast<uint8_t*>(L.o.w), 1, 0);
        launch_synth_q8_0(st, sub(VK_GATE), sigma_w, f, d, const_cast<uint8_t*>(L.gu.w), 2, 0);
        launch_synth_q8_0(st, sub(VK_UP), sigma_w, f, d, const_cast<uint8_t*>(L.gu.w), 2, 1);
        launch_synth_q8_0(st, sub(VK_DOWN), sigma_w, d, f, const_cast<uint8_t*>(L.down.w), 1, 0);
        launch_tile_q8_0(st, L.qkv, const_cast<uint8_t*>(L.bq_qkv.tiles));
        launch_tile_q8_0(st, L.o, const_cast<uint8_t*>(L.bq_o.tiles));
        launch_tile_q8_0(st, L.gu, const_cast<uint8_t*>(L.bq_gu.tiles));
        launch_tile_q8_0(st, L.down, const_cast<uint8_t*>(L.bq_down.tiles));
    }
    qm(mp, v->patch, v->bq_patch);
    qm(mg, v->merger, v->bq_merger);
    qm(m1, v->mm1, v->bq_mm1);
    qm(m2, v->mm2, v->bq_mm2);
    v->pre_ln = (float*)(base + o_pre);
    v->input_norm = (float*)(base + o_in);
    v->lut = (float*)(base + o_lut);
    launch_synth_q8_0(st, substream(seed, V_PATCH_STREAM), sigma_w, d, v->pcols, const_cast<uint8_t*>(v->patch.w), 1,
                      0, 3 * c.patch * c.patch);
    launch_synth_q8_0(st, substream(seed, V_MERGER_STREAM), sigma_w, d, 4 * d, const_cast<uint8_t*>(v->merger.w), 1, 0);
    launch_synth_q8_0(st, substream(seed, V_MM1_STREAM), sigma_w, c.proj_dim, d, const_cast<uint8_t*>(v->mm1.w), 1, 0);
    launch_synth_q8_0(st, substream(seed, V_MM2_STREAM), sigma_w, c.proj_dim, c.proj_dim,
                      const_cast<uint8_t*>(v->mm2.w), 1, 0);
    launch_synth_norm(st, substream(seed, V_PRE_LN_STREAM), d, v->pre_ln);
    launch_synth_norm(st, substream(seed, V_INPUT_NORM_STREAM), d, v->input_norm);
    launch_tile_q8_0(st, v->patch, const_cast<uint8_t*>(v->bq_patch.tiles));
    launch_tile_q8_0(st, v->merger, const_cast<uint8_t*>(v->bq_merger.tiles));
    launch_tile_q8_0(st, v->mm1, const_cast<uint8_t*>(v->bq_mm1.tiles));
    launch_tile_q8_0(st, v->mm2, const_cast<uint8_t*>(v->bq_mm2.tiles));
    // vision.rs:152-155: lut[c·256 + v] = (v / 255 − mean[c]) / std[c] in f32
    std::vector<float> lut(768);
    for (int ch = 0; ch < 3; ch++)
        for (int b = 0; b < 256; b++) lut[ch * 256 + b] = ((float)b / 255.0f - c.mean[ch]) / c.std[ch];
    e = cudaMemcpyAsync(v->lut, lut.data(), 768 * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        ocr_vision_destroy(v);
        return cuda_fail(e, "ocr_vision_synthetic");
    }
    *out = v;
    return OCR_OK;
}

ocr_status ocr_vision_destroy(ocr_vision* v) {
    if (!v) return OCR_OK;
    ocr_ctx* ctx = v->ctx;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (v->work) dfree(v->work, v->work_bytes, &ctx->mem_work);
    if (v->mem) dfree(v->mem, v->mem_bytes, &ctx->mem_weights);
    delete v;
    ctx_release(ctx);
    return OCR_OK;
}

ocr_status ocr_vision_config(const ocr_vision* v, ocr_vision_cfg* out) {
    if (!v || !out) return fail(OCR_ERR_ARG, "null argument");
    *out = v->cfg;
    return OCR_OK;
}

ocr_status ocr_vision_encode(ocr_vision* v, const uint8_t* rgb, int w, int h, int layers, float* out, size_t cap,
                             int* n_rows, int* row_width) {
    if (!v) return fail(OCR_ERR_ARG, "null encoder");
    Placement pl;
    pl.img_w = pl.width = w;
    pl.img_h = pl.height = h;
    return encode(v, rgb, pl, layers, out, cap, n_rows, row_width);
}

ocr_status ocr_vision_encode_page(ocr_vision* v, const uint8_t* rgb, int w0, int h0, float* out, size_t cap,
                                  int* n_rows) {
    if (!v || !rgb) return fail(OCR_ERR_ARG, "null encoder or image");
    if (w0 <= 0 || h0 <= 0) return fail(OCR_ERR_ARG, "image sizes must be positive");
    ocr_bake_plan p;
    plan_for(v->cfg.image_size, v->cfg.patch * v->cfg.merge, w0, h0, &p);
    Placement pl;
    pl.img_w = p.scaled_w;
    pl.img_h = p.scaled_h;
    pl.left = p.left;
    pl.top = p.top;
    pl.width = p.scaled_w + p.left + p.right;
    pl.height = p.scaled_h + p.top + p.bottom;
    if (p.scaled_w == w0 && p.scaled_h == h0) return encode(v, rgb, pl, -1, out, cap, n_rows, nullptr);
    // the Lanczos-3 resize first (a device copy of the scaled page, for the call), then the pad inside the gather
    ocr_ctx* ctx = v->ctx;
    OCR_CUDA(cudaSetDevice(ctx->device));
    const size_t sbytes = (size_t)p.scaled_w * p.scaled_h * 3;
    void* scaled = nullptr;
    OCR_CUDA(dalloc(&scaled, sbytes, &ctx->mem_work));
    ocr_status r = bake_scaled(ctx, rgb, w0, h0, p, (uint8_t*)scaled, is_device_ptr(rgb));
    if (r == OCR_OK) r = encode(v, (const uint8_t*)scaled, pl, -1, out, cap, n_rows, nullptr);
    dfree(scaled, sbytes, &ctx->mem_work);
    return r;
}

ocr_status ocr_image_bake(ocr_ctx* ctx, const uint8_t* rgb, int w0, int h0, int longest, int grid, uint8_t* out,
                          size_t cap, int* out_w, int* out_h) {
    if (!ctx || !rgb || !out) return fail(OCR_ERR_ARG, "null argument");
    if (w0 <= 0 || h0 <= 0 || longest <= 0 || grid <= 0) return fail(OCR_ERR_ARG, "sizes must be positive");
    ocr_bake_plan p;
    plan_for(longest, grid, w0, h0, &p);
    const int fw = p.scaled_w + p.left + p.right, fh = p.scaled_h + p.top + p.bottom;
    if ((size_t)fw * fh * 3 > cap)
        return fail(OCR_ERR_ARG, "output holds " + std::to_string(cap) + " bytes, the baked image " +
                                     std::to_string((size_t)fw * fh * 3));
    OCR_CUDA(cudaSetDevice(ctx->device));
    const size_t sbytes = (size_t)p.scaled_w * p.scaled_h * 3, fbytes = (size_t)fw * fh * 3;
    void* buf = nullptr;
    OCR_CUDA(dalloc(&buf, sbytes + fbytes, &ctx->mem_work));
    uint8_t* scaled = (uint8_t*)buf;
    uint8_t* canvas = scaled + sbytes;
    ocr_status r = bake_scaled(ctx, rgb, w0, h0, p, scaled, is_device_ptr(rgb));
    if (r == OCR_OK) {
        launch_bake_place(ctx->stream, scaled, p.scaled_w, p.scaled_h, p.left, p.top, fw, fh, canvas);
        cudaError_t e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaMemcpyAsync(out, canvas, fbytes, cudaMemcpyDefault, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) r = cuda_fail(e, "ocr_image_bake");
    }
    dfree(buf, sbytes + fbytes, &ctx->mem_work);
    if (r == OCR_OK) {
        if (out_w) *out_w = fw;
        if (out_h) *out_h = fh;
    }
    return r;
}

ocr_status ocr_op_attention_full(ocr_ctx* ctx, const float* d_q, int q_stride, int L, int n_head,
                                 const uint16_t* d_k_tiled, const uint16_t* d_vt_tiled, int n_pad, int n_keys,
                                 float scale, float* d_out, int out_stride) {
    if (!ctx || !d_q || !d_k_tiled || !d_vt_tiled || !d_out) return fail(OCR_ERR_ARG, "null argument");
    if (L <= 0 || n_head <= 0 || n_keys <= 0 || n_pad % 64 || n_keys > n_pad || q_stride < n_head * 64 ||
        out_stride < n_head * 64)
        return fail(OCR_ERR_ARG, "attention shape out of range");
    OCR_CUDA(cudaSetDevice(ctx->device));
    TcAttnArgs a;
    a.q = d_q;
    a.q_stride = q_stride;
    a.L = L;
    a.n_head = n_head;
    a.group = 1;
    a.k = reinterpret_cast<const __half*>(d_k_tiled);
    a.v = reinterpret_cast<const __half*>(d_vt_tiled);
    a.kv_head_stride = (size_t)n_pad * 64;
    a.n_keys = n_keys;
    a.scale = scale;
    a.out = d_out;
    a.out_stride = out_stride;
    a.err = ctx->d_err;
    launch_attention_full_tc(ctx->stream, a);
    OCR_CUDA(cudaGetLastError());
    return OCR_OK;
}

}  // extern "C"
