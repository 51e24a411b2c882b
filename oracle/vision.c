/*
 * vision.c — CPU restatement of the reference's vision encoder + projector and of the image bake's plan.
 * TEST INFRASTRUCTURE ONLY: the checker of libocrcuda.so's vision kernels and config 4's timed CPU baseline; never
 * linked into or called by the product.
 *
 * What each function restates (paths relative to b-straub/historic-htr-ocr):
 *   - the encoder graph (Vision::run, the F32 path)   app/crates/ocr-wgpu/src/vision.rs:266-317
 *   - K / V rounded to f16 for the attention          app/crates/ocr-wgpu/src/vision.rs:319-327 (run_f16: "f16: …
 *                                                     K / V for the attention"), heads_f16.wgsl
 *   - the pixel LUT and the patch im2col              vision.rs:152-155 (pixel_lut), shaders/patchify.wgsl:22-38
 *   - the 2D RoPE table and its application           vision.rs:159-175 (rope_table), shaders/rope2d.wgsl:25-45
 *   - full attention, scale 1/sqrt(d_head)            vision.rs:290-295, shaders/attention.wgsl
 *   - SwiGLU (silu(gate) * up)                        shaders/swiglu.wgsl:19-26
 *   - the projector: input_norm → 2×2 unfold → merger → mm.1 → GELU (tanh form, argument clamped ±15) → mm.2
 *                                                     vision.rs:405-423, shaders/unfold2x2.wgsl, shaders/gelu.wgsl
 *   - the bake's plan (longest edge, pads)            app/crates/ocr-core/src/imageops.rs:275-323 (plan)
 *   - the bake's resize: imageops::resize(img, w, h, FilterType::Lanczos3) (imageops.rs:320) of the `image` crate,
 *     pinned at 0.25.10 in app/Cargo.lock and not vendored: restated from that crate's published separable sampler —
 *     a vertical pass to f32, then a horizontal pass to u8 (clamped to [0, 255], rounded half away from zero); per
 *     output index o: ratio = in / out, sratio = max(ratio, 1), centre = (o + 0.5) ratio, taps [floor(centre - 3
 *     sratio), ceil(centre + 3 sratio)) clamped to the image, weight lanczos3((i - (centre - 0.5)) / sratio)
 *     normalised by their f32 sum, lanczos3(x) = sinc(x) sinc(x / 3) for |x| < 3, sinc(t) = sin(pi t) / (pi t)
 * Weights are q8_0 (config 4 asks q8_0; the reference loads bf16 / f32 vision weights): each matrix is a q8_0
 * matrix of the same shape, the patch embedding's 3·14·14 = 588 columns padded with zero columns to 768 (q8_0 needs
 * whole 32-blocks; the device contraction whole 256-column pieces). Accumulations are f64 (the order-free limit of
 * the reference's f32 sums); the f16 roundings of K and V are reproduced bit for bit.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

struct orc_vision {
    orc_vcfg cfg;
    int pcols;        /* the padded patch-embedding width */
    uint8_t** t;      /* [n_layer][ORC_V_N_KINDS] q8_0 blocks or f32 norms */
    uint8_t* patch;   /* [dim][pcols] q8_0 */
    float* pre_ln;
    float* input_norm;
    uint8_t* merger;  /* [dim][dim * merge²] */
    uint8_t* mm1;     /* [proj_dim][dim] */
    uint8_t* mm2;     /* [proj_dim][proj_dim] */
};

int orc_vision_patch_cols(const orc_vcfg* c) {
    int pp = 3 * c->patch * c->patch;
    return (pp + 255) / 256 * 256;
}

static void vkind_shape(const orc_vcfg* c, int kind, size_t* rows, size_t* cols) {
    size_t d = c->dim, f = c->n_ff;
    switch (kind) {
    case ORC_V_Q: case ORC_V_K: case ORC_V_V: case ORC_V_O: *rows = d; *cols = d; break;
    case ORC_V_GATE: case ORC_V_UP: *rows = f; *cols = d; break;
    case ORC_V_DOWN: *rows = d; *cols = f; break;
    default: *rows = 1; *cols = d; break; /* ln1, ln2 */
    }
}

/* rows x cols q8_0 blocks whose column c < valid holds sigma * gauss(seed, r * valid + c) and whose other columns are
 * zero (valid == cols: orc_synth_q8_0's values) */
void orc_synth_q8_0_padded(uint8_t* blocks, int rows, int cols, int valid, uint64_t seed, float sigma) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        float* x = (float*)malloc(sizeof(float) * (size_t)cols);
        for (int c = 0; c < cols; c++) x[c] = c < valid ? sigma * orc_gauss(seed, (uint64_t)r * valid + c) : 0.0f;
        orc_quantize_q8_0(x, (size_t)cols, blocks + (size_t)r * (cols / 32) * 34, NULL);
        free(x);
    }
}

orc_vision* orc_vision_synthetic(const orc_vcfg* cfg, uint64_t seed, float sigma_w) {
    orc_vision* v = (orc_vision*)calloc(1, sizeof(orc_vision));
    v->cfg = *cfg;
    const int d = cfg->dim, mm = cfg->merge * cfg->merge, pp = 3 * cfg->patch * cfg->patch;
    v->pcols = orc_vision_patch_cols(cfg);
    v->t = (uint8_t**)calloc((size_t)cfg->n_layer * ORC_V_N_KINDS, sizeof(uint8_t*));
    for (int l = 0; l < cfg->n_layer; l++)
        for (int k = 0; k < ORC_V_N_KINDS; k++) {
            size_t r, c;
            vkind_shape(cfg, k, &r, &c);
            uint64_t s = orc_substream(seed, ORC_V_LAYER_STREAM + (uint64_t)l * 16 + k);
            if (k == ORC_V_LN1 || k == ORC_V_LN2) {
                v->t[l * ORC_V_N_KINDS + k] = (uint8_t*)malloc(sizeof(float) * c);
                orc_fill_norm((float*)v->t[l * ORC_V_N_KINDS + k], c, s);
            } else {
                v->t[l * ORC_V_N_KINDS + k] = (uint8_t*)malloc(r * c / 32 * 34);
                orc_synth_q8_0(v->t[l * ORC_V_N_KINDS + k], r * c, s, sigma_w);
            }
        }
    v->patch = (uint8_t*)malloc((size_t)d * v->pcols / 32 * 34);
    orc_synth_q8_0_padded(v->patch, d, v->pcols, pp, orc_substream(seed, ORC_V_PATCH_STREAM), sigma_w);
    v->pre_ln = (float*)malloc(sizeof(float) * d);
    orc_fill_norm(v->pre_ln, d, orc_substream(seed, ORC_V_PRE_LN_STREAM));
    v->input_norm = (float*)malloc(sizeof(float) * d);
    orc_fill_norm(v->input_norm, d, orc_substream(seed, ORC_V_INPUT_NORM_STREAM));
    v->merger = (uint8_t*)malloc((size_t)d * d * mm / 32 * 34);
    orc_synth_q8_0(v->merger, (size_t)d * d * mm, orc_substream(seed, ORC_V_MERGER_STREAM), sigma_w);
    v->mm1 = (uint8_t*)malloc((size_t)cfg->proj_dim * d / 32 * 34);
    orc_synth_q8_0(v->mm1, (size_t)cfg->proj_dim * d, orc_substream(seed, ORC_V_MM1_STREAM), sigma_w);
    v->mm2 = (uint8_t*)malloc((size_t)cfg->proj_dim * cfg->proj_dim / 32 * 34);
    orc_synth_q8_0(v->mm2, (size_t)cfg->proj_dim * cfg->proj_dim, orc_substream(seed, ORC_V_MM2_STREAM), sigma_w);
    return v;
}

void orc_vision_free(orc_vision* v) {
    if (!v) return;
    for (int i = 0; i < v->cfg.n_layer * ORC_V_N_KINDS; i++) free(v->t[i]);
    free(v->t);
    free(v->patch);
    free(v->pre_ln);
    free(v->input_norm);
    free(v->merger);
    free(v->mm1);
    free(v->mm2);
    free(v);
}

/* ---- pieces ------------------------------------------------------------------------------------------------------ */

/* vision.rs:152-155: lut[c·256 + v] = (v / 255 − mean[c]) / std[c], f32 */
void orc_pixel_lut(const orc_vcfg* c, float* lut) {
    for (int ch = 0; ch < 3; ch++)
        for (int v = 0; v < 256; v++) lut[ch * 256 + v] = ((float)v / 255.0f - c->mean[ch]) / c->std[ch];
}

/* vision.rs:159-175 (ggml_rope_cache_init): [half][pos][k] → (cos, sin), k < d_head / 4; θ multiplied up in f32 */
void orc_rope2d_table(float theta, int d_head, int max_pos, float* out) {
    const int n_dims = d_head / 2;
    const float theta_scale = powf(theta, -2.0f / (float)n_dims);
    size_t o = 0;
    for (int half = 0; half < 2; half++) {
        const float freq_scale = half == 0 ? 1.0f : powf(theta, -2.0f / (float)d_head);
        for (int pos = 0; pos < max_pos; pos++) {
            float t = (float)pos;
            for (int k = 0; k < n_dims / 2; k++) {
                const float a = freq_scale * t;
                out[o++] = cosf(a);
                out[o++] = sinf(a);
                t *= theta_scale;
            }
        }
    }
}

/* patchify.wgsl:27-37: P[t][c·p·p + ky·p + kx] = lut[c·256 + rgb[((ty·p + ky)·w + tx·p + kx)·3 + c]], t = ty·px + tx;
 * columns past 3·p·p are zero (the padded conv input) */
static void patchify(const orc_vcfg* c, const float* lut, const uint8_t* rgb, int w, int px, int n, int pcols, float* P) {
    const int p = c->patch, pp = p * p;
#pragma omp parallel for schedule(static)
    for (int t = 0; t < n; t++)
        for (int col = 0; col < pcols; col++) {
            float v = 0.0f;
            if (col < 3 * pp) {
                const int ch = col / pp, ky = (col % pp) / p, kx = col % p;
                const int x = (t % px) * p + kx, y = (t / px) * p + ky;
                v = lut[ch * 256 + rgb[((size_t)y * w + x) * 3 + ch]];
            }
            P[(size_t)t * pcols + col] = v;
        }
}

/* y[r][:] (+)= W · x[r][:] for the rows listed (NULL: rows 0 … n-1) */
static void matmul(const uint8_t* W, int out_rows, int k, const float* x, int n, const int* list, float* y, int acc) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; i++) {
        const int r = list ? list[i] : i;
        orc_matvec_q8_0_serial(W, out_rows, k, x + (size_t)r * k, y + (size_t)r * out_rows, acc);
    }
}

/* rms_norm.wgsl: y = x / sqrt(mean(x²) + eps) · w, row by row */
static void rms_rows(const float* x, const float* w, float* y, int n, const int* list, int d, float eps) {
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; i++) {
        const int r = list ? list[i] : i;
        const float s = orc_rms_scale(x + (size_t)r * d, d, eps);
        for (int j = 0; j < d; j++) y[(size_t)r * d + j] = x[(size_t)r * d + j] * s * w[j];
    }
}

/* rope2d.wgsl:31-44 on one row of n_head heads: dims [0, d/2) by the patch row, [d/2, d) by the patch column, adjacent
 * pairs (2k, 2k + 1) rotated */
static void rope2d_row(float* row, int t, int px, int n_head, int d_head, const float* cs, int max_pos) {
    const int nk = d_head / 4;
    for (int h = 0; h < n_head; h++)
        for (int half = 0; half < 2; half++) {
            const int pos = half == 0 ? t / px : t % px;
            for (int k = 0; k < nk; k++) {
                const float* c = cs + ((size_t)(half * max_pos + pos) * nk + k) * 2;
                float* o = row + h * d_head + half * (d_head / 2) + 2 * k;
                const float x0 = o[0], x1 = o[1];
                o[0] = x0 * c[0] - x1 * c[1];
                o[1] = x0 * c[1] + x1 * c[0];
            }
        }
}

/* silu(g) · u (swiglu.wgsl:23-24) */
static inline float swiglu(float g, float u) { return g / (1.0f + expf(-g)) * u; }

/* gelu.wgsl:22-26 */
float orc_gelu_tanh(float x) {
    float t = 0.7978845608028654f * x * (1.0f + 0.044715f * x * x);
    if (t < -15.0f) t = -15.0f;
    if (t > 15.0f) t = 15.0f;
    return 0.5f * x * (1.0f + tanhf(t));
}

/* one encoder layer on the rows `list` (NULL: all n) of the residual x [n][d]; the keys and values of all n rows are
 * computed (every query attends to every patch) */
static void layer(const orc_vision* v, int l, float* x, int n, const int* list, int n_list, int px, const float* cs,
                  int max_pos) {
    const orc_vcfg* c = &v->cfg;
    const int d = c->dim, f = c->n_ff, H = c->n_head, dh = d / H;
    const uint8_t* const* T = (const uint8_t* const*)v->t + (size_t)l * ORC_V_N_KINDS;
    const int nq = list ? n_list : n;
    float* hn = (float*)malloc(sizeof(float) * (size_t)n * d);
    float* q = (float*)malloc(sizeof(float) * (size_t)n * d);
    float* kf = (float*)malloc(sizeof(float) * (size_t)n * d);
    float* vf = (float*)malloc(sizeof(float) * (size_t)n * d);
    uint16_t* k16 = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)n * d);
    uint16_t* v16 = (uint16_t*)malloc(sizeof(uint16_t) * (size_t)n * d);
    float* a = (float*)malloc(sizeof(float) * (size_t)n * d);
    rms_rows(x, (const float*)T[ORC_V_LN1], hn, n, NULL, d, c->eps);
    matmul(T[ORC_V_K], d, d, hn, n, NULL, kf, 0);
    matmul(T[ORC_V_V], d, d, hn, n, NULL, vf, 0);
    matmul(T[ORC_V_Q], d, d, hn, nq, list, q, 0);
#pragma omp parallel for schedule(static)
    for (int t = 0; t < n; t++) {
        rope2d_row(kf + (size_t)t * d, t, px, H, dh, cs, max_pos);
        for (int j = 0; j < d; j++) {
            k16[(size_t)t * d + j] = orc_f16_from_f32(kf[(size_t)t * d + j]);
            v16[(size_t)t * d + j] = orc_f16_from_f32(vf[(size_t)t * d + j]);
        }
    }
    const float scale = 1.0f / sqrtf((float)dh);
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
    for (int i = 0; i < nq; i++)
        for (int h = 0; h < H; h++) {
            const int t = list ? list[i] : i;
            float qh[256];
            memcpy(qh, q + (size_t)t * d + h * dh, sizeof(float) * dh);
            /* this head's rotation (rope2d_row's arithmetic on one head) */
            const int nk = dh / 4;
            for (int half = 0; half < 2; half++) {
                const int pos = half == 0 ? t / px : t % px;
                for (int k = 0; k < nk; k++) {
                    const float* cc = cs + ((size_t)(half * max_pos + pos) * nk + k) * 2;
                    float* o = qh + half * (dh / 2) + 2 * k;
                    const float x0 = o[0], x1 = o[1];
                    o[0] = x0 * cc[0] - x1 * cc[1];
                    o[1] = x0 * cc[1] + x1 * cc[0];
                }
            }
            orc_attend(qh, k16 + h * dh, v16 + h * dh, n, d, dh, scale, a + (size_t)t * d + h * dh);
        }
    matmul(T[ORC_V_O], d, d, a, nq, list, x, 1);
    rms_rows(x, (const float*)T[ORC_V_LN2], hn, nq, list, d, c->eps);
    float* g = (float*)malloc(sizeof(float) * (size_t)n * f);
    float* u = (float*)malloc(sizeof(float) * (size_t)n * f);
    matmul(T[ORC_V_GATE], f, d, hn, nq, list, g, 0);
    matmul(T[ORC_V_UP], f, d, hn, nq, list, u, 0);
#pragma omp parallel for schedule(static)
    for (int i = 0; i < nq; i++) {
        const int t = list ? list[i] : i;
        for (int j = 0; j < f; j++) g[(size_t)t * f + j] = swiglu(g[(size_t)t * f + j], u[(size_t)t * f + j]);
    }
    matmul(T[ORC_V_DOWN], d, f, g, nq, list, x, 1);
    free(hn), free(q), free(kf), free(vf), free(k16), free(v16), free(a), free(g), free(u);
}

static int grid_of(const orc_vcfg* c, int w, int h, int* px, int* py) {
    const int grid = c->patch * c->merge;
    if (w <= 0 || h <= 0 || w % grid || h % grid || (w > h ? w : h) > c->image_size) return -1;
    *px = w / c->patch;
    *py = h / c->patch;
    return 0;
}

/* patchify → patch conv → pre_ln: the residual x [n][d] */
static float* embed(const orc_vision* v, const uint8_t* rgb, int w, int n, int px) {
    const orc_vcfg* c = &v->cfg;
    float lut[768];
    orc_pixel_lut(c, lut);
    float* P = (float*)malloc(sizeof(float) * (size_t)n * v->pcols);
    patchify(c, lut, rgb, w, px, n, v->pcols, P);
    float* hb = (float*)malloc(sizeof(float) * (size_t)n * c->dim);
    matmul(v->patch, c->dim, v->pcols, P, n, NULL, hb, 0);
    float* x = (float*)malloc(sizeof(float) * (size_t)n * c->dim);
    rms_rows(hb, v->pre_ln, x, n, NULL, c->dim, c->eps);
    free(P);
    free(hb);
    return x;
}

int orc_vision_encode(const orc_vision* v, const uint8_t* rgb, int w, int h, int layers, float* out) {
    const orc_vcfg* c = &v->cfg;
    int px, py;
    if (grid_of(c, w, h, &px, &py) || layers > c->n_layer) return -1;
    const int n = px * py, d = c->dim, max_pos = px > py ? px : py;
    float* cs = (float*)malloc(sizeof(float) * 2 * (size_t)max_pos * (d / c->n_head / 4) * 2);
    orc_rope2d_table(c->rope_theta, d / c->n_head, max_pos, cs);
    float* x = embed(v, rgb, w, n, px);
    const int nl = layers < 0 ? c->n_layer : layers;
    for (int l = 0; l < nl; l++) layer(v, l, x, n, NULL, 0, px, cs, max_pos);
    free(cs);
    if (layers >= 0) {
        memcpy(out, x, sizeof(float) * (size_t)n * d);
        free(x);
        return n;
    }
    /* the projector (vision.rs:405-423) */
    const int mm = c->merge * c->merge, n_out = n / mm, pd = c->proj_dim;
    float* xn = (float*)malloc(sizeof(float) * (size_t)n * d);
    rms_rows(x, v->input_norm, xn, n, NULL, d, c->eps);
    float* Z = (float*)malloc(sizeof(float) * (size_t)n * d);
    const int oxn = px / 2;
    for (int o = 0; o < n_out; o++)
        for (int ch = 0; ch < d; ch++)
            for (int ky = 0; ky < 2; ky++)
                for (int kx = 0; kx < 2; kx++)
                    Z[(size_t)o * d * 4 + ch * 4 + ky * 2 + kx] =
                        xn[((size_t)(2 * (o / oxn) + ky) * px + 2 * (o % oxn) + kx) * d + ch];
    float* merged = (float*)malloc(sizeof(float) * (size_t)n_out * d);
    matmul(v->merger, d, d * mm, Z, n_out, NULL, merged, 0);
    float* m1 = (float*)malloc(sizeof(float) * (size_t)n_out * pd);
    matmul(v->mm1, pd, d, merged, n_out, NULL, m1, 0);
    for (size_t i = 0; i < (size_t)n_out * pd; i++) m1[i] = orc_gelu_tanh(m1[i]);
    matmul(v->mm2, pd, pd, m1, n_out, NULL, out, 0);
    free(x), free(xn), free(Z), free(merged), free(m1);
    return n_out;
}

int orc_vision_layer1_rows(const orc_vision* v, const uint8_t* rgb, int w, int h, const int* rows, int n_rows,
                           float* out) {
    const orc_vcfg* c = &v->cfg;
    int px, py;
    if (grid_of(c, w, h, &px, &py) || c->n_layer < 1) return -1;
    const int n = px * py, d = c->dim, max_pos = px > py ? px : py;
    for (int i = 0; i < n_rows; i++)
        if (rows[i] < 0 || rows[i] >= n) return -1;
    float* cs = (float*)malloc(sizeof(float) * 2 * (size_t)max_pos * (d / c->n_head / 4) * 2);
    orc_rope2d_table(c->rope_theta, d / c->n_head, max_pos, cs);
    float* x = embed(v, rgb, w, n, px);
    layer(v, 0, x, n, rows, n_rows, px, cs, max_pos);
    for (int i = 0; i < n_rows; i++) memcpy(out + (size_t)i * d, x + (size_t)rows[i] * d, sizeof(float) * d);
    free(cs);
    free(x);
    return n_rows;
}

/* imageops.rs:275-316 (plan): the longest edge scaled down to `longest` (rounded, at least 1), the short edge padded to
 * 56, then both padded up to the grid; each pad split half left / top (the smaller half), the rest right / bottom */
void orc_bake_plan(int longest, int grid, int w0, int h0, int* out) {
    double w = w0, h = h0, l = w > h ? w : h;
    if (l > longest) {
        const double s = (double)longest / l;
        w = round(w * s);
        h = round(h * s);
        if (w < 1.0) w = 1.0;
        if (h < 1.0) h = 1.0;
    }
    const int sw0 = (int)w, sh0 = (int)h;
    int left = 0, top = 0, right = 0, bottom = 0;
    const double min_short = 56.0;
    if ((w < h ? w : h) < min_short) {
        double nw = w <= h ? min_short : w, nh = w <= h ? h : min_short;
        const int pw = (int)(nw - w), ph = (int)(nh - h);
        left += pw / 2, right += pw - pw / 2, top += ph / 2, bottom += ph - ph / 2;
        w = nw, h = nh;
    }
    const double gw = ceil(w / grid) * grid, gh = ceil(h / grid) * grid;
    if (gw != w || gh != h) {
        const int pw = (int)(gw - w), ph = (int)(gh - h);
        left += pw / 2, right += pw - pw / 2, top += ph / 2, bottom += ph - ph / 2;
    }
    out[0] = sw0, out[1] = sh0, out[2] = left, out[3] = top, out[4] = right, out[5] = bottom;
}

int orc_bake_pad(const uint8_t* rgb, int w0, int h0, int longest, int grid, uint8_t* out) {
    int p[6];
    orc_bake_plan(longest, grid, w0, h0, p);
    if (p[0] != w0 || p[1] != h0) return -1;
    const int fw = p[0] + p[2] + p[4], fh = p[1] + p[3] + p[5];
    memset(out, 255, (size_t)fw * fh * 3);
    for (int y = 0; y < h0; y++) memcpy(out + ((size_t)(y + p[3]) * fw + p[2]) * 3, rgb + (size_t)y * w0 * 3, (size_t)w0 * 3);
    return 0;
}

/* ---- the bake's Lanczos-3 resize -------------------------------------------------------------------------------- */
static float sinc_f(float t) {
    const float a = t * 3.14159265358979323846f;
    return t == 0.0f ? 1.0f : sinf(a) / a;
}
static float lanczos3(float x) { return fabsf(x) < 3.0f ? sinc_f(x) * sinc_f(x / 3.0f) : 0.0f; }

int orc_resize_taps(int in, int out, int o, int* left, float* w, int cap) {
    const float ratio = (float)in / (float)out;
    const float sratio = ratio < 1.0f ? 1.0f : ratio;
    const float support = 3.0f * sratio;
    float centre = ((float)o + 0.5f) * ratio;
    long l = (long)floorf(centre - support), r = (long)ceilf(centre + support);
    if (l < 0) l = 0;
    if (l > in - 1) l = in - 1;
    if (r < l + 1) r = l + 1;
    if (r > in) r = in;
    centre -= 0.5f;
    const int n = (int)(r - l);
    if (n > cap) return -1;
    float sum = 0.0f;
    for (int i = 0; i < n; i++) {
        w[i] = lanczos3(((float)(l + i) - centre) / sratio);
        sum += w[i];
    }
    for (int i = 0; i < n; i++) w[i] /= sum;
    *left = (int)l;
    return n;
}

int orc_resize_lanczos3(const uint8_t* rgb, int w0, int h0, int w, int h, uint8_t* out) {
    enum { CAP = 4096 };
    float* tmp = (float*)malloc(sizeof(float) * (size_t)w0 * h * 3);
    float* wt = (float*)malloc(sizeof(float) * CAP);
    for (int y = 0; y < h; y++) { /* vertical: u8 → f32 [h][w0][3] */
        int l, n = orc_resize_taps(h0, h, y, &l, wt, CAP);
        if (n < 0) { free(tmp), free(wt); return -1; }
        for (int x = 0; x < w0; x++)
            for (int c = 0; c < 3; c++) {
                float t = 0.0f;
                for (int i = 0; i < n; i++) t += (float)rgb[((size_t)(l + i) * w0 + x) * 3 + c] * wt[i];
                tmp[((size_t)y * w0 + x) * 3 + c] = t;
            }
    }
    for (int x = 0; x < w; x++) { /* horizontal: f32 → u8 [h][w][3] */
        int l, n = orc_resize_taps(w0, w, x, &l, wt, CAP);
        if (n < 0) { free(tmp), free(wt); return -1; }
        for (int y = 0; y < h; y++)
            for (int c = 0; c < 3; c++) {
                float t = 0.0f;
                for (int i = 0; i < n; i++) t += tmp[((size_t)y * w0 + l + i) * 3 + c] * wt[i];
                t = t < 0.0f ? 0.0f : (t > 255.0f ? 255.0f : t);
                out[((size_t)y * w + x) * 3 + c] = (uint8_t)roundf(t);
            }
    }
    free(tmp);
    free(wt);
    return 0;
}

int orc_bake(const uint8_t* rgb, int w0, int h0, int longest, int grid, uint8_t* out) {
    int p[6];
    orc_bake_plan(longest, grid, w0, h0, p);
    const int fw = p[0] + p[2] + p[4], fh = p[1] + p[3] + p[5];
    const uint8_t* src = rgb;
    uint8_t* scaled = NULL;
    if (p[0] != w0 || p[1] != h0) {
        scaled = (uint8_t*)malloc((size_t)p[0] * p[1] * 3);
        if (orc_resize_lanczos3(rgb, w0, h0, p[0], p[1], scaled)) { free(scaled); return -1; }
        src = scaled;
    }
    memset(out, 255, (size_t)fw * fh * 3);
    for (int y = 0; y < p[1]; y++)
        memcpy(out + ((size_t)(y + p[3]) * fw + p[2]) * 3, src + (size_t)y * p[0] * 3, (size_t)p[0] * 3);
    free(scaled);
    return 0;
}
