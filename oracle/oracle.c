/*
 * oracle.c — CPU restatement of the reference's q8_0 text-decode path. TEST INFRASTRUCTURE ONLY: the checker for
 * libocrcuda.so's kernels and the timed CPU baseline; never linked into or called by the product.
 * Reference citations per function are in oracle.h and beside each definition below.
 * Built with -O3 -fopenmp -ffp-contract=off (Rust/WGSL semantics: no fused multiply-add unless written).
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ------------------------------------------------------------------------------------------------------------------ */
/* synthetic data                                                                                                     */

/* SplitMix64 as ocr_decode::sampling::Rng::next (sampling.rs:27-34), addressed by output index: output i is the mix of
 * the state after i+1 increments. */
uint64_t orc_splitmix64_at(uint64_t seed, uint64_t i) {
    uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t orc_substream(uint64_t seed, uint64_t k) { return orc_splitmix64_at(seed ^ 0x6F63722D62323030ull, k); }

static inline int32_t u16sum4(uint64_t z) {
    return (int32_t)(z & 0xffff) + (int32_t)((z >> 16) & 0xffff) + (int32_t)((z >> 32) & 0xffff) + (int32_t)(z >> 48);
}

float orc_gauss(uint64_t seed, uint64_t i) {
    int32_t s = u16sum4(orc_splitmix64_at(seed, 3 * i)) + u16sum4(orc_splitmix64_at(seed, 3 * i + 1)) +
                u16sum4(orc_splitmix64_at(seed, 3 * i + 2)) - 6 * 65535;
    return (float)s * (1.0f / 65536.0f);
}

void orc_fill_gauss(float* out, size_t n, uint64_t seed, float sigma) {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) out[i] = sigma * orc_gauss(seed, i);
}

void orc_fill_norm(float* out, size_t n, uint64_t seed) {
    for (size_t i = 0; i < n; i++) {
        float u = (float)(orc_splitmix64_at(seed, i) >> 40) / 16777216.0f * 2.0f - 1.0f;
        out[i] = 1.0f + 0.01f * u;
    }
}

void orc_fill_ids(int32_t* out, size_t n, uint64_t seed, uint32_t n_vocab) {
    for (size_t i = 0; i < n; i++) out[i] = (int32_t)(((orc_splitmix64_at(seed, i) >> 32) * (uint64_t)n_vocab) >> 32);
}

/* ------------------------------------------------------------------------------------------------------------------ */
/* f16: half 2.7.1's f16::from_f32 / to_f32 (round to nearest even, subnormals kept, NaN quieted)                     */

uint16_t orc_f16_from_f32(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u, exp = (x >> 23) & 0xffu, man = x & 0x7fffffu;
    if (exp == 0xffu) return (uint16_t)(man == 0 ? (sign | 0x7c00u) : (sign | 0x7e00u | (man >> 13)));
    int e = (int)exp - 127 + 15;
    if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        int shift = 14 - e;
        uint32_t hm = man >> shift, rem = man & ((1u << shift) - 1u), halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (hm & 1u))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t hm = man >> 13, rem = man & 0x1fffu;
    uint32_t out = sign | ((uint32_t)e << 10) | hm;
    if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) out++;
    return (uint16_t)out;
}

float orc_f32_from_f16(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16, exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, x;
    if (exp == 0) {
        float v = (float)man * (1.0f / 16777216.0f);
        return sign ? -v : v;
    }
    if (exp == 31) x = sign | 0x7f800000u | (man << 13);
    else x = sign | ((exp + 112u) << 23) | (man << 13);
    float f;
    memcpy(&f, &x, 4);
    return f;
}

/* ------------------------------------------------------------------------------------------------------------------ */
/* q8_0: text.rs:676-691 (ggml quantize_row_q8_0_ref): d = amax/127 stored f16, id = 1/d from the unrounded d,
 * q = round(x*id) half away from zero, saturating like Rust's `as i8`; dequant = q * f32(d) (ocr-gguf lib.rs:500-507) */

static inline int8_t sat_i8(float v) {
    if (v != v) return 0;
    if (v >= 127.0f) return 127;
    if (v <= -128.0f) return -128;
    return (int8_t)v;
}

static void quantize_block(const float* x, uint8_t* blk, float* deq) {
    float amax = 0.0f;
    for (int j = 0; j < 32; j++) {
        float a = fabsf(x[j]);
        if (a > amax) amax = a; /* f32::max ignores NaN */
    }
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t dh = orc_f16_from_f32(d);
    blk[0] = (uint8_t)(dh & 0xff);
    blk[1] = (uint8_t)(dh >> 8);
    float df = orc_f32_from_f16(dh);
    for (int j = 0; j < 32; j++) {
        int8_t q = sat_i8(roundf(x[j] * id));
        blk[2 + j] = (uint8_t)q;
        if (deq) deq[j] = (float)q * df;
    }
}

void orc_quantize_q8_0(const float* x, size_t n, uint8_t* blocks, float* deq) {
#pragma omp parallel for schedule(static)
    for (size_t b = 0; b < n / 32; b++) quantize_block(x + b * 32, blocks + b * 34, deq ? deq + b * 32 : NULL);
}

void orc_dequantize_q8_0(const uint8_t* blocks, size_t n, float* out) {
#pragma omp parallel for schedule(static)
    for (size_t b = 0; b < n / 32; b++) {
        const uint8_t* blk = blocks + b * 34;
        float d = orc_f32_from_f16((uint16_t)(blk[0] | (blk[1] << 8)));
        for (int j = 0; j < 32; j++) out[b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
    }
}

void orc_synth_q8_0(uint8_t* blocks, size_t n, uint64_t seed, float sigma) {
#pragma omp parallel for schedule(static)
    for (size_t b = 0; b < n / 32; b++) {
        float x[32];
        for (int j = 0; j < 32; j++) x[j] = sigma * orc_gauss(seed, b * 32 + j);
        quantize_block(x, blocks + b * 34, NULL);
    }
}

/* ------------------------------------------------------------------------------------------------------------------ */
/* primitive ops                                                                                                      */

/* text.rs:132-142: theta = (f32)pos * base.powf(-(2i as f32) / d as f32); (cos, sin) in f32 (glibc, as Rust's f32) */
void orc_rope_table(float base, int d_head, int n_pos, float* out) {
    int half = d_head / 2;
    for (int pos = 0; pos < n_pos; pos++)
        for (int i = 0; i < half; i++) {
            float theta = (float)pos * powf(base, -(float)(2 * i) / (float)d_head);
            out[((size_t)pos * half + i) * 2] = cosf(theta);
            out[((size_t)pos * half + i) * 2 + 1] = sinf(theta);
        }
}

/* rms_norm.wgsl:37: 1 / sqrt(mean(x^2) + eps), the sum of squares in f64 */
float orc_rms_scale(const float* x, int k, float eps) {
    double s = 0.0;
    for (int i = 0; i < k; i++) s += (double)x[i] * (double)x[i];
    return 1.0f / sqrtf((float)(s / k) + eps);
}

/* per-block f32 dot then x d (dmv_dot.wgsl:7-29, matvec_q8_0.wgsl:36-56), blocks summed in f64 */
static inline double row_dot_q8_0(const uint8_t* row, int nb, const float* x) {
    double s = 0.0;
    for (int b = 0; b < nb; b++) {
        const uint8_t* blk = row + (size_t)b * 34;
        const int8_t* q = (const int8_t*)(blk + 2);
        const float* xb = x + b * 32;
        float dot = 0.0f;
#pragma omp simd reduction(+ : dot)
        for (int j = 0; j < 32; j++) dot += (float)q[j] * xb[j];
        s += (double)dot * (double)orc_f32_from_f16((uint16_t)(blk[0] | (blk[1] << 8)));
    }
    return s;
}

void orc_matvec_q8_0_serial(const uint8_t* w, int rows, int k, const float* x, float* y, int accumulate) {
    int nb = k / 32;
    for (int r = 0; r < rows; r++) {
        float v = (float)row_dot_q8_0(w + (size_t)r * nb * 34, nb, x);
        y[r] = accumulate ? y[r] + v : v;
    }
}

void orc_matvec_q8_0(const uint8_t* w, int rows, int k, const float* x, float* y, int accumulate) {
    int nb = k / 32;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        float v = (float)row_dot_q8_0(w + (size_t)r * nb * 34, nb, x);
        y[r] = accumulate ? y[r] + v : v;
    }
}

/* qkv_post.wgsl:44-72: per-head RMSNorm (x * scale * w), then NEOX pairs (i, i + d/2) rotated by the table row */
void orc_head_norm_rope(const float* in, const float* w, const float* cs, int d, float eps, float* out) {
    float scale = orc_rms_scale(in, d, eps);
    float y[256];
    for (int i = 0; i < d; i++) y[i] = in[i] * scale * w[i];
    int half = d / 2;
    for (int i = 0; i < half; i++) {
        float c = cs[2 * i], s = cs[2 * i + 1];
        out[i] = y[i] * c - y[i + half] * s;
        out[i + half] = y[i] * s + y[i + half] * c;
    }
}

/* softmax(q . k_j * scale) . v over j < n_keys, K/V f16 (the tests' CPU reference, text.rs:813-822), in f64 */
void orc_attend(const float* q, const uint16_t* k, const uint16_t* v, int n_keys, int stride, int d, float scale,
                float* out) {
    double* sc = (double*)malloc(sizeof(double) * (size_t)(n_keys > 0 ? n_keys : 1));
    double mx = -INFINITY;
    for (int j = 0; j < n_keys; j++) {
        const uint16_t* kj = k + (size_t)j * stride;
        double s = 0.0;
        for (int i = 0; i < d; i++) s += (double)q[i] * (double)orc_f32_from_f16(kj[i]);
        sc[j] = s * (double)scale;
        if (sc[j] > mx) mx = sc[j];
    }
    double z = 0.0;
    for (int j = 0; j < n_keys; j++) {
        sc[j] = exp(sc[j] - mx);
        z += sc[j];
    }
    double acc[256];
    for (int i = 0; i < d; i++) acc[i] = 0.0;
    for (int j = 0; j < n_keys; j++) {
        const uint16_t* vj = v + (size_t)j * stride;
        double p = sc[j] / z;
        for (int i = 0; i < d; i++) acc[i] += p * (double)orc_f32_from_f16(vj[i]);
    }
    for (int i = 0; i < d; i++) out[i] = (float)acc[i];
    free(sc);
}

/* ------------------------------------------------------------------------------------------------------------------ */
/* the sampler: sampling.rs:38-62 (greedy branch)                                                                     */

void orc_apply_window_penalty(float* logits, float rp, int window, const int32_t* history, int n_hist) {
    int start = n_hist > window ? n_hist - window : 0;
    for (int j = start; j < n_hist; j++) {
        int32_t t = history[j], first = 1;
        for (int k = start; k < j; k++)
            if (history[k] == t) {
                first = 0;
                break;
            }
        if (!first) continue;
        float l = logits[t];
        logits[t] = l < 0.0f ? l * rp : l / rp;
    }
}

int32_t orc_choose_greedy(float* logits, int n_vocab, float rp, int window, float fp, const int32_t* history,
                          int n_hist, const int32_t* count_tok, const uint32_t* count_n, int n_counts) {
    if (rp != 1.0f) orc_apply_window_penalty(logits, rp, window, history, n_hist);
    if (fp > 0.0f)
        for (int i = 0; i < n_counts; i++) logits[count_tok[i]] -= fp * (float)count_n[i];
    int best = 0;
    for (int i = 0; i < n_vocab; i++)
        if (logits[i] > logits[best]) best = i;
    return best;
}

/* ------------------------------------------------------------------------------------------------------------------ */
/* the decoder: text.rs:4-10 (graph), 437-521 (prefill), 540-578 (one decode step on the F32 reference path)         */

struct orc_model {
    orc_cfg cfg;
    void** t;          /* [n_layer][ORC_N_KINDS] */
    size_t* nbytes;    /* same shape */
    uint8_t* tok_embd; /* [n_vocab][dim] q8_0 */
    float* output_norm;
};

struct orc_session {
    const orc_model* m;
    int n_ctx, n_past;
    int n_layer; /* its own count: a session may be freed after its model */
    uint16_t** k; /* [n_layer] → [n_ctx][kvd] f16 */
    uint16_t** v;
    float* rope; /* [n_ctx][d_head/2][2] */
};

static void kind_shape(const orc_cfg* c, int kind, size_t* rows, size_t* cols) {
    size_t qd = (size_t)c->n_head * c->d_head, kvd = (size_t)c->n_kv * c->d_head, d = c->dim, f = c->n_ff;
    switch (kind) {
    case ORC_Q: *rows = qd; *cols = d; break;
    case ORC_K: case ORC_V: *rows = kvd; *cols = d; break;
    case ORC_O: *rows = d; *cols = qd; break;
    case ORC_GATE: case ORC_UP: *rows = f; *cols = d; break;
    case ORC_DOWN: *rows = d; *cols = f; break;
    case ORC_Q_NORM: case ORC_K_NORM: *rows = 1; *cols = c->d_head; break;
    default: *rows = 1; *cols = d; break; /* attn_norm, ffn_norm */
    }
}

static int is_norm(int kind) {
    return kind == ORC_ATTN_NORM || kind == ORC_Q_NORM || kind == ORC_K_NORM || kind == ORC_FFN_NORM;
}

orc_model* orc_model_alloc(const orc_cfg* cfg) {
    orc_model* m = (orc_model*)calloc(1, sizeof(orc_model));
    m->cfg = *cfg;
    size_t n = (size_t)cfg->n_layer * ORC_N_KINDS;
    m->t = (void**)calloc(n, sizeof(void*));
    m->nbytes = (size_t*)calloc(n, sizeof(size_t));
    for (int l = 0; l < cfg->n_layer; l++)
        for (int k = 0; k < ORC_N_KINDS; k++) {
            size_t r, c;
            kind_shape(cfg, k, &r, &c);
            size_t nb = is_norm(k) ? r * c * 4 : r * c / 32 * 34;
            m->nbytes[l * ORC_N_KINDS + k] = nb;
            m->t[l * ORC_N_KINDS + k] = malloc(nb);
        }
    m->tok_embd = (uint8_t*)malloc((size_t)cfg->n_vocab * cfg->dim / 32 * 34);
    m->output_norm = (float*)malloc(sizeof(float) * cfg->dim);
    return m;
}

orc_model* orc_model_synthetic(const orc_cfg* cfg, uint64_t seed, float sigma_w, float sigma_e) {
    orc_model* m = orc_model_alloc(cfg);
    for (int l = 0; l < cfg->n_layer; l++)
        for (int k = 0; k < ORC_N_KINDS; k++) {
            size_t r, c;
            kind_shape(cfg, k, &r, &c);
            uint64_t s = orc_substream(seed, (uint64_t)l * 16 + k);
            if (is_norm(k)) orc_fill_norm((float*)m->t[l * ORC_N_KINDS + k], r * c, s);
            else orc_synth_q8_0((uint8_t*)m->t[l * ORC_N_KINDS + k], r * c, s, sigma_w);
        }
    orc_synth_q8_0(m->tok_embd, (size_t)cfg->n_vocab * cfg->dim, orc_substream(seed, ORC_TOK_EMBD_STREAM), sigma_e);
    orc_fill_norm(m->output_norm, cfg->dim, orc_substream(seed, ORC_OUTPUT_NORM_STREAM));
    return m;
}

void orc_model_free(orc_model* m) {
    if (!m) return;
    for (size_t i = 0; i < (size_t)m->cfg.n_layer * ORC_N_KINDS; i++) free(m->t[i]);
    free(m->t);
    free(m->nbytes);
    free(m->tok_embd);
    free(m->output_norm);
    free(m);
}

void* orc_model_tensor(orc_model* m, int layer, int kind, size_t* nbytes) {
    if (layer < 0) {
        if (kind == 0) {
            if (nbytes) *nbytes = (size_t)m->cfg.n_vocab * m->cfg.dim / 32 * 34;
            return m->tok_embd;
        }
        if (nbytes) *nbytes = sizeof(float) * m->cfg.dim;
        return m->output_norm;
    }
    if (nbytes) *nbytes = m->nbytes[layer * ORC_N_KINDS + kind];
    return m->t[layer * ORC_N_KINDS + kind];
}

const orc_cfg* orc_model_cfg(const orc_model* m) { return &m->cfg; }

#define T(m, l, k) ((m)->t[(l) * ORC_N_KINDS + (k)])

orc_session* orc_session_new(const orc_model* m, int n_ctx) {
    const orc_cfg* c = &m->cfg;
    orc_session* s = (orc_session*)calloc(1, sizeof(orc_session));
    s->m = m;
    s->n_ctx = n_ctx;
    s->n_layer = c->n_layer;
    size_t kvd = (size_t)c->n_kv * c->d_head;
    s->k = (uint16_t**)calloc(c->n_layer, sizeof(uint16_t*));
    s->v = (uint16_t**)calloc(c->n_layer, sizeof(uint16_t*));
    for (int l = 0; l < c->n_layer; l++) {
        s->k[l] = (uint16_t*)calloc((size_t)n_ctx * kvd, 2);
        s->v[l] = (uint16_t*)calloc((size_t)n_ctx * kvd, 2);
    }
    s->rope = (float*)malloc(sizeof(float) * (size_t)n_ctx * c->d_head);
    orc_rope_table(c->rope_base, c->d_head, n_ctx, s->rope);
    return s;
}

void orc_session_free(orc_session* s) {
    if (!s) return;
    for (int l = 0; l < s->n_layer; l++) {
        free(s->k[l]);
        free(s->v[l]);
    }
    free(s->k);
    free(s->v);
    free(s->rope);
    free(s);
}

int orc_session_n_past(const orc_session* s) { return s->n_past; }
void orc_session_set_n_past(orc_session* s, int n_past) { s->n_past = n_past; }
const uint16_t* orc_session_k(const orc_session* s, int layer) { return s->k[layer]; }
const uint16_t* orc_session_v(const orc_session* s, int layer) { return s->v[layer]; }

/* overwrite KV rows [row0, row0 + n) of a layer with given f16 rows ([n][kvd]): a test takes the device's cache as the
 * oracle's, so the oracle's decode step checks the device's decode step alone (not its prefill) */
int orc_session_set_kv(orc_session* s, int layer, int row0, int n, const uint16_t* k, const uint16_t* v) {
    const orc_cfg* c = &s->m->cfg;
    const size_t kvd = (size_t)c->n_kv * c->d_head;
    if (layer < 0 || layer >= c->n_layer || row0 < 0 || n < 0 || row0 + n > s->n_ctx) return 1;
    memcpy(s->k[layer] + (size_t)row0 * kvd, k, (size_t)n * kvd * 2);
    memcpy(s->v[layer] + (size_t)row0 * kvd, v, (size_t)n * kvd * 2);
    return 0;
}

/* Y[L][N] = X[L][K] . deq(W[N][K])^T (+ Y if acc): prefill projections (the tiled matmul's product, text.rs:485-512) */
static void gemm_q8_0(const uint8_t* w, int n, int k, const float* x, int l, float* y, int acc) {
    const int TN = 32;
    int nb = k / 32;
#pragma omp parallel
    {
        float* wt = (float*)malloc(sizeof(float) * (size_t)TN * k);
#pragma omp for schedule(dynamic, 1)
        for (int n0 = 0; n0 < n; n0 += TN) {
            int tn = n - n0 < TN ? n - n0 : TN;
            for (int r = 0; r < tn; r++) {
                const uint8_t* row = w + (size_t)(n0 + r) * nb * 34;
                for (int b = 0; b < nb; b++) {
                    const uint8_t* blk = row + (size_t)b * 34;
                    float d = orc_f32_from_f16((uint16_t)(blk[0] | (blk[1] << 8)));
                    for (int j = 0; j < 32; j++) wt[(size_t)r * k + b * 32 + j] = (float)(int8_t)blk[2 + j] * d;
                }
            }
            for (int i = 0; i < l; i++) {
                const float* xi = x + (size_t)i * k;
                for (int r = 0; r < tn; r++) {
                    const float* wr = wt + (size_t)r * k;
                    float s = 0.0f;
#pragma omp simd reduction(+ : s)
                    for (int j = 0; j < k; j++) s += xi[j] * wr[j];
                    float* yo = y + (size_t)i * n + n0 + r;
                    *yo = acc ? *yo + s : s;
                }
            }
        }
        free(wt);
    }
}

static void rms_rows(const float* x, const float* w, float* y, int rows, int dim, float eps) {
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++) {
        float sc = orc_rms_scale(x + (size_t)r * dim, dim, eps);
        for (int i = 0; i < dim; i++) y[(size_t)r * dim + i] = x[(size_t)r * dim + i] * sc * w[i];
    }
}

static void embed_row(const orc_model* m, int32_t tok, float* x) {
    int d = m->cfg.dim;
    orc_dequantize_q8_0(m->tok_embd + (size_t)tok * d / 32 * 34, d, x);
}

/* the layers over n rows at positions pos0..pos0+n-1 (x [n][dim] updated in place); decode = n 1 */
static void layers(orc_session* s, float* x, int n, int pos0) {
    const orc_model* m = s->m;
    const orc_cfg* c = &m->cfg;
    int d = c->dim, f = c->n_ff, dh = c->d_head, qd = c->n_head * dh, kvd = c->n_kv * dh, half = dh / 2;
    int grp = c->n_head / c->n_kv;
    float scale = 1.0f / sqrtf((float)dh);
    float* h = (float*)malloc(sizeof(float) * (size_t)n * d);
    float* q = (float*)malloc(sizeof(float) * (size_t)n * qd);
    float* kr = (float*)malloc(sizeof(float) * (size_t)n * kvd);
    float* vr = (float*)malloc(sizeof(float) * (size_t)n * kvd);
    float* a = (float*)malloc(sizeof(float) * (size_t)n * qd);
    float* g = (float*)malloc(sizeof(float) * (size_t)n * f);
    float* u = (float*)malloc(sizeof(float) * (size_t)n * f);
    for (int l = 0; l < c->n_layer; l++) {
        rms_rows(x, (const float*)T(m, l, ORC_ATTN_NORM), h, n, d, c->eps);
        if (n == 1) {
            orc_matvec_q8_0((const uint8_t*)T(m, l, ORC_Q), qd, d, h, q, 0);
            orc_matvec_q8_0((const uint8_t*)T(m, l, ORC_K), kvd, d, h, kr, 0);
            orc_matvec_q8_0((const uint8_t*)T(m, l, ORC_V), kvd, d, h, vr, 0);
        } else {
            gemm_q8_0((const uint8_t*)T(m, l, ORC_Q), qd, d, h, n, q, 0);
            gemm_q8_0((const uint8_t*)T(m, l, ORC_K), kvd, d, h, n, kr, 0);
            gemm_q8_0((const uint8_t*)T(m, l, ORC_V), kvd, d, h, n, vr, 0);
        }
        /* q / k: per-head norm + RoPE; K, V → the f16 cache rows (qkv_post.wgsl) */
#pragma omp parallel for schedule(static)
        for (int t = 0; t < n; t++) {
            const float* cs = s->rope + (size_t)(pos0 + t) * half * 2;
            float tmp[256];
            for (int hh = 0; hh < c->n_head; hh++) {
                float* qh = q + (size_t)t * qd + hh * dh;
                orc_head_norm_rope(qh, (const float*)T(m, l, ORC_Q_NORM), cs, dh, c->eps, tmp);
                memcpy(qh, tmp, sizeof(float) * dh);
            }
            uint16_t* krow = s->k[l] + (size_t)(pos0 + t) * kvd;
            uint16_t* vrow = s->v[l] + (size_t)(pos0 + t) * kvd;
            for (int j = 0; j < c->n_kv; j++) {
                orc_head_norm_rope(kr + (size_t)t * kvd + j * dh, (const float*)T(m, l, ORC_K_NORM), cs, dh, c->eps,
                                   tmp);
                for (int i = 0; i < dh; i++) krow[j * dh + i] = orc_f16_from_f32(tmp[i]);
            }
            for (int i = 0; i < kvd; i++) vrow[i] = orc_f16_from_f32(vr[(size_t)t * kvd + i]);
        }
        /* causal GQA attention over the cache (q head hh → kv head hh / grp) */
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
        for (int t = 0; t < n; t++)
            for (int hh = 0; hh < c->n_head; hh++) {
                int kh = hh / grp;
                orc_attend(q + (size_t)t * qd + hh * dh, s->k[l] + kh * dh, s->v[l] + kh * dh, pos0 + t + 1, kvd, dh,
                           scale, a + (size_t)t * qd + hh * dh);
            }
        if (n == 1) orc_matvec_q8_0((const uint8_t*)T(m, l, ORC_O), d, qd, a, x, 1);
        else gemm_q8_0((const uint8_t*)T(m, l, ORC_O), d, qd, a, n, x, 1);
        rms_rows(x, (const float*)T(m, l, ORC_FFN_NORM), h, n, d, c->eps);
        if (n == 1) {
            orc_matvec_q8_0((const uint8_t*)T(m, l, ORC_GATE), f, d, h, g, 0);
            orc_matvec_q8_0((const uint8_t*)T(m, l, ORC_UP), f, d, h, u, 0);
        } else {
            gemm_q8_0((const uint8_t*)T(m, l, ORC_GATE), f, d, h, n, g, 0);
            gemm_q8_0((const uint8_t*)T(m, l, ORC_UP), f, d, h, n, u, 0);
        }
#pragma omp parallel for schedule(static)
        for (size_t i = 0; i < (size_t)n * f; i++) {
            double gv = g[i];
            g[i] = (float)(gv / (1.0 + exp(-gv)) * (double)u[i]);
        }
        if (n == 1) orc_matvec_q8_0((const uint8_t*)T(m, l, ORC_DOWN), d, f, g, x, 1);
        else gemm_q8_0((const uint8_t*)T(m, l, ORC_DOWN), d, f, g, n, x, 1);
    }
    free(h); free(q); free(kr); free(vr); free(a); free(g); free(u);
}

/* text.rs:655-658: output_norm, then the tied token_embd matvec */
static void head(const orc_model* m, const float* x, float* logits) {
    const orc_cfg* c = &m->cfg;
    float* h = (float*)malloc(sizeof(float) * c->dim);
    rms_rows(x, m->output_norm, h, 1, c->dim, c->eps);
    orc_matvec_q8_0(m->tok_embd, c->n_vocab, c->dim, h, logits, 0);
    free(h);
}

int orc_prefill(orc_session* s, const int32_t* ids, const float* embd, int n, float* logits) {
    const orc_cfg* c = &s->m->cfg;
    if (n <= 0 || s->n_past + n > s->n_ctx) return -1;
    float* x = (float*)malloc(sizeof(float) * (size_t)n * c->dim);
    for (int i = 0; i < n; i++) {
        if (ids && ids[i] >= 0) {
            if (ids[i] >= c->n_vocab) { free(x); return -2; }
            embed_row(s->m, ids[i], x + (size_t)i * c->dim);
        } else {
            memcpy(x + (size_t)i * c->dim, embd + (size_t)i * c->dim, sizeof(float) * c->dim);
        }
    }
    layers(s, x, n, s->n_past);
    if (logits) head(s->m, x + (size_t)(n - 1) * c->dim, logits);
    s->n_past += n;
    free(x);
    return 0;
}

int orc_step(orc_session* s, int32_t tok, float* logits) {
    const orc_cfg* c = &s->m->cfg;
    if (tok < 0 || tok >= c->n_vocab) return -2;
    if (s->n_past + 1 > s->n_ctx) return -1;
    float* x = (float*)malloc(sizeof(float) * c->dim);
    embed_row(s->m, tok, x);
    layers(s, x, 1, s->n_past);
    head(s->m, x, logits);
    s->n_past += 1;
    free(x);
    return 0;
}

/* the gap between the largest and the second largest logit, and the second one's index (the first of equals) */
static float top2_margin(const float* l, int n, int32_t* second) {
    float b1 = -INFINITY, b2 = -INFINITY;
    int32_t i1 = -1, i2 = -1;
    for (int i = 0; i < n; i++) {
        float v = l[i];
        if (v > b1) { b2 = b1; i2 = i1; b1 = v; i1 = i; }
        else if (v > b2) { b2 = v; i2 = i; }
    }
    if (second) *second = i2;
    return b1 - b2;
}

/* text.rs:587-625 + Choice (text.rs:185-231): history seed = the last `window` ids, then every chosen token */
int orc_decode(orc_session* s, const float* first_logits, float rp, int window, float fp, const int32_t* history,
               int n_hist, int max_new, int32_t* ids_out, float* margins_out) {
    return orc_decode_top2(s, first_logits, rp, window, fp, history, n_hist, max_new, ids_out, margins_out, NULL);
}

int orc_decode_top2(orc_session* s, const float* first_logits, float rp, int window, float fp, const int32_t* history,
                    int n_hist, int max_new, int32_t* ids_out, float* margins_out, int32_t* second_out) {
    const orc_cfg* c = &s->m->cfg;
    int seed = n_hist > window ? window : n_hist;
    int32_t* hist = (int32_t*)malloc(sizeof(int32_t) * (size_t)(seed + max_new));
    memcpy(hist, history + (n_hist - seed), sizeof(int32_t) * seed);
    uint32_t* counts = fp > 0.0f ? (uint32_t*)calloc(c->n_vocab, 4) : NULL;
    int32_t* ctok = fp > 0.0f ? (int32_t*)malloc(sizeof(int32_t) * (size_t)max_new) : NULL;
    uint32_t* cnt = fp > 0.0f ? (uint32_t*)malloc(sizeof(uint32_t) * (size_t)max_new) : NULL;
    int n_distinct = 0;
    float* l = (float*)malloc(sizeof(float) * c->n_vocab);
    memcpy(l, first_logits, sizeof(float) * c->n_vocab);
    int rc = 0;
    for (int i = 0; i < max_new; i++) {
        if (i > 0 && (rc = orc_step(s, ids_out[i - 1], l)) != 0) break;
        if (fp > 0.0f) {
            n_distinct = 0;
            for (int j = 0; j < i; j++) {
                int32_t t = ids_out[j];
                int seen = 0;
                for (int k = 0; k < n_distinct; k++)
                    if (ctok[k] == t) { seen = 1; break; }
                if (!seen) { ctok[n_distinct] = t; cnt[n_distinct] = counts[t]; n_distinct++; }
            }
        }
        int32_t t = orc_choose_greedy(l, c->n_vocab, rp, window, fp, hist, seed + i, ctok, cnt, n_distinct);
        int32_t second = -1;
        const float margin = top2_margin(l, c->n_vocab, &second);
        if (margins_out) margins_out[i] = margin;
        if (second_out) second_out[i] = second;
        ids_out[i] = t;
        hist[seed + i] = t;
        if (counts) counts[t]++;
    }
    free(hist); free(counts); free(ctok); free(cnt); free(l);
    return rc;
}
