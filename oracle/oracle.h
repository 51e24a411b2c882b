/*
 * oracle.h — CPU restatement of the reference's q8_0 text-decode path (TEST INFRASTRUCTURE ONLY).
 *
 * This library is the checker, never the product: only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference leg load it. The product (libocrcuda.so) never links or calls it.
 *
 * Every function restates one piece of b-straub/historic-htr-ocr (paths relative to that project):
 *   - ocr_decode::sampling::choose            app/crates/ocr-decode/src/sampling.rs:38-90
 *   - the q8_0 quantizer (ggml quantize_row_q8_0_ref, the tests' q8_0())  app/crates/ocr-wgpu/src/text.rs:676-691
 *   - q8_0 dequant / block layout             app/crates/ocr-gguf/src/lib.rs:129-135, 500-507
 *   - rope_table                              app/crates/ocr-wgpu/src/text.rs:132-142
 *   - RMSNorm                                 app/crates/ocr-wgpu/src/shaders/rms_norm.wgsl:37-39
 *   - q8_0 matvec                             app/crates/ocr-wgpu/src/shaders/matvec_q8_0.wgsl:29-73
 *   - q/k norm → RoPE NEOX → f16 KV           app/crates/ocr-wgpu/src/shaders/qkv_post.wgsl:31-83
 *   - decode attention (f32 on f16 K/V)       app/crates/ocr-wgpu/src/text.rs:813-822 (CPU ref of the tests)
 *   - SwiGLU                                  app/crates/ocr-wgpu/src/shaders/swiglu.wgsl, dmv_ffn.wgsl:46-48
 *   - the Qwen3 layer order (decode/prefill)  app/crates/ocr-wgpu/src/text.rs:4-10, 437-521, 540-578
 *   - the GPU Choice's history / window       app/crates/ocr-wgpu/src/text.rs:185-231
 * Accumulations the reference does in f32 in an adapter-dependent order are done here in f64 (the order-free limit);
 * every rounding the reference defines exactly (the penalty's f32 product / quotient, the f16 KV store, the q8_0
 * quantizer) is reproduced bit for bit. Build with -ffp-contract=off (Rust never fuses a*b+c).
 */
#ifndef OCR_ORACLE_H
#define OCR_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------- synthetic seeded data (shared spec with the product's generator) ---------- */
/* SplitMix64 (sampling.rs:24-35): the i-th output (0-based) of a stream seeded with `seed` */
uint64_t orc_splitmix64_at(uint64_t seed, uint64_t i);
/* the seed of sub-stream `k` of `seed` (one per tensor) */
uint64_t orc_substream(uint64_t seed, uint64_t k);
/* N(0,1) stand-in: Irwin–Hall sum of 12 u16 uniforms from outputs 3i..3i+2, centred, / 2^16 (exact in f32) */
float orc_gauss(uint64_t seed, uint64_t i);
/* out[i] = sigma * orc_gauss(seed, i), one f32 multiply */
void orc_fill_gauss(float* out, size_t n, uint64_t seed, float sigma);
/* out[i] = 1 + 0.01 * u, u = top 24 bits of output i mapped to [-1, 1) (the norm weights, like text.rs:1304) */
void orc_fill_norm(float* out, size_t n, uint64_t seed);
/* history ids uniform on [0, n_vocab): (output i >> 32) * n_vocab >> 32 */
void orc_fill_ids(int32_t* out, size_t n, uint64_t seed, uint32_t n_vocab);

/* ---------- f16 (half 2.7.1 semantics: round to nearest even, subnormals kept) ---------- */
uint16_t orc_f16_from_f32(float f);
float orc_f32_from_f16(uint16_t h);

/* ---------- q8_0 ---------- */
/* quantize n (multiple of 32) floats into n/32 GGUF blocks of 34 bytes (f16 d, 32 x i8); deq optional */
void orc_quantize_q8_0(const float* x, size_t n, uint8_t* blocks, float* deq);
void orc_dequantize_q8_0(const uint8_t* blocks, size_t n, float* out);
/* synthetic q8_0 tensor: sigma * gauss(substream(seed,k)) quantized (rows*cols values, cols % 32 == 0) */
void orc_synth_q8_0(uint8_t* blocks, size_t n, uint64_t seed, float sigma);

/* ---------- primitive ops ---------- */
void orc_rope_table(float base, int d_head, int n_pos, float* out /* [n_pos][d_head/2][2] */);
float orc_rms_scale(const float* x, int k, float eps);
/* y[n] = (acc ? y[n] : 0) + sum_b d_b * dot(q_b, x_b)   (W = rows x k q8_0 GGUF blocks) */
void orc_matvec_q8_0(const uint8_t* w, int rows, int k, const float* x, float* y, int accumulate);
/* head_in [128] raw → per-head RMSNorm(w) → RoPE NEOX at table row `cs` ([64][2]) → out */
void orc_head_norm_rope(const float* head_in, const float* w, const float* cs, int d, float eps, float* out);
/* decode attention of one q head over n_keys f16 keys/values (rows strided by `stride` halves) → out[d] */
void orc_attend(const float* q, const uint16_t* k, const uint16_t* v, int n_keys, int stride, int d, float scale, float* out);

/* ---------- the sampler: ocr_decode::sampling::choose, greedy branch (sampling.rs:38-62) ---------- */
/* logits penalised in place; history = the window's source (prompt tail + outputs); counts as (token, count) pairs */
int32_t orc_choose_greedy(float* logits, int n_vocab, float rp, int window, float fp, const int32_t* history,
                          int n_hist, const int32_t* count_tok, const uint32_t* count_n, int n_counts);
/* the penalty alone (for the exactness sweep, text.rs:1061-1099) */
void orc_apply_window_penalty(float* logits, float rp, int window, const int32_t* history, int n_hist);

/* ---------- the decoder ---------- */
typedef struct {
    int n_layer, dim, n_head, n_kv, d_head, n_ff, n_vocab;
    float eps, rope_base;
} orc_cfg;

typedef struct orc_model orc_model;
typedef struct orc_session orc_session;

/* tensor kinds of one layer, in the order the synthetic generator numbers its sub-streams */
enum { ORC_ATTN_NORM = 0, ORC_Q, ORC_K, ORC_V, ORC_O, ORC_Q_NORM, ORC_K_NORM, ORC_FFN_NORM, ORC_GATE, ORC_UP, ORC_DOWN,
       ORC_N_KINDS };
#define ORC_TOK_EMBD_STREAM 100000u
#define ORC_OUTPUT_NORM_STREAM 100001u

/* a synthetic model: weights sigma_w (matrices), token_embd sigma_e, norms 1 + 0.01 U(-1,1) */
orc_model* orc_model_synthetic(const orc_cfg* cfg, uint64_t seed, float sigma_w, float sigma_e);
/* an empty model whose tensors the caller fills (orc_model_tensor) */
orc_model* orc_model_alloc(const orc_cfg* cfg);
void orc_model_free(orc_model* m);
/* the raw storage of a tensor: q8_0 GGUF blocks (matrices) or f32 (norms); layer = -1 for token_embd/output_norm */
void* orc_model_tensor(orc_model* m, int layer, int kind, size_t* nbytes);
const orc_cfg* orc_model_cfg(const orc_model* m);

orc_session* orc_session_new(const orc_model* m, int n_ctx);
void orc_session_free(orc_session* s);
int orc_session_n_past(const orc_session* s);
void orc_session_set_n_past(orc_session* s, int n_past);
/* prefill n rows: ids[i] >= 0 → token_embd row, ids[i] < 0 → embd row i ([n][dim] f32); logits of the last row */
int orc_prefill(orc_session* s, const int32_t* ids, const float* embd, int n, float* logits);
/* one token at n_past → logits */
int orc_step(orc_session* s, int32_t tok, float* logits);
/* greedy decode with the windowed penalty: the first choice from `logits` (the prompt's), then step+choose */
int orc_decode(orc_session* s, const float* first_logits, float rp, int window, float fp, const int32_t* history,
               int n_hist, int max_new, int32_t* ids_out, float* margins_out);
/* orc_decode that also gives, per choice, the runner-up token (the second largest penalised logit) */
int orc_decode_top2(orc_session* s, const float* first_logits, float rp, int window, float fp, const int32_t* history,
                    int n_hist, int max_new, int32_t* ids_out, float* margins_out, int32_t* second_out);
/* KV cache rows of a layer (f16, [n_ctx][n_kv*d_head]) */
const uint16_t* orc_session_k(const orc_session* s, int layer);
const uint16_t* orc_session_v(const orc_session* s, int layer);
/* overwrite KV rows [row0, row0 + n) of a layer ([n][n_kv*d_head] f16 each); 0 = ok */
int orc_session_set_kv(orc_session* s, int layer, int row0, int n, const uint16_t* k, const uint16_t* v);

int orc_num_threads(void);
/* orc_matvec_q8_0 on the calling thread alone (for callers already inside a parallel loop) */
void orc_matvec_q8_0_serial(const uint8_t* w, int rows, int k, const float* x, float* y, int accumulate);

/* ---------- the vision encoder + projector (vision.c; vision.rs:266-423) ---------- */
typedef struct {
    int n_layer, dim, n_head, n_ff, patch, merge, image_size, proj_dim;
    float eps, rope_theta;
    float mean[3], std[3];
} orc_vcfg;

typedef struct orc_vision orc_vision;

/* tensor kinds of one encoder layer, numbered like their synthetic sub-streams */
enum { ORC_V_LN1 = 0, ORC_V_Q, ORC_V_K, ORC_V_V, ORC_V_O, ORC_V_LN2, ORC_V_GATE, ORC_V_UP, ORC_V_DOWN, ORC_V_N_KINDS };
#define ORC_V_LAYER_STREAM 200000u      /* layer l, kind k: sub-stream ORC_V_LAYER_STREAM + l * 16 + k */
#define ORC_V_PATCH_STREAM 300000u
#define ORC_V_PRE_LN_STREAM 300001u
#define ORC_V_INPUT_NORM_STREAM 300002u
#define ORC_V_MERGER_STREAM 300003u
#define ORC_V_MM1_STREAM 300004u
#define ORC_V_MM2_STREAM 300005u

/* the patch embedding's padded width: 3 * patch² rounded up to a multiple of 256 (zero columns past 3 * patch²) */
int orc_vision_patch_cols(const orc_vcfg* c);
void orc_synth_q8_0_padded(uint8_t* blocks, int rows, int cols, int valid, uint64_t seed, float sigma);
orc_vision* orc_vision_synthetic(const orc_vcfg* cfg, uint64_t seed, float sigma_w);
void orc_vision_free(orc_vision* v);
void orc_pixel_lut(const orc_vcfg* c, float* lut /* [3][256] */);
void orc_rope2d_table(float theta, int d_head, int max_pos, float* out /* [2][max_pos][d_head/4][2] */);
float orc_gelu_tanh(float x);
/* a baked image rgb [h][w][3] → out [n_tokens][proj_dim]; layers >= 0 stops after that many encoder layers and gives
 * the residual [n_patches][dim]. Returns the rows written, -1 for an image that is not baked. */
int orc_vision_encode(const orc_vision* v, const uint8_t* rgb, int w, int h, int layers, float* out);
/* the residual after the first encoder layer for the listed patch rows only ([n_rows][dim]); the keys and values of
 * every patch are computed */
int orc_vision_layer1_rows(const orc_vision* v, const uint8_t* rgb, int w, int h, const int* rows, int n_rows,
                           float* out);
/* the bake (imageops.rs:275-323): out = [scaled_w, scaled_h, left, top, right, bottom] */
void orc_bake_plan(int longest, int grid, int w0, int h0, int* out);
/* the bake of an image that needs no resize: white pads per the plan; -1 when the plan resizes */
int orc_bake_pad(const uint8_t* rgb, int w0, int h0, int longest, int grid, uint8_t* out);
/* the Lanczos-3 resampling taps of output index o (in → out samples): *left and the normalised weights; their count */
int orc_resize_taps(int in, int out, int o, int* left, float* w, int cap);
/* imageops::resize(.., Lanczos3) of the image crate 0.25: rgb [h0][w0][3] → out [h][w][3] */
int orc_resize_lanczos3(const uint8_t* rgb, int w0, int h0, int w, int h, uint8_t* out);
/* the whole bake (imageops.rs:318-323): the resize when the plan scales, then the white pads → [fh][fw][3] */
int orc_bake(const uint8_t* rgb, int w0, int h0, int longest, int grid, uint8_t* out);

#ifdef __cplusplus
}
#endif
#endif
