/*
 * ocr_cuda.h — the C ABI of libocrcuda.so, a B200 (sm_100a) q8_0 text-decode engine for the LightOnOCR-style VLM.
 *
 * It replaces, behind the same shapes of call, the wgpu text decoder of b-straub/historic-htr-ocr (paths relative to
 * that project). Each entry point names the reference interface it stands in for. All calls return an ocr_status
 * (0 = OCR_OK); on failure ocr_last_error() holds a message (per host thread). Handles are single-thread-affine, like
 * the reference's Gpu (RefCell inside, not Sync): one host thread drives one ocr_ctx. The caller owns every host
 * buffer; the library owns all device memory it allocates. Device pointers in the low-level ops (ocr_op_*) are plain
 * CUDA device addresses on the context's device; those ops run on the context's stream and return when queued unless
 * stated otherwise (ocr_ctx_sync waits).
 */
#ifndef OCR_CUDA_H
#define OCR_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int ocr_status;
enum {
    OCR_OK = 0,
    OCR_ERR_ARG = 1,      /* an argument is out of range (a token outside the vocabulary, a size, a null pointer) */
    OCR_ERR_CUDA = 2,     /* a CUDA call failed; the message has cudaGetErrorString */
    OCR_ERR_FORMAT = 3,   /* the GGUF file is malformed or holds what this engine does not run */
    OCR_ERR_IO = 4,       /* the file could not be read */
    OCR_ERR_STATE = 5,    /* the call does not fit the session's state (positions overflow, no logits yet) */
    OCR_ERR_DEVICE = 6,   /* a kernel reported a device-side error (a bounded wait gave up, a bad index) */
};

typedef struct ocr_ctx ocr_ctx;
typedef struct ocr_model ocr_model;
typedef struct ocr_session ocr_session;

/* TextConfig (app/crates/ocr-wgpu/src/text.rs:37-82) */
typedef struct {
    int32_t n_layer, dim, n_head, n_kv, d_head, n_ff, n_vocab, n_ctx_train;
    float eps, rope_base;
} ocr_text_cfg;

/* the greedy preset's knobs (app/crates/ocr-decode/src/presets.rs:18-35; Preset::greedy, temperature 0):
 * rp = repetitionPenalty (1 = off; a positive normal f32 otherwise, text.rs:154-163), window = repetitionWindow (>= 1),
 * fp = frequencyPenalty (0 = off), max_new = maxNewTokens */
typedef struct {
    float rp;
    int32_t window;
    float fp;
    int32_t max_new;
} ocr_sampler_cfg;

/* ---- errors ---------------------------------------------------------------------------------------------------- */
/* the message of the last failed call on this host thread ("" if none) — anyhow's error text in the reference */
const char* ocr_last_error(void);
/* the library's version string and the device code it carries ("sm_100a") */
const char* ocr_version(void);

/* ---- context: one device, one stream, the device arena (replaces Gpu::create, gpu.rs:1172-1324) ---------------- */
ocr_status ocr_ctx_create(int device, ocr_ctx** out);
/* releases the caller's handle. Destroy calls may come in any order: a context stays alive while a model made in it
 * does, a model while one of its sessions does; the last release frees. No handle is used after its own destroy. */
ocr_status ocr_ctx_destroy(ocr_ctx* ctx);
/* wait for everything queued on the context's stream; returns OCR_ERR_DEVICE if a kernel flagged an error */
ocr_status ocr_ctx_sync(ocr_ctx* ctx);
/* the context's cudaStream_t (as void*), for callers that order their own work against it */
ocr_status ocr_ctx_stream(ocr_ctx* ctx, void** stream);
/* bytes of device memory the library holds, by kind (GpuBytes, sampling.rs:137-146): weights, kv_cache, work */
ocr_status ocr_ctx_memory(ocr_ctx* ctx, uint64_t* weights, uint64_t* kv_cache, uint64_t* work);

/* ---- model (TextModel::load, text.rs:332-375; Gguf::from_source, ocr-gguf/src/lib.rs:300-338) -------------------- */
/* a qwen3 text GGUF: q8_0 matrices, f32 norms, tied token_embd — streamed to the device and repacked there */
ocr_status ocr_model_load_gguf(ocr_ctx* ctx, const char* path, ocr_model** out);
/* the same from bytes in memory (TensorSource for Vec<u8>, ocr-gguf/src/lib.rs:71-84) */
ocr_status ocr_model_load_gguf_memory(ocr_ctx* ctx, const void* bytes, size_t n_bytes, ocr_model** out);
/* a seeded synthetic model of the given shape, generated and quantized on the device (no file): matrices
 * sigma_w * g, token_embd sigma_e * g (g the generator's N(0,1) stand-in), norms 1 + 0.01 u — the same values, bit for
 * bit, as the CPU test generator of the same seed */
ocr_status ocr_model_synthetic(ocr_ctx* ctx, const ocr_text_cfg* cfg, uint64_t seed, float sigma_w, float sigma_e,
                               ocr_model** out);
ocr_status ocr_model_config(const ocr_model* m, ocr_text_cfg* out);
/* copy one tensor back in GGUF form (q8_0 34-byte blocks, or f32 for norms): layer -1 with kind 0 = token_embd, kind
 * 1 = output_norm; kinds of a layer: 0 attn_norm 1 q 2 k 3 v 4 o 5 q_norm 6 k_norm 7 ffn_norm 8 gate 9 up 10 down.
 * `out` NULL → *n_bytes = the size needed */
ocr_status ocr_model_tensor_gguf(const ocr_model* m, int layer, int kind, void* out, size_t* n_bytes);
/* a 64-bit FNV-1a checksum of all repacked weight bytes (identity checks across loads / generators) */
ocr_status ocr_model_checksum(const ocr_model* m, uint64_t* out);
ocr_status ocr_model_destroy(ocr_model* m);

/* ---- session: KV cache + decode scratch for `batch` independent sequences (Session, text.rs:242-434) ----------- */
/* n_ctx = positions per sequence (prompt + new tokens), <= n_ctx_train; the KV cache is allocated once, whole */
ocr_status ocr_session_create(ocr_model* m, int n_ctx, int batch, ocr_session** out);
ocr_status ocr_session_destroy(ocr_session* s);
ocr_status ocr_session_n_past(const ocr_session* s, int slot, int* out);
/* rewind a slot to n_past positions (<= its current n_past): later steps overwrite the rows beyond */
ocr_status ocr_session_rewind(ocr_session* s, int slot, int n_past);
/* copy KV rows [row0, row0 + n_rows) of one layer and slot to the host as the reference's Session holds them per
 * layer (text.rs:242-328: [n_ctx][n_kv * d_head] f16), k_out and v_out [n_rows][n_kv * 128] f16 bit patterns
 * (inspection and tests). Synchronous. */
ocr_status ocr_session_kv(const ocr_session* s, int layer, int slot, int row0, int n_rows, uint16_t* k_out,
                          uint16_t* v_out);

/* TextModel::prefill (text.rs:437-521) for one slot: n_rows rows at positions n_past…; row i is token ids[i] when
 * ids != NULL and ids[i] >= 0, else embedding row i of embd ([n_rows][dim] f32, Input::Embeddings; host or device
 * memory, e.g. the output of ocr_vision_encode). ids is a host buffer.
 * logits_out (nullable, [n_vocab]) = the last row's logits; they also stay on the device for the first choice. */
ocr_status ocr_prefill(ocr_session* s, int slot, const int32_t* ids, const float* embd, int n_rows, float* logits_out);

/* TextModel::step (text.rs:524-537): one token per slot (tok[slot] < 0 = slot idle) at each slot's n_past → logits
 * ([batch][n_vocab], nullable). The CPU token choice path: logits come back every step. */
ocr_status ocr_step(ocr_session* s, const int32_t* tok, float* logits_out);

/* TextModel::decode_gpu + Choice (text.rs:185-231, 587-625) for one slot: greedy choices with the windowed
 * repetition penalty (and frequency penalty), the token chosen on the device and fed back without a host round trip.
 * history = the window's start (prompt tail) as ocr-decode's generate gets it; choice 0 comes from the slot's current
 * logits (the prefill's or the last step's). on_token (nullable) sees each id in order; returning 0 ends the read
 * (steps already queued past it finish unseen). ids_out [max_new] gets the ids, *n_out their count. */
typedef int (*ocr_token_cb)(void* user, int32_t token);
ocr_status ocr_decode(ocr_session* s, int slot, const ocr_sampler_cfg* cfg, const int32_t* history, int n_hist,
                      ocr_token_cb on_token, void* user, int32_t* ids_out, int* n_out);

/* the per-dispatch profiler (OCR_WGPU_PROFILE's role, gpu.rs:1006-1016, 1416-1436): one decode step of every slot
 * with tok[slot] >= 0 (at its n_past, like ocr_step, logits kept on the device), run eagerly with a CUDA event after
 * each kernel. out[i] = that kernel's name, layer (-1 for the LM head), device microseconds from the previous event,
 * and the algorithmic bytes it must move (weights read once, KV rows read, activations). The slots' positions
 * advance as with ocr_step. cap entries at most; *n = the count. */
typedef struct {
    char name[32];
    int32_t layer;
    float us;
    double bytes;
} ocr_kernel_time;
/* One step of every slot with active[slot] != 0 taking one Input::Embeddings row (embd [B][dim], row b for slot b)
   at its position: TextModel::prefill of a single embedding row (text.rs:437-521), for every slot at once — the same
   KV rows and logits as ocr_prefill(s, b, NULL, row b, 1, …) slot by slot, in one batched step. logits_out
   (nullable): [B][n_vocab]. */
ocr_status ocr_step_embd(ocr_session* s, const int32_t* active, const float* embd, float* logits_out);
ocr_status ocr_profile_step(ocr_session* s, const int32_t* tok, ocr_kernel_time* out, int cap, int* n);
/* The in-chain timeline of one decode step (the same slots and tokens as ocr_profile_step): the step captured `reps`
   (2..16) times back to back into one graph whose launches are chained as the decode's graph chains them
   (programmatic dependent launch), each CTA recording %globaltimer at its start, at its dependency wait's release and
   at its end. Reports the last repetition's launches: `us` = the end of the launch's latest CTA less the end of the
   launch before it (what the launch adds to the chained step). Positions do not advance between repetitions; after
   the call each active slot holds one more token, as after ocr_profile_step. Test and inspection entry point. */
ocr_status ocr_timeline_step(ocr_session* s, const int32_t* tok, int reps, ocr_kernel_time* out, int cap, int* n);

/* the same for every slot at once (batched decode; each slot its own history): history [batch][n_hist] (a shared
 * length), ids_out [batch][max_new]. All slots run max_new choices. */
ocr_status ocr_decode_batch(ocr_session* s, const ocr_sampler_cfg* cfg, const int32_t* history, int n_hist,
                            int32_t* ids_out);

/* The page engine: Engine::read_text (app/crates/ocr-wgpu/src/engine.rs:447-524) for a stream of pages, one page per
 * slot of the session at a time (continuous batching). Between chunks of up to `chunk` decode steps, every free slot
 * takes io->next's page: its rows prefilled (as ocr_prefill), the window seeded from its history (as ocr_decode),
 * choice 0 from the prefill's logits; then the slot decodes with the others until the page's max_new choices are
 * made — the budget counts down on the device, so slots end mid-chunk without a host round trip — and io->done gets
 * the page back with its ids. All pages share cfg's penalties; cfg->max_new bounds every page's max_new. Pages come
 * and go in the caller's memory: a page's embd / ids / history must stay valid until it is done. Returns when next
 * has no page and every slot is done, when done returns 0 (pages in other slots are dropped unread), or on error. */
typedef struct {
    int64_t id;             /* the caller's page number (echoed back) */
    const int32_t* ids;     /* prompt rows: token ids (nullable: all rows from embd), as ocr_prefill */
    const float* embd;      /* [n_rows][dim] embedding rows (Input::Embeddings) */
    int32_t n_rows;
    const int32_t* history; /* the window's start, as ocr_decode */
    int32_t n_hist;
    int32_t max_new;        /* choices to make (>= 1) */
    int32_t* ids_out;       /* [max_new] the chosen ids */
    int32_t n_out;          /* set when done: the ids made */
} ocr_page;
typedef struct {
    void* user;
    int (*next)(void* user, ocr_page* page); /* fill *page, return 1; or 0 when there is no further page */
    int (*done)(void* user, ocr_page* page); /* a page is read; return 0 to stop the engine */
} ocr_page_io;
ocr_status ocr_read_pages(ocr_session* s, const ocr_sampler_cfg* cfg, int chunk, const ocr_page_io* io);

/* ocr_decode::sampling::choose, greedy branch (sampling.rs:38-62) ≡ choose_pen → choose_max → choose_pick
 * (shaders/choose_*.wgsl) on logits already on the device (d_logits [n_vocab] f32, left unchanged): the windowed
 * penalty over the DISTINCT tokens of history[n_hist - window, n_hist), the frequency penalty over (count_tok,
 * count_n) pairs (host arrays, n_counts entries), the first maximum. Returns the token in *tok (host). Synchronous. */
ocr_status ocr_sample_logits(ocr_ctx* ctx, const float* d_logits, int n_vocab, const ocr_sampler_cfg* cfg,
                             const int32_t* history, int n_hist, const int32_t* count_tok, const uint32_t* count_n,
                             int n_counts, int32_t* tok);

/* ---- the vision encoder + projector (replaces Vision, app/crates/ocr-wgpu/src/vision.rs:37-450) ------------------ */
typedef struct ocr_vision ocr_vision;

/* VisionConfig (vision.rs:37-88): the Pixtral-shaped ViT and the LightOnOCR projector. dim / n_head must be 64
 * (vision.rs:71-73), merge 2 and n_ff >= 4 dim (the 2x2 unfold, vision.rs:412-414). */
typedef struct {
    int32_t n_layer, dim, n_head, n_ff, patch, merge, image_size, proj_dim;
    float eps, rope_theta;
    float mean[3], std[3];
} ocr_vision_cfg;

/* the bake's plan (BakePlan, app/crates/ocr-core/src/imageops.rs:262-316): the image scaled to scaled_w x scaled_h
 * (longest edge <= longest, never up), then white pads on each side up to 56 px on the short edge and the grid */
typedef struct {
    int32_t scaled_w, scaled_h, left, top, right, bottom;
} ocr_bake_plan;
/* imageops.rs:275-316 plan(Bake { longest, grid }, w0, h0). Host only. */
ocr_status ocr_bake_plan_for(int longest, int grid, int w0, int h0, ocr_bake_plan* out);

/* A seeded synthetic encoder with q8_0 weights (the reference loads bf16 / f32 mmproj weights, vision.rs:131-135;
 * BASELINE config 4 asks q8_0): every matrix sigma_w * N(0,1)-like values quantised, the patch embedding's 3 p²
 * columns padded with zero columns to a multiple of 256, norms 1 + 0.01 U(-1,1). Bit-identical to the CPU
 * oracle's orc_vision_synthetic of the same seed (sub-streams 200000 + layer * 16 + kind, 300000 … 300005). */
ocr_status ocr_vision_synthetic(ocr_ctx* ctx, const ocr_vision_cfg* cfg, uint64_t seed, float sigma_w,
                                ocr_vision** out);
ocr_status ocr_vision_destroy(ocr_vision* v);
ocr_status ocr_vision_config(const ocr_vision* v, ocr_vision_cfg* out);

/* Vision::encode / encode_gpu (vision.rs:256-317): rgb [h][w][3] bytes of a BAKED image — both sides multiples of
 * patch * merge, the longest <= image_size, else OCR_ERR_ARG ("not baked"), like the reference — in host or device
 * memory. layers < 0: the image's embeddings for the text model, [n_tokens][proj_dim] f32 with n_tokens = (w / 28) *
 * (h / 28); layers = k in 0 … n_layer: the residual stream [n_patches][dim] after k encoder layers (the reference's
 * bisect hook, vision.rs:253-255). out: host or device memory of cap floats; *n_rows and *row_width (nullable) get
 * the shape. Synchronous. */
ocr_status ocr_vision_encode(ocr_vision* v, const uint8_t* rgb, int w, int h, int layers, float* out, size_t cap,
                             int* n_rows, int* row_width);
/* The bake and the encode of a page in one call: rgb [h0][w0][3] of any size (host or device), scaled per
 * ocr_bake_plan_for(image_size, patch * merge, …) on the device when its longest edge is above image_size (the
 * bake's Lanczos-3 resize, as ocr_image_bake) and placed in its white canvas — the pad is made inside the patch
 * gather, no baked copy is formed — then encoded as ocr_vision_encode(layers = -1). */
ocr_status ocr_vision_encode_page(ocr_vision* v, const uint8_t* rgb, int w0, int h0, float* out, size_t cap,
                                  int* n_rows);
/* imageops::bake (app/crates/ocr-core/src/imageops.rs:318-323) on the device: rgb [h0][w0][3] (host or device) →
 * out [out_h][out_w][3] (host or device, cap bytes): the longest edge scaled down to `longest` with the Lanczos-3
 * filter of imageops::resize (the `image` crate 0.25: separable, a vertical pass into f32 then a horizontal pass into
 * bytes, rounded half away from zero), then white pads to the `grid` per the plan. Synchronous. */
ocr_status ocr_image_bake(ocr_ctx* ctx, const uint8_t* rgb, int w0, int h0, int longest, int grid, uint8_t* out,
                          size_t cap, int* out_w, int* out_h);

/* ---- GGUF reader, host only (ocr_gguf::Gguf, app/crates/ocr-gguf/src/lib.rs:213-509) ------------------------------ */
typedef struct ocr_gguf ocr_gguf;
/* Gguf::open / Gguf::from_source (lib.rs:291-338): the header from a growing prefix, every tensor inside the file */
ocr_status ocr_gguf_open(const char* path, ocr_gguf** out);
ocr_status ocr_gguf_open_memory(const void* bytes, size_t n_bytes, ocr_gguf** out);
ocr_status ocr_gguf_close(ocr_gguf* g);
ocr_status ocr_gguf_header(const ocr_gguf* g, uint32_t* version, uint64_t* n_tensors, uint64_t* alignment,
                           uint64_t* data_offset);
/* Gguf::u32 / f32 / str / f32_array (lib.rs:415-460); a string is copied NUL-terminated into out[cap] */
ocr_status ocr_gguf_get_u32(const ocr_gguf* g, const char* key, uint32_t* out);
ocr_status ocr_gguf_get_f32(const ocr_gguf* g, const char* key, float* out);
ocr_status ocr_gguf_get_str(const ocr_gguf* g, const char* key, char* out, size_t cap);
ocr_status ocr_gguf_f32_array(const ocr_gguf* g, const char* key, float* out, size_t cap, size_t* n);
/* Gguf::info (lib.rs:462-465): ggml type (0 f32, 1 f16, 8 q8_0, 30 bf16), shape (ggml order), absolute offset */
ocr_status ocr_gguf_tensor(const ocr_gguf* g, const char* name, int* ggml_type, uint64_t shape[4], int* n_dims,
                           uint64_t* file_offset);
/* Gguf::to_f32 (lib.rs:494-509) of a small tensor (<= 1 MiB) */
ocr_status ocr_gguf_to_f32(const ocr_gguf* g, const char* name, float* out, size_t cap, size_t* n);
/* TextConfig::from_gguf + TextModel::load's tensor checks (text.rs:51-82, 111-128, 332-375), no device */
ocr_status ocr_gguf_text_config(const ocr_gguf* g, ocr_text_cfg* out);
/* VisionConfig::from_gguf (app/crates/ocr-wgpu/src/vision.rs:55-88) of an mmproj GGUF: clip.projector_type must be
 * "lightonocr", clip.use_silu true, the head dim 64; the clip.vision.* sizes, layer_norm_epsilon, image_mean /
 * image_std (3 values each); rope_theta 10000 (clip.cpp's constant). Host only. */
ocr_status ocr_gguf_vision_config(const ocr_gguf* g, ocr_vision_cfg* out);

/* ---- low-level ops on device buffers (the kernels behind the calls above; tests and the LM-head benchmark) ------ */
/* choose_pen.wgsl: the windowed repetition penalty in place on d_logits [n_vocab] over the distinct tokens of
 * d_hist[n_hist - window, n_hist) (device ids) — the device function the fused sampler applies */
ocr_status ocr_op_penalize(ocr_ctx* ctx, float* d_logits, int n_vocab, float rp, int window, const int32_t* d_hist,
                           int n_hist);
/* The device row layout of a q8_0 matrix [rows][cols] (cols a multiple of 32): row r at w + r * stride holds the int8
 * quants [cols], then the f16 scales [cols / 32], zero-padded to stride = ocr_q8_row_bytes(cols), a multiple of 16.
 * Any run of rows is one contiguous 16-B-aligned range (one bulk copy). Returns 0 for an invalid cols. */
int ocr_q8_row_bytes(int cols);
/* GGUF q8_0 blocks (34 B each, rows x cols/32 blocks, 2-B aligned) → the row layout at d_rows (16-B aligned,
 * rows x ocr_q8_row_bytes(cols) bytes). Same q and d bits. (Gpu::upload_tensor's q8_0 case, gpu.rs:1595-1647) */
ocr_status ocr_op_repack_q8_0(ocr_ctx* ctx, const void* d_blocks, int rows, int cols, uint8_t* d_rows);
/* y[b][r] (+)= sum_c W[r][c] * xn[b][c] for b < nb: xn = x, or RMSNorm(x) * norm_w when norm_w != NULL
 * (dmv.wgsl / dmv_norm / matvec_q8_0.wgsl). accumulate = 1 adds onto y. W in the row layout; x [nb][cols],
 * y [nb][rows]. */
ocr_status ocr_op_matvec_q8_0(ocr_ctx* ctx, const uint8_t* d_w, int rows, int cols, const float* d_x,
                              const float* d_norm_w, float eps, int nb, float* d_y, int accumulate);
/* the LM head fused with the sampler (dmv_norm → choose_pen → choose_max → choose_pick): logits = W . RMSNorm(x) *
 * norm_w over n_vocab rows (W in the row layout), the windowed penalty on the distinct tokens of
 * d_hist[len - window, len) (device, len = *d_len), argmax (first maximum) → *d_tok, d_hist[len] = token,
 * *d_len += 1. d_logits (nullable) receives the raw logits. One slot. */
ocr_status ocr_op_lm_head_sample(ocr_ctx* ctx, const uint8_t* d_w, int n_vocab, int dim, const float* d_x,
                                 const float* d_norm_w, float eps, float rp, int window, int32_t* d_hist,
                                 int32_t* d_len, int32_t* d_tok, float* d_logits);
/* ocr_op_lm_head_sample without any device allocation (no counterpart in the reference, which allocates through
 * wgpu). The CTAs' partials and the completion ticket live in a 16 KB static device array, one per device, instead of
 * the context's scratch: an LM head of more CTAs than it holds is refused with OCR_ERR_ARG. The first call on a device
 * looks the array up (cudaGetSymbolAddress) — make it before any stream capture. Two calls that may overlap in time
 * on one device (different contexts or streams) race on the array; calls on one context's stream are ordered. */
ocr_status ocr_op_lm_head_sample_noalloc(ocr_ctx* ctx, const uint8_t* d_w, int n_vocab, int dim, const float* d_x,
                                         const float* d_norm_w, float eps, float rp, int window, int32_t* d_hist,
                                         int32_t* d_len, int32_t* d_tok, float* d_logits);
/* decode attention of one token (qkv_post.wgsl + attn_decode.wgsl + attn_merge.wgsl): raw qkv [n_head + 2 n_kv][128]
 * f32 → per-head RMSNorm (q_norm / k_norm), RoPE NEOX at `pos` from the table rope [n_ctx][64][2], K/V rows `pos`
 * stored f16 into k_cache / v_cache ([n_kv][n_ctx][128] f16), then softmax(q k / sqrt(128)) v over keys 0…pos → out
 * [n_head][128] f32. */
ocr_status ocr_op_attention_decode(ocr_ctx* ctx, float* d_qkv, const float* d_q_norm, const float* d_k_norm,
                                   const float* d_rope, uint16_t* d_k_cache, uint16_t* d_v_cache, int n_head, int n_kv,
                                   int n_ctx, int pos, float eps, float* d_out);

/* Test hook for the device's bounded waits (the reference's Health rule, app/crates/ocr-wgpu/src/gpu.rs:901-970: a
 * device failure becomes an error, not a hang). Every kernel waits on mbarriers for at most a fixed number of polls,
 * then flags an error and skips the work. This runs one such wait that cannot complete, limited to `tries` polls of
 * about 1 µs: *waited_out = 1 when it gave up. The context's error flag stays set — the next ocr_ctx_sync returns
 * OCR_ERR_DEVICE and clears it; the context stays usable. Synchronous. */
ocr_status ocr_op_wait_probe(ocr_ctx* ctx, int tries, int* waited_out);
/* The vision encoder's attention alone (test entry point; the reference's attention_coop.wgsl, vision.rs:290-295):
 * softmax(q k^T * scale) v over keys 0 … n_keys - 1 for L query rows of n_head heads of 64 (q row r, head h at
 * d_q[r * q_stride + h * 64], f32), the keys and values f16 per head in the tiled layout the encoder's RoPE kernel
 * writes (n_pad a multiple of 64; head h's tiles at h * n_pad * 64 halves; per 64-key tile, K row r's 16-byte
 * piece p at r * 128 + ((p ^ (r % 8)) << 4) bytes, V transposed: dim row d's piece q of keys 8q … 8q + 7 at
 * d * 128 + ((q ^ (d % 8)) << 4); keys past n_keys zero) → d_out[r * out_stride + h * 64] f32. Queued on the
 * context's stream. */
ocr_status ocr_op_attention_full(ocr_ctx* ctx, const float* d_q, int q_stride, int L, int n_head,
                                 const uint16_t* d_k_tiled, const uint16_t* d_vt_tiled, int n_pad, int n_keys,
                                 float scale, float* d_out, int out_stride);

#ifdef __cplusplus
}
#endif
#endif
