// kernels.cuh — parameter blocks and launchers of the device kernels (sm_100a).
//
// Device layout of a q8_0 matrix [rows][cols] (cols % 32 == 0), repacked at load from GGUF's 34-byte blocks:
//   row r at w + r * stride:  int8 quants [cols] | f16 scales [cols / 32] | zero pad to a 16-B multiple
//   stride = round_up(cols + cols / 16, 16)
// value(r, c) = quants[c] * f32(scales[c / 32]) — the same q and d bits as the GGUF blocks. Any run of rows is one
// contiguous, 16-B aligned, 16-B multiple byte range: one bulk-async copy (cp.async.bulk) moves a stage of rows.
#pragma once

#include "common.cuh"

namespace ocr {

__host__ __device__ constexpr int q8_stride(int cols) { return (cols + cols / 16 + 15) / 16 * 16; }

struct QMat {
    const uint8_t* w = nullptr;
    int rows = 0, cols = 0, stride = 0;
};

// ---- weights: repack / synthetic generation (k_weights.cu) ---------------------------------------------------------
// GGUF blocks [rows][cols/32] x 34 B → the row layout at destination row r * row_mul + row_add
void launch_repack_q8_0(cudaStream_t st, const uint8_t* blocks, int rows, int cols, uint8_t* w, int row_mul,
                        int row_add);
// the synthetic generator (bit-identical to the oracle's orc_synth_q8_0 / orc_fill_norm); valid > 0: only columns
// below it hold values (sigma * gauss(r * valid + col)), the rest zeros (orc_synth_q8_0_padded)
void launch_synth_q8_0(cudaStream_t st, uint64_t seed, float sigma, int rows, int cols, uint8_t* w, int row_mul,
                       int row_add, int valid = 0);
void launch_synth_norm(cudaStream_t st, uint64_t seed, int n, float* out);
// back to GGUF blocks (ocr_model_tensor_gguf): source rows r * row_mul + row_add
void launch_unpack_q8_0(cudaStream_t st, const uint8_t* w, int rows, int cols, int row_mul, int row_add,
                        uint8_t* blocks);
// W_o (rows x cols, row layout) cut into `parts` column slices of cols/parts: slice j, row r = the row's quants of
// those columns | their f16 scales | zero pad to q8_stride(cols / parts) (the decode attention's fused o-projection
// reads the slice of its kv head's q heads as one contiguous run)
void launch_slice_o(cudaStream_t st, const uint8_t* w, int rows, int cols, int parts, uint8_t* out);

// ---- the token choice's arguments (shared by the LM head, the standalone choice and the penalty) ------------------
struct LmArgs {
    int sample = 0;  // 0: logits only
    float rp = 1.0f;
    int window = 1;
    int use_fp = 0;
    float fp = 0.0f;
    int32_t* hist = nullptr;  // [B][hist_cap]
    int hist_cap = 0;
    int32_t* len = nullptr;   // [B]
    int32_t* tok = nullptr;   // [B]
    int32_t* pos = nullptr;   // [B] advanced by one per choice when advance_pos
    int advance_pos = 0;
    uint32_t* counts = nullptr;  // [B][n_vocab] (use_fp)
    float* fpen = nullptr;       // [B][n_vocab]
    const int32_t* active = nullptr;
    float* part = nullptr;       // scratch: [B][grid][2] + [B] NaN-at-token-0 flags
    uint32_t* done = nullptr;    // scratch counters (self-resetting)
    int nb = 1;                  // slots in the partials' layout
    // continuous batching (ocr_read_pages): each choice counts down the slot's budget, and the slot goes idle (its
    // active flag cleared, read by the next step's kernels) when the budget is spent; null = no budgets
    int32_t* remaining = nullptr;  // [B]
    int32_t* active_w = nullptr;   // [B] the active flags, writable
    int* err = nullptr;
};

// ---- the streamed matvec family (k_matvec.cu) -----------------------------------------------------------------------
enum MvMode : int { MV_STORE = 0, MV_ADD = 1, MV_SWIGLU = 2, MV_LMHEAD = 3 };

// What the next kernel of the step will read, pulled into L2 by this kernel's CTAs as they start (each CTA its share):
// a weight matrix, and/or a layer's KV rows [0, pos[b]) of every active (slot, kv head). Those bytes then stream
// from HBM while this kernel and the dependency chain run, and the next kernel's copies hit L2.
struct L2Next {
    const uint8_t* w = nullptr;  // 16-B aligned
    size_t w_bytes = 0;          // multiple of 16
    const uint8_t* w2 = nullptr;  // a second matrix (the fused FFN reads two)
    size_t w2_bytes = 0;
    const __half* kc = nullptr;  // [B][n_kv][n_ctx][128]
    const __half* vc = nullptr;
    const int32_t* pos = nullptr;
    const int32_t* active = nullptr;
    int n_kv = 0, n_ctx = 0, nb = 0;
};
// issues CTA `part`'s share of `p` (one thread calls it): 1/parts of the matrix, and 1/parts of each KV run (whole
// 256-B rows), in prefetches of at most 64 KB
__device__ __forceinline__ void l2_next(const L2Next& p, int part, int parts) {
    constexpr uint32_t CH = 64u << 10;
    auto mat = [&](const uint8_t* w, size_t bytes) {
        if (!w || !bytes) return;
        const size_t share = ((bytes + parts - 1) / parts + 15) / 16 * 16;
        const size_t lo = (size_t)part * share, hi = min(bytes, lo + share);
        for (size_t o = lo; o < hi; o += CH) prefetch_l2(w + o, (uint32_t)min((size_t)CH, hi - o));
    };
    mat(p.w, p.w_bytes);
    mat(p.w2, p.w2_bytes);
    if (p.kc) {
        for (int b = 0; b < p.nb; b++) {
            if (p.active && !p.active[b]) continue;
            const int rows = min(max(p.pos[b], 0), p.n_ctx);
            const int r0 = (int)((long)rows * part / parts), r1 = (int)((long)rows * (part + 1) / parts);
            if (r1 <= r0) continue;
            for (int j = 0; j < p.n_kv; j++) {
                const long base = (((long)b * p.n_kv + j) * p.n_ctx + r0) * 128;
                const uint32_t bytes = (uint32_t)(r1 - r0) * 256;
                for (uint32_t o = 0; o < bytes; o += CH) {
                    const uint32_t n = min(CH, bytes - o);
                    prefetch_l2(reinterpret_cast<const uint8_t*>(p.kc + base) + o, n);
                    prefetch_l2(reinterpret_cast<const uint8_t*>(p.vc + base) + o, n);
                }
            }
        }
    }
}

struct MvArgs {
    QMat w;
    const float* x = nullptr;  // [B][x_stride] input rows
    int x_stride = 0;
    const float* nw = nullptr;  // RMSNorm weights (null = no norm)
    float eps = 1e-6f;
    // layer-0 embedding: x = token_embd[tok[b]] (dequantized), written to x_out by the grid's first CTA
    const int32_t* tok = nullptr;
    QMat emb;
    float* x_out = nullptr;
    // x = x + (xadd[b][0] + … + xadd[b][n_add - 1]) ([B][n_add][cols] partial products, n_add <= MAX_ADD,
    // cols <= 4 x the consumer threads), also written to x_out by the grid's first CTA
    const float* xadd = nullptr;
    int n_add = 0;
    float* y = nullptr;  // [B][y_stride] (LM head: raw logits [B][n_vocab], may be null)
    int y_stride = 0;
    int mode = MV_STORE;
    int nb = 1;  // slots
    const int32_t* active = nullptr;  // [B] (null = all); an idle slot's rows are not written
    LmArgs lm;   // MV_LMHEAD: the choice
    L2Next next;
    int* err = nullptr;
    TlSlot* tl = nullptr;  // the in-chain timeline slot of this launch (null: not recorded)
};
constexpr int MAX_ADD = 8;
void launch_matvec(cudaStream_t st, const MvArgs& a, int num_sms, bool pdl);
// grid of the LM head (the partials' layout) for n_vocab rows
int lm_head_grid(int num_sms, int n_vocab, int dim);

// the choice alone over logits on the device (choice 0 from the prompt's logits; ocr_sample_logits)
// slots [slot_base, slot_base + n_slots) of logits [B][logits_stride]; a.nb = B (the partials' layout)
void launch_sample(cudaStream_t st, const float* logits, int logits_stride, int n_vocab, const LmArgs& a,
                   int num_sms, int slot_base, int n_slots);
int sample_grid(int num_sms);
// the windowed penalty alone, in place (a.sample = 1, a.len → n_hist, a.hist, a.rp, a.window)
void launch_penalize(cudaStream_t st, float* logits, int n_vocab, const LmArgs& a, int num_sms);

// ---- attention (k_attn.cu) -------------------------------------------------------------------------------------------
struct AttnArgs {
    float* qkv = nullptr;  // [B][(n_head + 2 n_kv) * 128] raw projections
    int qkv_stride = 0;
    const float* q_norm = nullptr;
    const float* k_norm = nullptr;
    const float* rope = nullptr;  // [n_ctx][64][2]
    __half* kc = nullptr;         // [B][n_kv][n_ctx][128]
    __half* vc = nullptr;
    const int32_t* pos = nullptr;  // [B] the token's position (device)
    const int32_t* active = nullptr;
    int n_head = 16, n_kv = 8, n_ctx = 0, splits = 16;  // splits: CTAs per cluster (4, 8 or 16)
    float eps = 1e-6f, scale = 0.0f;
    float* out = nullptr;       // [B][out_stride] the attention output (when wo is null)
    int out_stride = 0;
    // the fused o-projection (when wo is set): the cluster of kv head j multiplies its q heads' merged output by
    // W_o's slice j (launch_slice_o: [n_kv][dim rows] of q8_stride(G * 128) bytes) → opart[b][j][dim], the
    // per-head partial products that the next kernel sums in a fixed order
    const uint8_t* wo = nullptr;
    int dim = 0;
    float* opart = nullptr;
    // the fused qkv projection (when wqkv.w is set; qkv is then unused): the slot's residual row is staged from `in`
    // (as the qkv matvec would) and the cluster of kv head j computes its q heads' and its k / v rows of wqkv, each
    // CTA (G + 2)·128 / CL consecutive ones
    MvArgs in;
    QMat wqkv;
    int nb = 1;
    L2Next next;
    int* err = nullptr;
    TlSlot* tl = nullptr;  // the in-chain timeline slot of this launch (null: not recorded)
};
void launch_attention_decode(cudaStream_t st, const AttnArgs& a, bool pdl);
// the cluster size the launch of `a` will use (its `splits`, or fewer when those clusters cannot be resident)
int attention_cluster(const AttnArgs& a);
// true when the qkv projection can be fused for a group of g q heads in clusters of cl CTAs at this model width
bool attention_fuses_qkv(int g, int cl, int dim);

// ---- the fused FFN (k_ffn.cu) ----------------------------------------------------------------------------------------
// One slot: x + (o-partials) → residual, RMSNorm → gate|up → SwiGLU → down, in FFN_NCLU thread-block clusters of
// FFN_CL CTAs. Cluster c owns h[c·n_ff/FFN_NCLU …) — its gate|up rows are one contiguous run of the interleaved
// matrix — and multiplies it by its column slice of W_down (launch_slice_o with FFN_NCLU parts), leaving FFN_NCLU
// partial products of the down projection that the next kernel's staging sums in a fixed order.
constexpr int FFN_CL = 16;
constexpr int FFN_NCLU = 8;
struct FfnArgs {
    MvArgs in;  // the staging: in.x, in.xadd / n_add (o-partials), in.x_out (the new residual), in.nw, in.eps;
                // in.w.cols = dim
    QMat gu;    // gate|up, rows interleaved [2 n_ff][dim]
    const uint8_t* wd = nullptr;  // W_down cut by h slice: [FFN_NCLU][dim][q8_stride(n_ff / FFN_NCLU)]
    int n_ff = 0;
    float* dpart = nullptr;  // [FFN_NCLU][dim]
    L2Next next;
    int* err = nullptr;
    TlSlot* tl = nullptr;  // the in-chain timeline slot of this launch (null: not recorded)
};
// the dynamic shared memory the fused FFN needs for this shape, or 0 when the shape does not fit it
int ffn_smem(int dim, int n_ff);
// true when the fused FFN's clusters can be resident on this device (asks the occupancy API once per shape)
bool ffn_usable(int dim, int n_ff);
void launch_ffn(cudaStream_t st, const FfnArgs& a, bool pdl);
int attention_splits(int num_sms, int nb, int n_kv, int n_ctx);

// ---- the batched decode contraction on the tensor cores (k_bgemm.cu) -----------------------------------------------
// For batches of slots the matvecs become skinny GEMMs Y[slot][row] = sum_k W[row][k] x[slot][k], run by tcgen05.mma
// (kind::f16, f32 accumulators in tensor memory) on exact f16 splits of both operands: each weight q * d (exact in
// f32) is the sum of two f16 values w_hi + w_lo, each activation x = x_hi + x_lo, and the MMAs accumulate
// w_hi x_hi + w_hi x_lo + w_lo x_hi — the f32 matvec's result to within f32 rounding (the dropped w_lo x_lo term is
// below 2^-22 of the product).
//
// The activation operand ("x16") of a group of BG_SLOTS slots over K columns is K/128 chunks of BG_CHUNK_BYTES:
// rows n < 32 hold f16(x[slot n]) (hi), rows 32 + n hold f16(x - hi) (lo). A chunk is two 8 KB halves of 64 columns,
// each in tcgen05's K-major 128-byte-swizzle layout: row n's 64 halves are 128 bytes at n * 128, their 16-byte
// pieces (8 columns each) stored at piece ((k % 64) / 8) ^ (n % 8) — so one bulk copy of a chunk is an MMA operand as
// it lands, and the tensor cores read it without bank conflicts.
constexpr int BG_SLOTS = 32;
constexpr uint32_t BG_CHUNK_BYTES = 16384;
__host__ __device__ constexpr size_t x16_offset(int n, int k) {
    return (size_t)(k >> 7) * BG_CHUNK_BYTES + (size_t)((k >> 6) & 1) * 8192 + (size_t)n * 128 +
           (size_t)(((((k & 63) >> 3) ^ (n & 7))) << 4) + (size_t)((k & 7) << 1);
}
__host__ __device__ constexpr size_t x16_group_bytes(int K) { return (size_t)(K / 128) * BG_CHUNK_BYTES; }

// The tile-major copy of a matrix that the contraction streams (derived on the device at load): per 128-row tile t
// and 128-column chunk c, block t * (cols / 128) + c of BG_TILE_BYTES — the rows' 128 quant bytes (row r at r * 128,
// its 16-byte piece p at ((p ^ (r % 8)) * 16): the swizzle of the operand reads) and then the rows' 4 block scales
// (r * 8, f16) — so a stage of the stream is one contiguous 17 KB copy. Rows past the matrix are zero.
constexpr uint32_t BG_TILE_BYTES = 17408;
struct BgMaps {
    const uint8_t* tiles = nullptr;
};
size_t bgemm_tiled_bytes(int rows, int cols);
void launch_tile_q8_0(cudaStream_t st, const QMat& w, uint8_t* out);
struct BgArgs {
    QMat w;
    const uint8_t* x16 = nullptr;  // [groups][K/128] chunks (the slots' activations, hi / lo)
    int mode = MV_STORE;           // MV_STORE, MV_ADD, MV_SWIGLU (rows interleaved gate, up), MV_LMHEAD
    float* y = nullptr;            // [B][y_stride] (SwiGLU: [B][rows/2]; LM head: raw logits [B][rows], may be null)
    int y_stride = 0;
    uint8_t* y16 = nullptr;        // SwiGLU: the result also as the next contraction's operand (x16 over rows/2)
    int nb = 1;                    // slots (blockIdx.y takes groups of BG_SLOTS)
    const int32_t* active = nullptr;
    LmArgs lm;                     // MV_LMHEAD: the choice (lm.nb = nb, partials [nb][grid])
    // split-K: each 128-row tile's K chunks shared by ksplit CTAs, whose f32 partials [groups][tiles][ksplit][32][128]
    // the tile's last CTA sums in split order (tickets [groups][tiles], zero between launches); 1 = no split
    int ksplit = 1;
    float* part = nullptr;
    uint32_t* tickets = nullptr;
    // The RMS-normalised operand built in the kernel (instead of copied from x16): the slots' residual rows xn [B][K],
    // the norm weights nw [K], and the sums of squares of each row over K/128 column tiles, ssq_in [K/128][B] (written
    // by the contraction that produced the residual). Then every CTA takes one work item whose K chunks fit its stages
    // (bgemm_norm_in_ok).
    const float* xn = nullptr;
    const float* nw = nullptr;
    const float* ssq_in = nullptr;
    float eps = 1e-6f;
    // MV_ADD: the new residual rows' sums of squares per 128-row tile, ssq_out [rows/128][B] (for the next norm)
    float* ssq_out = nullptr;
    // thousands of rows (unsplit, plain operand): three groups of 32 per CTA, their operands merged into MMAs of N = 192
    int wide = 0;
    int* err = nullptr;
    TlSlot* tl = nullptr;  // the in-chain timeline slot of this launch (null: not recorded)
};
// true when the tensor-core contraction takes this shape (cols a multiple of 256, at most 4096)
bool bgemm_shape_ok(int rows, int cols);
// true when a launch of this shape can build its normalised operand in the kernel (BgArgs::xn): one work item per
// CTA, each item's K chunks at most the copy stages
bool bgemm_norm_in_ok(int num_sms, int rows, int cols, int ksplit);
// CTAs of a launch: one per work item (a 128-row tile's split), at most one per SM (a persistent CTA takes items
// blockIdx.x + k * grid)
int bgemm_grid(int num_sms, int rows, int ksplit = 1);
// the K split for a matrix: enough items to give every SM one (at most one per 128-column chunk); 1 for the LM head
int bgemm_ksplit(int num_sms, int rows, int cols);
// scratch of a split launch: partial floats and tickets per slot group
size_t bgemm_part_floats(int rows, int ksplit);
int bgemm_tickets(int rows);
void launch_bgemm(cudaStream_t st, const BgArgs& a, const BgMaps& m, int num_sms, bool pdl);

// The activations of a batch as the contraction's operand: per slot x (+ the partial products in order, or the token's
// embedding row), written back to x_out when set, RMS-normalised by nw when set, split hi / lo into x16. Slots past
// nb or idle get zeros.
struct PrepArgs {
    const float* x = nullptr;  // [B][x_stride]
    int x_stride = 0;
    const float* xadd = nullptr;  // [B][n_add][K] (summed in order, then added to x)
    int n_add = 0;
    const int32_t* tok = nullptr;  // layer 0: x = token_embd[tok[b]] dequantized
    QMat emb;
    float* x_out = nullptr;  // may alias x (each slot's row is read, then written, by one CTA)
    const float* nw = nullptr;
    float eps = 1e-6f;
    int K = 0, nb = 1;
    const int32_t* active = nullptr;
    uint8_t* x16 = nullptr;
    int* err = nullptr;
    TlSlot* tl = nullptr;  // the in-chain timeline slot of this launch (null: not recorded)
};
void launch_xprep(cudaStream_t st, const PrepArgs& a, bool pdl);

// ---- decode attention for batches (k_attn_batch.cu) -------------------------------------------------------------------
// One CTA (or `split` CTAs) per (slot, kv head) streaming its keys; the q/k norm + RoPE + K/V store of the new token
// as in AttnArgs; the G heads' merged rows written as the o-projection's operand (x16 over n_head x 128 columns)
// and, when out is set, as f32 rows.
constexpr int AB_MAX_SPLIT = 16;
struct AttnBatchArgs {
    const float* qkv = nullptr;  // [B][qkv_stride] raw projections
    int qkv_stride = 0;
    const float* q_norm = nullptr;
    const float* k_norm = nullptr;
    const float* rope = nullptr;  // [n_ctx][64][2]
    __half* kc = nullptr;         // [B][n_kv][n_ctx][128]
    __half* vc = nullptr;
    const int32_t* pos = nullptr;
    const int32_t* active = nullptr;
    int n_head = 16, n_kv = 8, n_ctx = 0, nb = 1;
    float eps = 1e-6f, scale = 0.0f;
    float* out = nullptr;  // [B][out_stride] (nullable)
    int out_stride = 0;
    uint8_t* x16 = nullptr;  // [groups] the o-projection's operand (nullable)
    float* part = nullptr;   // split > 1: [B * n_kv][split][G][132]
    uint32_t* done = nullptr;  // split > 1: [B * n_kv] tickets (zero between launches)
    int* err = nullptr;
    TlSlot* tl = nullptr;  // the in-chain timeline slot of this launch (null: not recorded)
};
// CTAs per (slot, kv head) for a batch: enough to fill two CTAs per SM, at most AB_MAX_SPLIT
int attn_batch_split(int num_sms, int nb, int n_kv);
void launch_attention_batch(cudaStream_t st, const AttnBatchArgs& a, int split, bool pdl);

// ---- the bounded-wait test hook (k_probe.cu) ----
// one mbarrier wait that cannot complete, limited to `tries` polls of ~1 µs: *waited_out = 1 and DEV_TIMEOUT flagged
void launch_wait_probe(cudaStream_t st, int* err, uint32_t tries, int* waited_out);

// ---- prefill (k_prefill.cu) -------------------------------------------------------------------------------------------
void launch_embed_rows(cudaStream_t st, const int32_t* ids, int n, QMat emb, float* x);
void launch_rmsnorm_rows(cudaStream_t st, const float* x, const float* w, float* y, int rows, int dim, float eps);
// Y[L][N] (+)= X[L][K] . W^T; swiglu: W rows interleaved (gate, up) → Y[L][N/2] = silu(gate) * up
void launch_gemm_q8_0(cudaStream_t st, const float* x, int L, QMat w, float* y, int accumulate, int swiglu);
// per-row q/k head norm + RoPE (q in place), K/V rows pos0 + r stored f16
void launch_qk_norm_rope_store(cudaStream_t st, float* qkv, int L, int n_head, int n_kv, const float* q_norm,
                               const float* k_norm, const float* rope, int pos0, float eps, __half* kc, __half* vc,
                               int n_ctx);
// causal attention of L queries (positions pos0…) over the f16 cache rows 0…pos0+r → out [L][n_head*128]
void launch_attention_prefill(cudaStream_t st, const float* qkv, int L, int n_head, int n_kv, const __half* kc,
                              const __half* vc, int n_ctx, int pos0, float scale, float* out);
// the same causal attention on the tensor cores (k_attn_prefill_tc.cu): 128-query tiles, f16 hi / lo splits of Q and
// of the probabilities, two softmax passes; `err` takes a bounded wait's timeout
void launch_attention_prefill_tc(cudaStream_t st, const float* qkv, int L, int n_head, int n_kv, const __half* kc,
                                 const __half* vc, int n_ctx, int pos0, float scale, float* out, int* err);
// the general form of that kernel: query row r, head h at q[r * q_stride + h * D]; key / value row j of kv head
// h / group at k[(h / group) * kv_head_stride + j * D] (f16); causal (query r at position pos0 + r sees keys ≤ its
// position) or full (every query sees keys 0 … n_keys - 1); the output row r, head h as f32 at
// out[r * out_stride + h * D] and / or split f16 hi / lo into out16 (x16 groups of 32 rows over out16_K columns)
struct TcAttnArgs {
    const float* q = nullptr;
    int q_stride = 0;
    int L = 0, n_head = 0, group = 1;
    const __half* k = nullptr;
    const __half* v = nullptr;
    size_t kv_head_stride = 0;
    int pos0 = 0, n_keys = 0;
    float scale = 1.0f;
    float* out = nullptr;
    int out_stride = 0;
    uint8_t* out16 = nullptr;
    int out16_K = 0;
    int* err = nullptr;
};
// the full attention of head dim 64 (the vision encoder) over k / v in the tiled layouts launch_rope2d_heads writes
// (kv_head_stride = n_pad * 64): each 64-key tile of K and of V^T one bulk copy, two CTAs per SM
void launch_attention_full_tc(cudaStream_t st, const TcAttnArgs& a);

// ---- the vision encoder's own kernels (k_vision.cu) --------------------------------------------------------------------
// The placement of a (not yet baked) image inside the baked canvas: the image's pixel (x, y) sits at (x + left,
// y + top) of a canvas width x height; every other canvas pixel is white (the bake's pad).
struct Placement {
    int img_w = 0, img_h = 0, left = 0, top = 0, width = 0, height = 0;
};
// rgb bytes [img_h][img_w][3] → the patch embedding's operand (x16 groups of 32 patches over K columns): patch
// t = ty * px + tx, column c * p² + ky * p + kx = lut[c][pixel(tx * p + kx, ty * p + ky)[c]], columns past 3 p² zero
void launch_patchify(cudaStream_t st, const uint8_t* rgb, const Placement& pl, int patch, const float* lut, int K,
                     uint8_t* x16);
// the q and k parts of qkv rows [n][3 * dim] rotated by the 2D RoPE (in place for q); k and v written f16 per head
// in tiles of 64 keys already in the attention's operand layouts (K: key rows, V: transposed, both K-major with the
// 128-byte swizzle; d_head 64; keys past n zero): head h's tiles at kh + h * n_pad * 64, each 64 * 64 halves
void launch_rope2d_heads(cudaStream_t st, float* qkv, int n, int n_head, int d_head, int px, const float* cs,
                         int max_pos, __half* kh, __half* vh, int n_pad);
// the projector's input: x [n][dim] RMS-normalised by w, 2x2-unfolded (merged token o = oy * px/2 + ox gets column
// c * 4 + ky * 2 + kx = xn[(2 oy + ky) * px + 2 ox + kx][c]) into the merger's operand (x16 over 4 dim columns)
void launch_unfold_prep(cudaStream_t st, const float* x, const float* w, float eps, int px, int py, int dim,
                        uint8_t* x16);
// rows [n][K] → GELU (tanh form) → x16 operand (act = 1), or the plain split (act = 0)
void launch_act_prep(cudaStream_t st, const float* y, int n, int K, int act, uint8_t* x16);
// the bake's Lanczos-3 resize, rgb [h0][w0][3] → out [h][w][3] through tmp [h][w0][3] f32: per output row y the taps
// vleft[y] … + vcnt[y] - 1 with weights vw[y * vmax …], per output column x likewise (h…)
void launch_resize(cudaStream_t st, const uint8_t* rgb, int w0, int h0, int w, int h, const int* vleft,
                   const int* vcnt, const float* vw, int vmax, const int* hleft, const int* hcnt, const float* hw,
                   int hmax, float* tmp, uint8_t* out);
// src [sh][sw][3] placed at (left, top) of a white canvas [fh][fw][3]
void launch_bake_place(cudaStream_t st, const uint8_t* src, int sw, int sh, int left, int top, int fw, int fh,
                       uint8_t* out);

}  // namespace ocr
