// runtime.cu — the host runtime behind ocr_cuda.h: context (device, stream, byte ledger), model (GGUF streaming
// upload + device repack, or the seeded synthetic generator), session (KV cache, decode scratch, device-side sampler
// state), prefill, step, and the run-ahead decode loop replaying one captured CUDA graph per token.
//
// Reference map (b-straub/historic-htr-ocr): Gpu (app/crates/ocr-wgpu/src/gpu.rs:972-1324), TextModel::load /
// session / prefill / step / decode_gpu (text.rs:332-625), Choice (text.rs:167-232), TextConfig::from_gguf
// (text.rs:51-82), rope_table (text.rs:132-142).
#include <cuda_runtime.h>
#include <math.h>
#include <string.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "ctx.h"
#include "gguf.h"
#include "kernels.cuh"

namespace ocr {

thread_local std::string g_err;
void set_error(const std::string& m) { g_err = m; }
ocr_status fail(ocr_status c, const std::string& m) {
    g_err = m;
    return c;
}
ocr_status cuda_fail(cudaError_t e, const char* what) {
    g_err = std::string(what) + ": " + cudaGetErrorString(e);
    return OCR_ERR_CUDA;
}

}  // namespace ocr

using namespace ocr;

constexpr size_t STAGE_BYTES = 64u << 20;

namespace ocr {

// device memory, zeroed before it is returned. cudaMemset on device memory is asynchronous and runs on the legacy
// stream, which does not order against the contexts' non-blocking streams: without the wait, the zeroing of a buffer
// grown between two kernels of a context could land after (on top of) the later kernel's writes.
cudaError_t dalloc(void** p, size_t n, uint64_t* ctr) {
    cudaError_t e = cudaMalloc(p, n ? n : 16);
    if (e != cudaSuccess) return e;
    e = cudaMemset(*p, 0, n ? n : 16);
    if (e == cudaSuccess) e = cudaStreamSynchronize(nullptr);
    if (ctr) *ctr += n;
    return e;
}

void dfree(void* p, size_t n, uint64_t* ctr) {
    if (p) cudaFree(p);
    if (ctr) *ctr -= n;
}

ocr_status ensure_op_scratch(ocr_ctx* ctx, size_t n) {
    if (ctx->op_scratch_bytes >= n) return OCR_OK;
    if (ctx->op_scratch) {
        OCR_CUDA(cudaStreamSynchronize(ctx->stream));
        dfree(ctx->op_scratch, ctx->op_scratch_bytes, &ctx->mem_work);
        ctx->op_scratch = nullptr;
        ctx->op_scratch_bytes = 0;
    }
    OCR_CUDA(dalloc(&ctx->op_scratch, n, &ctx->mem_work));
    ctx->op_scratch_bytes = n;
    return OCR_OK;
}

ocr_status check_device_error(ocr_ctx* ctx) {
    int err = 0;
    OCR_CUDA(cudaMemcpy(&err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (err != DEV_OK) {
        OCR_CUDA(cudaMemsetAsync(ctx->d_err, 0, sizeof(int), ctx->stream));  // (ordered before later kernels)
        return fail(OCR_ERR_DEVICE, err == DEV_BAD_POS     ? "a kernel saw a position outside the KV cache"
                                    : err == DEV_TIMEOUT ? "a kernel's bounded wait ran out (its work was skipped)"
                                                         : "a kernel saw an index outside its buffer");
    }
    return OCR_OK;
}

}  // namespace ocr

// ---------------------------------------------------------------------------------------------------------------------
// model
// ---------------------------------------------------------------------------------------------------------------------
struct LayerW {
    QMat qkv, o, gu, down;  // qkv rows [q | k | v]; gu rows interleaved (gate 0, up 0, gate 1, …)
    float *attn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr, *ffn_norm = nullptr;
    uint8_t* o_s = nullptr;  // W_o cut per kv head (launch_slice_o), derived on the device after the load
    uint8_t* d_s = nullptr;  // W_down cut into FFN_NCLU h slices (the fused FFN), when the shape fits it
    BgMaps bq_qkv, bq_o, bq_gu, bq_down;  // the tensor-core contraction's views of the matrices (model tc)
};

struct ocr_model {
    int refs = 1;  // the caller's handle + one per live session
    ocr_ctx* ctx = nullptr;
    ocr_text_cfg cfg{};
    void* mem = nullptr;
    size_t mem_bytes = 0;
    std::vector<LayerW> layers;
    QMat tok;
    float* out_norm = nullptr;
    bool tc = false;  // the batched contractions can run on the tensor cores (shapes fit, tensor maps made)
    BgMaps bq_tok;
};

namespace {

struct Planner {
    size_t off = 0;
    size_t take(size_t n) {
        const size_t o = off;
        off = (off + n + 255) / 256 * 256;
        return o;
    }
};

// offsets of every tensor in the model's one allocation
struct Layout {
    struct MatOff {
        size_t off;
        int rows, cols;
    };
    struct LayerOff {
        MatOff qkv, o, gu, down;
        size_t attn_norm, q_norm, k_norm, ffn_norm, o_s, d_s;
        size_t t_qkv = 0, t_o = 0, t_gu = 0, t_down = 0;  // the tile-major copies (tensor-core contractions)
    };
    std::vector<LayerOff> layers;
    MatOff tok;
    size_t out_norm, total;
    bool tc = false;
    size_t t_tok = 0;
};

// the batched contractions can run on the tensor cores: every matrix's shape fits them (OCR_TC=0 turns them off)
bool tc_shapes(const ocr_text_cfg& c) {
    const char* env = getenv("OCR_TC");
    if (env && env[0] == '0') return false;
    const int qd = c.n_head * c.d_head;
    return bgemm_shape_ok(c.n_vocab, c.dim) && bgemm_shape_ok(2 * c.n_ff, c.dim) && bgemm_shape_ok(c.dim, c.n_ff) &&
           bgemm_shape_ok(qd + 2 * c.n_kv * c.d_head, c.dim) && bgemm_shape_ok(c.dim, qd);
}

Layout plan(const ocr_text_cfg& c) {
    Planner p;
    Layout L;
    const int qd = c.n_head * c.d_head, kvd = c.n_kv * c.d_head;
    auto mat = [&](int rows, int cols) {
        Layout::MatOff m;
        m.rows = rows;
        m.cols = cols;
        m.off = p.take((size_t)rows * q8_stride(cols));
        return m;
    };
    for (int l = 0; l < c.n_layer; l++) {
        Layout::LayerOff lo;
        lo.qkv = mat(qd + 2 * kvd, c.dim);
        lo.o = mat(c.dim, qd);
        lo.gu = mat(2 * c.n_ff, c.dim);
        lo.down = mat(c.dim, c.n_ff);
        lo.attn_norm = p.take((size_t)c.dim * 4);
        lo.q_norm = p.take((size_t)c.d_head * 4);
        lo.k_norm = p.take((size_t)c.d_head * 4);
        lo.ffn_norm = p.take((size_t)c.dim * 4);
        lo.o_s = p.take((size_t)c.n_kv * c.dim * q8_stride(qd / c.n_kv));
        lo.d_s = ffn_smem(c.dim, c.n_ff) ? p.take((size_t)FFN_NCLU * c.dim * q8_stride(c.n_ff / FFN_NCLU)) : 0;
        L.layers.push_back(lo);
    }
    L.tok = mat(c.n_vocab, c.dim);
    L.out_norm = p.take((size_t)c.dim * 4);
    L.tc = tc_shapes(c);
    if (L.tc) {
        for (auto& lo : L.layers) {
            lo.t_qkv = p.take(bgemm_tiled_bytes(lo.qkv.rows, lo.qkv.cols));
            lo.t_o = p.take(bgemm_tiled_bytes(lo.o.rows, lo.o.cols));
            lo.t_gu = p.take(bgemm_tiled_bytes(lo.gu.rows, lo.gu.cols));
            lo.t_down = p.take(bgemm_tiled_bytes(lo.down.rows, lo.down.cols));
        }
        L.t_tok = p.take(bgemm_tiled_bytes(L.tok.rows, L.tok.cols));
    }
    L.total = p.off;
    return L;
}

QMat qmat(void* base, const Layout::MatOff& m) {
    QMat q;
    q.w = (const uint8_t*)base + m.off;
    q.rows = m.rows;
    q.cols = m.cols;
    q.stride = q8_stride(m.cols);
    return q;
}

ocr_status check_cfg(const ocr_text_cfg& c) {
    if (c.n_layer < 1 || c.dim < 32 || c.n_head < 1 || c.n_kv < 1 || c.n_ff < 32 || c.n_vocab < 1)
        return fail(OCR_ERR_ARG, "text config: every dimension must be positive");
    if (c.d_head != 128) return fail(OCR_ERR_FORMAT, "head dim " + std::to_string(c.d_head) + ": the attention kernels are written for 128");
    if (c.n_head % c.n_kv != 0) return fail(OCR_ERR_FORMAT, std::to_string(c.n_head) + " q heads on " + std::to_string(c.n_kv) + " kv heads");
    const int g = c.n_head / c.n_kv;
    if (g != 1 && g != 2 && g != 4 && g != 8) return fail(OCR_ERR_FORMAT, "GQA groups of 1, 2, 4 or 8 query heads only");
    if (c.dim % 32 || c.n_ff % 32) return fail(OCR_ERR_FORMAT, "dims " + std::to_string(c.dim) + " / " + std::to_string(c.n_ff) + ": q8_0 rows must be whole blocks");
    if (c.n_ctx_train < 1) return fail(OCR_ERR_ARG, "n_ctx_train must be positive");
    return OCR_OK;
}

// the layouts derived from the loaded weights (W_o's per-kv-head slices; the tile-major copies)
void derive_weights(ocr_model* m, cudaStream_t st) {
    const auto& c = m->cfg;
    for (auto& L : m->layers) {
        launch_slice_o(st, L.o.w, L.o.rows, L.o.cols, c.n_kv, L.o_s);
        if (L.d_s) launch_slice_o(st, L.down.w, L.down.rows, L.down.cols, FFN_NCLU, L.d_s);
        if (m->tc) {
            launch_tile_q8_0(st, L.qkv, const_cast<uint8_t*>(L.bq_qkv.tiles));
            launch_tile_q8_0(st, L.o, const_cast<uint8_t*>(L.bq_o.tiles));
            launch_tile_q8_0(st, L.gu, const_cast<uint8_t*>(L.bq_gu.tiles));
            launch_tile_q8_0(st, L.down, const_cast<uint8_t*>(L.bq_down.tiles));
        }
    }
    if (m->tc) launch_tile_q8_0(st, m->tok, const_cast<uint8_t*>(m->bq_tok.tiles));
}

ocr_status model_alloc(ocr_ctx* ctx, const ocr_text_cfg& c, ocr_model** out) {
    OCR_TRY(check_cfg(c));
    OCR_CUDA(cudaSetDevice(ctx->device));
    Layout L = plan(c);
    auto* m = new ocr_model;
    m->ctx = ctx;
    m->cfg = c;
    cudaError_t e = dalloc(&m->mem, L.total, &ctx->mem_weights);
    if (e != cudaSuccess) {
        delete m;
        return cuda_fail(e, "cudaMalloc(weights)");
    }
    ctx->refs++;
    m->mem_bytes = L.total;
    for (const auto& lo : L.layers) {
        LayerW w;
        w.qkv = qmat(m->mem, lo.qkv);
        w.o = qmat(m->mem, lo.o);
        w.gu = qmat(m->mem, lo.gu);
        w.down = qmat(m->mem, lo.down);
        w.attn_norm = (float*)((char*)m->mem + lo.attn_norm);
        w.q_norm = (float*)((char*)m->mem + lo.q_norm);
        w.k_norm = (float*)((char*)m->mem + lo.k_norm);
        w.ffn_norm = (float*)((char*)m->mem + lo.ffn_norm);
        w.o_s = (uint8_t*)m->mem + lo.o_s;
        w.d_s = lo.d_s ? (uint8_t*)m->mem + lo.d_s : nullptr;
        if (L.tc) {
            w.bq_qkv.tiles = (const uint8_t*)m->mem + lo.t_qkv;
            w.bq_o.tiles = (const uint8_t*)m->mem + lo.t_o;
            w.bq_gu.tiles = (const uint8_t*)m->mem + lo.t_gu;
            w.bq_down.tiles = (const uint8_t*)m->mem + lo.t_down;
        }
        m->layers.push_back(w);
    }
    m->tok = qmat(m->mem, L.tok);
    m->out_norm = (float*)((char*)m->mem + L.out_norm);
    m->tc = L.tc;
    if (m->tc) m->bq_tok.tiles = (const uint8_t*)m->mem + L.t_tok;
    *out = m;
    return OCR_OK;
}

// where a GGUF-level tensor (layer, kind) lives: matrix + its row mapping, or a norm vector
struct Where {
    bool is_norm = false;
    QMat mat;
    int rows = 0, row_mul = 1, row_add = 0;
    float* norm = nullptr;
    int n = 0;
};

bool where(const ocr_model* m, int layer, int kind, Where& w) {
    const auto& c = m->cfg;
    const int qd = c.n_head * c.d_head, kvd = c.n_kv * c.d_head;
    if (layer < 0) {
        if (kind == 0) {
            w.mat = m->tok;
            w.rows = c.n_vocab;
            return true;
        }
        if (kind == 1) {
            w.is_norm = true;
            w.norm = m->out_norm;
            w.n = c.dim;
            return true;
        }
        return false;
    }
    if (layer >= c.n_layer) return false;
    const LayerW& L = m->layers[layer];
    switch (kind) {
    case 0: w.is_norm = true; w.norm = L.attn_norm; w.n = c.dim; return true;
    case 1: w.mat = L.qkv; w.rows = qd; return true;
    case 2: w.mat = L.qkv; w.rows = kvd; w.row_add = qd; return true;
    case 3: w.mat = L.qkv; w.rows = kvd; w.row_add = qd + kvd; return true;
    case 4: w.mat = L.o; w.rows = c.dim; return true;
    case 5: w.is_norm = true; w.norm = L.q_norm; w.n = c.d_head; return true;
    case 6: w.is_norm = true; w.norm = L.k_norm; w.n = c.d_head; return true;
    case 7: w.is_norm = true; w.norm = L.ffn_norm; w.n = c.dim; return true;
    case 8: w.mat = L.gu; w.rows = c.n_ff; w.row_mul = 2; return true;
    case 9: w.mat = L.gu; w.rows = c.n_ff; w.row_mul = 2; w.row_add = 1; return true;
    case 10: w.mat = L.down; w.rows = c.dim; return true;
    default: return false;
    }
}

ocr_status ensure_stage(ocr_ctx* ctx) {
    if (ctx->h_stage) return OCR_OK;
    OCR_CUDA(cudaMallocHost(&ctx->h_stage, STAGE_BYTES));
    OCR_CUDA(cudaMalloc(&ctx->d_stage, STAGE_BYTES));
    ctx->stage_bytes = STAGE_BYTES;
    return OCR_OK;
}

// stream one GGUF tensor file → pinned staging → device staging → its place (repacked)
ocr_status upload_tensor(ocr_model* m, const Gguf& g, const GTensor& t, const Where& w) {
    ocr_ctx* ctx = m->ctx;
    OCR_TRY(ensure_stage(ctx));
    std::string msg;
    if (w.is_norm) {
        const size_t n = (size_t)w.n * 4;
        if (!g.src->read_at(t.file_offset, ctx->h_stage, n, msg)) return fail(OCR_ERR_IO, msg);
        OCR_CUDA(cudaMemcpyAsync(w.norm, ctx->h_stage, n, cudaMemcpyHostToDevice, ctx->stream));
        OCR_CUDA(cudaStreamSynchronize(ctx->stream));
        return OCR_OK;
    }
    const int cols = w.mat.cols;
    const size_t row_bytes = (size_t)cols / 32 * 34;
    const int rows_per = (int)std::max<size_t>(1, ctx->stage_bytes / row_bytes);
    for (int r0 = 0; r0 < w.rows; r0 += rows_per) {
        const int nr = std::min(rows_per, w.rows - r0);
        const size_t n = (size_t)nr * row_bytes;
        if (!g.src->read_at(t.file_offset + (uint64_t)r0 * row_bytes, ctx->h_stage, n, msg)) return fail(OCR_ERR_IO, msg);
        OCR_CUDA(cudaMemcpyAsync(ctx->d_stage, ctx->h_stage, n, cudaMemcpyHostToDevice, ctx->stream));
        launch_repack_q8_0(ctx->stream, (const uint8_t*)ctx->d_stage, nr, cols, const_cast<uint8_t*>(w.mat.w),
                           w.row_mul, r0 * w.row_mul + w.row_add);
        OCR_CUDA(cudaGetLastError());
        OCR_CUDA(cudaStreamSynchronize(ctx->stream));
    }
    return OCR_OK;
}

// TextConfig::from_gguf (text.rs:51-82)
ocr_status cfg_from_gguf(const Gguf& g, ocr_text_cfg& c) {
    std::string msg, arch;
    if (!g.get_str("general.architecture", arch, msg)) return fail(OCR_ERR_FORMAT, msg);
    if (arch != "qwen3") return fail(OCR_ERR_FORMAT, "architecture \"" + arch + "\": this engine runs qwen3 only");
    uint32_t v[8];
    const char* keys[] = {"qwen3.attention.key_length", "qwen3.attention.value_length", "qwen3.attention.head_count",
                          "qwen3.attention.head_count_kv", "qwen3.block_count", "qwen3.embedding_length",
                          "qwen3.feed_forward_length", "qwen3.context_length"};
    for (int i = 0; i < 8; i++)
        if (!g.get_u32(keys[i], v[i], msg)) return fail(OCR_ERR_FORMAT, msg);
    if (v[0] != 128 || v[1] != 128)
        return fail(OCR_ERR_FORMAT, "head dim " + std::to_string(v[0]) + ": the attention kernels are written for 128");
    if (v[3] == 0 || v[2] % v[3] != 0)
        return fail(OCR_ERR_FORMAT, std::to_string(v[2]) + " q heads on " + std::to_string(v[3]) + " kv heads");
    if (g.has_key("qwen3.rope.scaling.type") || g.has_key("qwen3.rope.dimension_count"))
        return fail(OCR_ERR_FORMAT, "rope scaling / partial rope in the GGUF: not part of this engine's graph");
    const GTensor* tok = g.info("token_embd.weight");
    if (!tok) return fail(OCR_ERR_FORMAT, "GGUF has no tensor token_embd.weight");
    c.d_head = (int)v[0];
    c.n_head = (int)v[2];
    c.n_kv = (int)v[3];
    c.n_layer = (int)v[4];
    c.dim = (int)v[5];
    c.n_ff = (int)v[6];
    c.n_ctx_train = (int)v[7];
    if (!g.get_f32("qwen3.attention.layer_norm_rms_epsilon", c.eps, msg)) return fail(OCR_ERR_FORMAT, msg);
    if (!g.get_f32("qwen3.rope.freq_base", c.rope_base, msg)) return fail(OCR_ERR_FORMAT, msg);
    c.n_vocab = (int)tok->shape.back();
    return OCR_OK;
}

// the GGUF tensor names of a layer's kinds (ocr_model_tensor_gguf numbering)
const char* const KIND_NAMES[11] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output", "attn_q_norm",
                                    "attn_k_norm", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};

// a kind's expected GGUF form: a matrix [cols, rows] q8_0 or an f32 vector [n]
void kind_shape(const ocr_text_cfg& c, int kind, bool& is_norm, int& rows, int& cols) {
    const int qd = c.n_head * c.d_head, kvd = c.n_kv * c.d_head;
    is_norm = false;
    switch (kind) {
    case 0: case 7: is_norm = true; rows = 1; cols = c.dim; break;
    case 5: case 6: is_norm = true; rows = 1; cols = c.d_head; break;
    case 1: rows = qd; cols = c.dim; break;
    case 2: case 3: rows = kvd; cols = c.dim; break;
    case 4: rows = c.dim; cols = qd; break;
    case 8: case 9: rows = c.n_ff; cols = c.dim; break;
    default: rows = c.dim; cols = c.n_ff; break;
    }
}

ocr_status check_tensor(const Gguf& g, const std::string& name, bool is_norm, int rows, int cols) {
    const GTensor* t = g.info(name);
    if (!t) return fail(OCR_ERR_FORMAT, "GGUF has no tensor " + name);
    if (is_norm) {
        if (t->type != GType::F32 || t->shape.size() != 1 || t->shape[0] != (uint64_t)cols)
            return fail(OCR_ERR_FORMAT, name + ": expected F32 [" + std::to_string(cols) + "]");
        return OCR_OK;
    }
    if (t->shape.size() != 2 || t->shape[0] != (uint64_t)cols || t->shape[1] != (uint64_t)rows)
        return fail(OCR_ERR_FORMAT, name + ": shape, expected [" + std::to_string(cols) + ", " + std::to_string(rows) + "]");
    if (t->type != GType::Q8_0) return fail(OCR_ERR_FORMAT, name + ": the text decoder's kernels read q8_0 weights");
    return OCR_OK;
}

// TextConfig::from_gguf + every check TextModel::load makes before it uploads (text.rs:51-82, 111-128, 332-375)
ocr_status validate_gguf(const Gguf& g, ocr_text_cfg& c) {
    OCR_TRY(cfg_from_gguf(g, c));
    const int qd = c.n_head * c.d_head;
    if (c.dim % 32 != 0 || c.n_ff % 32 != 0 || qd % 32 != 0)
        return fail(OCR_ERR_FORMAT, "dims " + std::to_string(c.dim) + " / " + std::to_string(c.n_ff) + " / " +
                                        std::to_string(qd) + ": q8_0 rows must be whole blocks");
    for (int i = 0; i < c.n_layer; i++) {
        for (const char* absent : {"attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down"}) {
            const std::string b = "blk." + std::to_string(i) + "." + absent + ".bias";
            if (g.has(b)) return fail(OCR_ERR_FORMAT, b + " is in the GGUF but not part of this engine's graph");
        }
        if (g.has("blk." + std::to_string(i) + ".attn_qkv.weight"))
            return fail(OCR_ERR_FORMAT, "blk." + std::to_string(i) + ": a fused attn_qkv — this engine reads separate q / k / v");
        for (int k = 0; k < 11; k++) {
            bool is_norm;
            int rows, cols;
            kind_shape(c, k, is_norm, rows, cols);
            OCR_TRY(check_tensor(g, "blk." + std::to_string(i) + "." + KIND_NAMES[k] + ".weight", is_norm, rows, cols));
        }
    }
    if (g.has("output.weight")) return fail(OCR_ERR_FORMAT, "output.weight is in the GGUF: this engine ties the output to token_embd");
    OCR_TRY(check_tensor(g, "token_embd.weight", false, c.n_vocab, c.dim));
    OCR_TRY(check_tensor(g, "output_norm.weight", true, 1, c.dim));
    return check_cfg(c);
}

// TextModel::load (text.rs:332-375) from a parsed GGUF
ocr_status load_gguf(ocr_ctx* ctx, Gguf& g, ocr_model** out) {
    ocr_text_cfg c{};
    OCR_TRY(validate_gguf(g, c));
    ocr_model* m = nullptr;
    OCR_TRY(model_alloc(ctx, c, &m));
    auto load_one = [&](int layer, int kind, const std::string& name) -> ocr_status {
        Where w;
        where(m, layer, kind, w);
        return upload_tensor(m, g, *g.info(name), w);
    };
    ocr_status st = OCR_OK;
    for (int l = 0; l < c.n_layer && st == OCR_OK; l++)
        for (int k = 0; k < 11 && st == OCR_OK; k++)
            st = load_one(l, k, "blk." + std::to_string(l) + "." + KIND_NAMES[k] + ".weight");
    if (st == OCR_OK) st = load_one(-1, 0, "token_embd.weight");
    if (st == OCR_OK) st = load_one(-1, 1, "output_norm.weight");
    if (st == OCR_OK) {
        derive_weights(m, ctx->stream);
        cudaError_t e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) st = cuda_fail(e, "derive_weights");
    }
    if (st != OCR_OK) {
        std::string keep = g_err;
        ocr_model_destroy(m);
        g_err = keep;
        return st;
    }
    *out = m;
    return OCR_OK;
}

}  // namespace

// ---------------------------------------------------------------------------------------------------------------------
// session
// ---------------------------------------------------------------------------------------------------------------------
struct ocr_session {
    ocr_model* m = nullptr;
    ocr_ctx* ctx = nullptr;
    int n_ctx = 0, B = 0, qkv_w = 0, qd = 0, splits = 1;
    __half *kc = nullptr, *vc = nullptr;
    size_t kv_bytes = 0;
    void* work = nullptr;
    size_t work_bytes = 0;
    float *rope = nullptr, *x = nullptr, *qkv = nullptr, *attn = nullptr, *g = nullptr, *logits = nullptr;
    float* x2 = nullptr;     // the second residual buffer of the fused layer
    float* opart = nullptr;  // [B][n_kv][dim] the attention clusters' o-projection partials (null: unfused layer)
    float* dpart = nullptr;  // [FFN_NCLU][dim] the fused FFN's down partials (one slot)
    bool tc = false;            // batched contractions on the tensor cores (more than 8 slots)
    uint8_t* x16a = nullptr;    // [groups] operands of width dim (x16 layout)
    uint8_t* x16g = nullptr;    // [groups] operands of width n_ff (the SwiGLU output)
    bool battn = false;         // the batched attention (k_attn_batch) and the o-projection on the tensor cores
    int ab_split = 1;           // its CTAs per (slot, kv head)
    uint8_t* x16o = nullptr;    // [groups] operands of width n_head x 128 (the attention's output)
    float* ab_part = nullptr;   // [B * n_kv][split][G][132] partials (split > 1)
    uint32_t* ab_done = nullptr;  // [B * n_kv] tickets
    float* bg_part = nullptr;     // the split contractions' partials (sized for the largest)
    uint32_t* bg_tickets = nullptr;
    // [dim / 128][B] the residual rows' sums of squares per 128-column tile, written by the residual-adding
    // contractions, read by the next contraction that RMS-normalises its operand itself (null: separate prep kernels)
    float* ssq = nullptr;
    float* lm_part = nullptr;
    uint32_t* lm_done = nullptr;
    int32_t *pos = nullptr, *len = nullptr, *tok = nullptr, *active = nullptr;
    int32_t* remaining = nullptr;  // [B] token budgets of the page engine (ocr_read_pages), after `active`
    bool pages = false;            // steps recorded now count budgets down (the page engine is running)
    int32_t* hist = nullptr;
    int hist_cap = 0;
    uint32_t* counts = nullptr;
    float* fpen = nullptr;
    std::vector<int> n_past, has_logits;
    // prefill scratch
    void* pf = nullptr;
    size_t pf_bytes = 0;
    // the decode step's graph and what it was captured with
    cudaGraphExec_t gexec = nullptr;
    float g_rp = 0, g_fp = 0;
    int g_window = -1, g_use_fp = -1;
    bool g_pages = false;
    int32_t* g_hist = nullptr;
    int32_t* h_ids = nullptr;  // pinned readback
    size_t h_ids_n = 0;
    std::vector<cudaEvent_t> step_ev;  // run-ahead: one event per queued step (ring)

    __half* kcl(int l) const { return kc + (size_t)l * B * m->cfg.n_kv * n_ctx * 128; }
    __half* vcl(int l) const { return vc + (size_t)l * B * m->cfg.n_kv * n_ctx * 128; }
};

namespace {

// the per-dispatch profiler: an event after every launch, with the kernel's name, layer and algorithmic bytes
struct Prof {
    cudaStream_t st = nullptr;
    std::vector<cudaEvent_t> ev;
    std::vector<ocr_kernel_time> rec;
    std::vector<int> pos;  // host positions of the active slots (the attention's key counts)
    // the in-chain timeline (ocr_timeline_step): launch i records into tl[i]; no events, the launches chained
    TlSlot* tl = nullptr;
    int tl_cap = 0;
    void mark(const char* name, int layer, double bytes) {
        if (!tl) {
            cudaEvent_t e;
            cudaEventCreate(&e);
            cudaEventRecord(e, st);
            ev.push_back(e);
        }
        ocr_kernel_time k{};
        snprintf(k.name, sizeof(k.name), "%s", name);
        k.layer = layer;
        k.bytes = bytes;
        rec.push_back(k);
    }
};

double mat_bytes(const QMat& w) { return (double)w.rows * w.stride; }

// the timeline slot of the next launch (null unless a timeline is being recorded)
TlSlot* tl_slot(const Prof* p) {
    return p && p->tl && (int)p->rec.size() < p->tl_cap ? p->tl + p->rec.size() : nullptr;
}

LmArgs sampler_args(ocr_session* s, const ocr_sampler_cfg* cfg);

// One decode step of a batch of more than 8 slots, its contractions on the tensor cores (k_bgemm.cu). Per layer:
// the slots' residual rows (layer 0: their tokens' embedding rows) RMS-normalised into the operand (prep), the qkv
// contraction, the batched attention (k_attn_batch.cu) writing the o-projection's operand, the o-projection adding
// onto the residual, the FFN's operand prep, the gate|up contraction whose SwiGLU epilogue writes the down
// contraction's operand, and the down contraction adding onto the residual. Then the LM head's prep and its
// contraction with the windowed penalty and the choice. (With OCR_BATTN=0 the attention is the cluster kernel with
// the o-projection fused per kv head, and the FFN's prep sums its partial products.)
void record_step_tc(ocr_session* s, bool sample, float rp, int window, int use_fp, float fp, Prof* prof,
                    bool x_given) {
    const ocr_model* m = s->m;
    const auto& c = m->cfg;
    ocr_ctx* ctx = s->ctx;
    cudaStream_t st = ctx->stream;
    const bool pdl = ctx->pdl && (!prof || prof->tl);
    const double nact = prof ? (double)prof->pos.size() : 0.0;
    auto prep = [&](int layer, const float* nw, const float* xadd, int n_add, bool embed, bool chain) {
        PrepArgs p;
        p.x = s->x;
        p.x_stride = c.dim;
        p.xadd = xadd;
        p.n_add = n_add;
        if (embed) {
            p.tok = s->tok;
            p.emb = m->tok;
        }
        p.x_out = (embed || xadd) ? s->x : nullptr;
        p.nw = nw;
        p.eps = c.eps;
        p.K = c.dim;
        p.nb = s->B;
        p.active = s->active;
        p.x16 = s->x16a;
        p.err = ctx->d_err;
        p.tl = tl_slot(prof);
        launch_xprep(st, p, chain);
        if (prof)
            prof->mark(embed ? "prep (embed, norm, hi/lo)" : xadd ? "prep (sum, norm, hi/lo)" : "prep (norm, hi/lo)",
                       layer, nact * c.dim * (8.0 + 4.0 * n_add + (xadd ? 4.0 : 0.0)));
    };
    auto gemm = [&](const QMat& w, const BgMaps& bq, const uint8_t* x16, int mode, float* y, int y_stride,
                    uint8_t* y16) {
        BgArgs g;
        g.w = w;
        g.x16 = x16;
        g.mode = mode;
        g.y = y;
        g.y_stride = y_stride;
        g.y16 = y16;
        g.nb = s->B;
        g.active = s->active;
        g.err = ctx->d_err;
        g.tl = tl_slot(prof);
        if (mode != MV_LMHEAD) {
            g.ksplit = bgemm_ksplit(ctx->num_sms, w.rows, w.cols);
            g.part = s->bg_part;
            g.tickets = s->bg_tickets;
        }
        return g;
    };
    // the norms inside the contractions: the residual-adding ones write the new rows' sums of squares, the qkv
    // (layers after the first) and gate|up contractions build their normalised operand from the residual
    const bool nin = s->ssq != nullptr && s->battn;
    auto norm_in = [&](BgArgs g, const float* nw) {
        g.xn = s->x;
        g.nw = nw;
        g.ssq_in = s->ssq;
        g.eps = c.eps;
        return g;
    };
    auto ssq_out = [&](BgArgs g) {
        if (nin) g.ssq_out = s->ssq;
        return g;
    };
    for (int l = 0; l < c.n_layer; l++) {
        const LayerW& L = m->layers[l];
        const bool qkv_in = nin && l > 0;
        if (!qkv_in) prep(l, L.attn_norm, nullptr, 0, l == 0 && !x_given, pdl && l > 0);
        BgArgs gq = gemm(L.qkv, L.bq_qkv, s->x16a, MV_STORE, s->qkv, s->qkv_w, nullptr);
        if (qkv_in) gq = norm_in(gq, L.attn_norm);
        launch_bgemm(st, gq, L.bq_qkv, ctx->num_sms, pdl);
        if (prof) prof->mark("qkv (tcgen05)", l, mat_bytes(L.qkv) + nact * (c.dim * 4.0 + s->qkv_w * 4.0));
        double kv = 0;
        if (prof)
            for (int p : prof->pos) kv += (double)(p + 1) * c.n_kv * 128 * 2 * 2;
        if (s->battn) {
            // the batched attention writes the o-projection's operand; the o-projection adds onto the residual
            AttnBatchArgs a;
            a.qkv = s->qkv;
            a.qkv_stride = s->qkv_w;
            a.q_norm = L.q_norm;
            a.k_norm = L.k_norm;
            a.rope = s->rope;
            a.kc = s->kcl(l);
            a.vc = s->vcl(l);
            a.pos = s->pos;
            a.active = s->active;
            a.n_head = c.n_head;
            a.n_kv = c.n_kv;
            a.n_ctx = s->n_ctx;
            a.nb = s->B;
            a.eps = c.eps;
            a.scale = 1.0f / sqrtf((float)c.d_head);
            a.x16 = s->x16o;
            a.part = s->ab_part;
            a.done = s->ab_done;
            a.err = ctx->d_err;
            a.tl = tl_slot(prof);
            launch_attention_batch(st, a, s->ab_split, pdl);
            if (prof) prof->mark("attention (batched)", l, kv + nact * (s->qkv_w * 4.0 + s->qd * 4.0));
            launch_bgemm(st, ssq_out(gemm(L.o, L.bq_o, s->x16o, MV_ADD, s->x, c.dim, nullptr)), L.bq_o, ctx->num_sms, pdl);
            if (prof) prof->mark("o + residual (tcgen05)", l, mat_bytes(L.o) + nact * (s->qd * 4.0 + c.dim * 8.0));
            if (!nin) prep(l, L.ffn_norm, nullptr, 0, false, pdl);
        } else {
            AttnArgs a;
            a.qkv = s->qkv;
            a.qkv_stride = s->qkv_w;
            a.q_norm = L.q_norm;
            a.k_norm = L.k_norm;
            a.rope = s->rope;
            a.kc = s->kcl(l);
            a.vc = s->vcl(l);
            a.pos = s->pos;
            a.active = s->active;
            a.n_head = c.n_head;
            a.n_kv = c.n_kv;
            a.n_ctx = s->n_ctx;
            a.splits = s->splits;
            a.eps = c.eps;
            a.scale = 1.0f / sqrtf((float)c.d_head);
            a.out = s->attn;
            a.out_stride = s->qd;
            a.nb = s->B;
            a.err = ctx->d_err;
            a.wo = L.o_s;
            a.dim = c.dim;
            a.opart = s->opart;
            a.tl = tl_slot(prof);
            launch_attention_decode(st, a, pdl);
            if (prof)
                prof->mark("attention + o-proj", l,
                           kv + (double)c.n_kv * c.dim * q8_stride(s->qd / c.n_kv) +
                               nact * (s->qkv_w * 4.0 + c.n_kv * c.dim * 4.0));
            prep(l, L.ffn_norm, s->opart, c.n_kv, false, pdl);
        }
        BgArgs gg = gemm(L.gu, L.bq_gu, s->x16a, MV_SWIGLU, nullptr, 0, s->x16g);
        if (nin) gg = norm_in(gg, L.ffn_norm);
        launch_bgemm(st, gg, L.bq_gu, ctx->num_sms, pdl);
        if (prof) prof->mark("gate|up + swiglu (tcgen05)", l, mat_bytes(L.gu) + nact * (c.dim * 4.0 + c.n_ff * 4.0));
        launch_bgemm(st, ssq_out(gemm(L.down, L.bq_down, s->x16g, MV_ADD, s->x, c.dim, nullptr)), L.bq_down,
                     ctx->num_sms, pdl);
        if (prof) prof->mark("down + residual (tcgen05)", l, mat_bytes(L.down) + nact * (c.n_ff * 4.0 + c.dim * 8.0));
    }
    prep(-1, m->out_norm, nullptr, 0, false, pdl);
    BgArgs h = gemm(m->tok, m->bq_tok, s->x16a, MV_LMHEAD, s->logits, c.n_vocab, nullptr);
    ocr_sampler_cfg sc{rp, window, fp, 1};
    h.lm = sampler_args(s, &sc);
    if (!sample) h.lm.remaining = h.lm.active_w = nullptr;
    h.lm.sample = sample ? 1 : 0;
    h.lm.use_fp = use_fp;
    h.lm.advance_pos = sample ? 1 : 0;
    h.lm.nb = s->B;
    launch_bgemm(st, h, m->bq_tok, ctx->num_sms, pdl);
    if (prof)
        prof->mark(sample ? "lm head + choice (tcgen05)" : "lm head (tcgen05)", -1,
                   mat_bytes(m->tok) + nact * (c.dim * 4.0 + c.n_vocab * 4.0));
}

// one decode step of every active slot: 5 kernels per layer + the LM head (with the choice when sample). The first
// layer embeds the slots' tokens, or with x_given takes the rows already in s->x (Input::Embeddings rows).
void record_step(ocr_session* s, bool sample, float rp, int window, int use_fp, float fp, Prof* prof = nullptr,
                 bool x_given = false) {
    if (s->tc) {
        record_step_tc(s, sample, rp, window, use_fp, fp, prof, x_given);
        return;
    }
    const ocr_model* m = s->m;
    const auto& c = m->cfg;
    ocr_ctx* ctx = s->ctx;
    cudaStream_t st = ctx->stream;
    // programmatic dependent launch chains each kernel to the one before it in the stream; the profiler's events
    // between launches would break that chain, so a profiled step launches without it (a timeline keeps it)
    const bool pdl = ctx->pdl && (!prof || prof->tl);
    // each kernel pulls what a later kernel of the step reads into L2 (the attention's KV two kernels ahead, a
    // matrix two kernels ahead, past the attention which reads none)
    auto kv_of = [&](int l) {
        L2Next n;
        n.kc = s->kcl(l);
        n.vc = s->vcl(l);
        n.pos = s->pos;
        n.active = s->active;
        n.n_kv = c.n_kv;
        n.n_ctx = s->n_ctx;
        n.nb = s->B;
        return n;
    };
    auto with_w = [](L2Next n, const QMat& w) {
        n.w = w.w;
        n.w_bytes = (size_t)w.rows * w.stride;
        return n;
    };
    // Fused (the decode shapes this engine targets): the attention cluster of each kv head also multiplies its heads'
    // output by its slice of W_o, and the gate/up kernel sums those n_kv partial products onto the residual, which
    // it writes to the other of two residual buffers (its other CTAs are still reading the first). Otherwise the
    // o-projection is its own kernel, adding in place.
    // One slot with a fitting shape goes further: the FFN is one kernel of FFN_NCLU clusters whose down-projection
    // partials the next layer's first kernel (or the LM head) sums onto the residual. Residual buffers then: the
    // layer's first kernel writes x (layer input + FFN partials), the FFN kernel x2 (x + o-partials).
    // With the o-projection fused, the qkv projection moves into the attention clusters too when their shape allows
    // (decided per layer): the attention kernel stages the residual itself. One slot: 2 kernels per layer.
    const bool fused = s->opart != nullptr;
    const bool ffn = s->dpart != nullptr && ffn_usable(c.dim, c.n_ff);
    const bool fqkv = fused;
    for (int l = 0; l < c.n_layer; l++) {
        const LayerW& L = m->layers[l];
        float* xin = fused && !ffn && (l & 1) ? s->x2 : s->x;   // this layer's input residual
        float* xout = fused ? ((l & 1) && !ffn ? s->x : s->x2) : s->x;  // and its output
        MvArgs q;
        q.w = L.qkv;
        q.nw = L.attn_norm;
        q.eps = c.eps;
        q.y = s->qkv;
        q.y_stride = s->qkv_w;
        q.nb = s->B;
        q.active = s->active;
        q.mode = MV_STORE;
        q.err = ctx->d_err;
        q.next = l == 0 ? kv_of(0) : L2Next();
        if (fused) {
            q.next.w = L.o_s;
            q.next.w_bytes = (size_t)c.n_kv * c.dim * q8_stride(s->qd / c.n_kv);
        } else {
            q.next = with_w(q.next, L.o);
        }
        q.x_stride = c.dim;
        if (l == 0 && !x_given) {
            q.tok = s->tok;
            q.emb = m->tok;
            q.x_out = xin;
        } else if (l > 0 && ffn) {
            q.x = s->x2;
            q.xadd = s->dpart;
            q.n_add = FFN_NCLU;
            q.x_out = s->x;
        } else {
            q.x = xin;
        }
        const double nact = prof ? (double)prof->pos.size() : 0.0;
        AttnArgs a;
        a.qkv = s->qkv;
        a.qkv_stride = s->qkv_w;
        a.q_norm = L.q_norm;
        a.k_norm = L.k_norm;
        a.rope = s->rope;
        a.kc = s->kcl(l);
        a.vc = s->vcl(l);
        a.pos = s->pos;
        a.active = s->active;
        a.n_head = c.n_head;
        a.n_kv = c.n_kv;
        a.n_ctx = s->n_ctx;
        a.splits = s->splits;
        a.eps = c.eps;
        a.scale = 1.0f / sqrtf((float)c.d_head);
        a.out = s->attn;
        a.out_stride = s->qd;
        a.nb = s->B;
        a.err = ctx->d_err;
        a.next = with_w(L2Next(), L.gu);
        if (ffn) {
            a.next.w2 = L.d_s;
            a.next.w2_bytes = (size_t)FFN_NCLU * c.dim * q8_stride(c.n_ff / FFN_NCLU);
        }
        if (fused) {
            a.wo = L.o_s;
            a.dim = c.dim;
            a.opart = s->opart;
        }
        // the qkv projection inside the attention clusters when their shape allows: the attention kernel stages the
        // residual row itself (the qkv matvec's arguments) and, as that matvec would, starts the step at layer 0
        a.in = q;
        a.wqkv = L.qkv;
        const bool fq = fqkv && attention_fuses_qkv(c.n_head / c.n_kv, attention_cluster(a), c.dim);
        if (!fq) {
            a.wqkv = QMat();
            q.tl = tl_slot(prof);
            launch_matvec(st, q, ctx->num_sms, pdl && l > 0);
            if (prof) prof->mark("qkv (norm + q|k|v)", l, mat_bytes(L.qkv) + nact * (c.dim * 8.0 + s->qkv_w * 4.0));
        }
        a.tl = tl_slot(prof);
        launch_attention_decode(st, a, pdl && (l > 0 || !fq));
        if (prof) {
            double kv = 0;
            for (int p : prof->pos) kv += (double)(p + 1) * c.n_kv * 128 * 2 * 2;
            if (fq)
                prof->mark("qkv + attention + o-proj", l,
                           mat_bytes(L.qkv) + kv + (double)c.n_kv * c.dim * q8_stride(s->qd / c.n_kv) +
                               nact * (c.dim * 8.0 + c.n_kv * c.dim * 4.0));
            else if (fused)
                prof->mark("attention + o-proj", l,
                           kv + (double)c.n_kv * c.dim * q8_stride(s->qd / c.n_kv) +
                               nact * (s->qkv_w * 4.0 + c.n_kv * c.dim * 4.0));
            else
                prof->mark("attention (split-KV)", l, kv + nact * (s->qkv_w * 4.0 + s->qd * 4.0));
        }
        if (!fused) {
        MvArgs o;
        o.w = L.o;
        o.x = s->attn;
        o.x_stride = s->qd;
        o.y = s->x;
        o.y_stride = c.dim;
        o.mode = MV_ADD;
        o.nb = s->B;
        o.active = s->active;
        o.err = ctx->d_err;
        o.next = with_w(L2Next(), L.down);
        o.tl = tl_slot(prof);
        launch_matvec(st, o, ctx->num_sms, pdl);
        if (prof) prof->mark("o (+ residual)", l, mat_bytes(L.o) + nact * (s->qd * 4.0 + c.dim * 8.0));
        }

        if (ffn) {
            FfnArgs f;
            f.in.w.cols = c.dim;
            f.in.x = s->x;
            f.in.x_stride = c.dim;
            f.in.xadd = s->opart;
            f.in.n_add = c.n_kv;
            f.in.x_out = s->x2;
            f.in.nw = L.ffn_norm;
            f.in.eps = c.eps;
            f.gu = L.gu;
            f.wd = L.d_s;
            f.n_ff = c.n_ff;
            f.dpart = s->dpart;
            f.err = ctx->d_err;
            if (l + 1 < c.n_layer) {
                f.next = with_w(kv_of(l + 1), m->layers[l + 1].qkv);
                f.next.w2 = m->layers[l + 1].o_s;  // read by the next attention (its o-projection)
                f.next.w2_bytes = (size_t)c.n_kv * c.dim * q8_stride(s->qd / c.n_kv);
            }
            f.tl = tl_slot(prof);
            launch_ffn(st, f, pdl);
            if (prof)
                prof->mark("ffn (gate|up, swiglu, down)", l,
                           mat_bytes(L.gu) + (double)FFN_NCLU * c.dim * q8_stride(c.n_ff / FFN_NCLU) +
                               c.dim * 4.0 * (2 + c.n_kv + FFN_NCLU));
            continue;
        }
        MvArgs f;
        f.w = L.gu;
        f.x = xin;
        if (fused) {
            f.xadd = s->opart;
            f.n_add = c.n_kv;
            f.x_out = xout;
        }
        f.x_stride = c.dim;
        f.nw = L.ffn_norm;
        f.eps = c.eps;
        f.y = s->g;
        f.y_stride = c.n_ff;
        f.mode = MV_SWIGLU;
        f.nb = s->B;
        f.active = s->active;
        f.err = ctx->d_err;
        if (l + 1 < c.n_layer) f.next = with_w(L2Next(), m->layers[l + 1].qkv);
        f.tl = tl_slot(prof);
        launch_matvec(st, f, ctx->num_sms, pdl);
        if (prof)
            prof->mark(fused ? "sum + gate|up + swiglu" : "gate|up + swiglu", l,
                       mat_bytes(L.gu) + nact * (c.dim * (fused ? 8.0 + 4.0 * c.n_kv : 8.0) + c.n_ff * 4.0));

        MvArgs dn;
        dn.w = L.down;
        dn.x = s->g;
        dn.x_stride = c.n_ff;
        dn.y = xout;
        dn.y_stride = c.dim;
        dn.mode = MV_ADD;
        dn.nb = s->B;
        dn.active = s->active;
        dn.err = ctx->d_err;
        if (l + 1 < c.n_layer) dn.next = kv_of(l + 1);
        dn.tl = tl_slot(prof);
        launch_matvec(st, dn, ctx->num_sms, pdl);
        if (prof) prof->mark("down (+ residual)", l, mat_bytes(L.down) + nact * (c.n_ff * 4.0 + c.dim * 8.0));
    }
    MvArgs lm;
    lm.w = m->tok;
    lm.x = fused && !ffn && (c.n_layer & 1) ? s->x2 : s->x;
    if (ffn) {
        lm.x = s->x2;
        lm.xadd = s->dpart;
        lm.n_add = FFN_NCLU;
    }
    lm.x_stride = c.dim;
    lm.nw = m->out_norm;
    lm.eps = c.eps;
    lm.nb = s->B;
    lm.mode = MV_LMHEAD;
    lm.y = s->logits;
    lm.active = s->active;
    lm.err = ctx->d_err;
    lm.lm.sample = sample ? 1 : 0;
    lm.lm.rp = rp;
    lm.lm.window = window;
    lm.lm.use_fp = use_fp;
    lm.lm.fp = fp;
    lm.lm.hist = s->hist;
    lm.lm.hist_cap = s->hist_cap;
    lm.lm.len = s->len;
    lm.lm.tok = s->tok;
    lm.lm.pos = s->pos;
    lm.lm.advance_pos = sample ? 1 : 0;
    lm.lm.counts = s->counts;
    lm.lm.fpen = s->fpen;
    lm.lm.active = s->active;
    lm.lm.part = s->lm_part;
    lm.lm.done = s->lm_done;
    lm.lm.nb = s->B;
    lm.lm.err = ctx->d_err;
    if (s->pages && sample) {
        lm.lm.remaining = s->remaining;
        lm.lm.active_w = s->active;
    }
    lm.next = with_w(kv_of(0), m->layers[0].qkv);  // the next step's first kernels
    if (fused) {
        lm.next.w2 = m->layers[0].o_s;
        lm.next.w2_bytes = (size_t)c.n_kv * c.dim * q8_stride(s->qd / c.n_kv);
    }
    lm.tl = tl_slot(prof);
    launch_matvec(st, lm, ctx->num_sms, pdl);
    if (prof)
        prof->mark(sample ? "lm head + choice" : "lm head", -1, mat_bytes(m->tok) + (prof ? prof->pos.size() : 0) * (c.dim * 8.0 + c.n_vocab * 4.0));
}

// rope_table (text.rs:132-142): theta = (f32)pos * base^(-2i/d) in f32, (cos, sin) by the host libm
std::vector<float> rope_table(float base, int d, int n_pos) {
    std::vector<float> out((size_t)n_pos * d);
    const int half = d / 2;
    for (int p = 0; p < n_pos; p++)
        for (int i = 0; i < half; i++) {
            const float theta = (float)p * powf(base, -(float)(2 * i) / (float)d);
            out[((size_t)p * half + i) * 2] = cosf(theta);
            out[((size_t)p * half + i) * 2 + 1] = sinf(theta);
        }
    return out;
}

ocr_status ensure_hist(ocr_session* s, int need) {
    if (s->hist_cap >= need) return OCR_OK;
    int cap = std::max(need, std::max(4096, s->hist_cap * 2));
    OCR_CUDA(cudaStreamSynchronize(s->ctx->stream));
    if (s->hist) dfree(s->hist, (size_t)s->B * s->hist_cap * 4, &s->ctx->mem_work);
    OCR_CUDA(dalloc((void**)&s->hist, (size_t)s->B * cap * 4, &s->ctx->mem_work));
    s->hist_cap = cap;
    if (s->h_ids) cudaFreeHost(s->h_ids);
    OCR_CUDA(cudaMallocHost((void**)&s->h_ids, (size_t)s->B * cap * 4));
    s->h_ids_n = (size_t)s->B * cap;
    return OCR_OK;
}

ocr_status ensure_counts(ocr_session* s) {
    if (s->counts) return OCR_OK;
    const size_t n = (size_t)s->B * s->m->cfg.n_vocab;
    OCR_CUDA(dalloc((void**)&s->counts, n * 4, &s->ctx->mem_work));
    OCR_CUDA(dalloc((void**)&s->fpen, n * 4, &s->ctx->mem_work));
    return OCR_OK;
}

// gpu_choice_capable (text.rs:154-163) + Preset::validate's ranges (presets.rs:37-57)
ocr_status check_sampler(const ocr_sampler_cfg* cfg) {
    if (!cfg) return fail(OCR_ERR_ARG, "no sampler config");
    if (cfg->rp != 1.0f && !(std::isnormal(cfg->rp) && cfg->rp > 0.0f))
        return fail(OCR_ERR_ARG, "the repetition penalty is no positive normal f32");
    if (cfg->window < 1) return fail(OCR_ERR_ARG, "repetition window must be >= 1");
    if (!(cfg->fp >= 0.0f)) return fail(OCR_ERR_ARG, "frequency penalty must be >= 0");
    if (cfg->max_new < 1) return fail(OCR_ERR_ARG, "max_new must be >= 1");
    return OCR_OK;
}

LmArgs sampler_args(ocr_session* s, const ocr_sampler_cfg* cfg) {
    LmArgs a;
    a.nb = s->B;
    a.sample = 1;
    a.rp = cfg->rp;
    a.window = cfg->window;
    a.use_fp = cfg->fp > 0.0f ? 1 : 0;
    a.fp = cfg->fp;
    a.hist = s->hist;
    a.hist_cap = s->hist_cap;
    a.len = s->len;
    a.tok = s->tok;
    a.pos = s->pos;
    a.counts = s->counts;
    a.fpen = s->fpen;
    a.active = s->active;
    a.part = s->lm_part;
    a.done = s->lm_done;
    a.err = s->ctx->d_err;
    if (s->pages) {
        a.remaining = s->remaining;
        a.active_w = s->active;
    }
    return a;
}

ocr_status capture_graph(ocr_session* s, const ocr_sampler_cfg* cfg) {
    const int use_fp = cfg->fp > 0.0f ? 1 : 0;
    if (s->gexec && s->g_rp == cfg->rp && s->g_window == cfg->window && s->g_use_fp == use_fp && s->g_fp == cfg->fp &&
        s->g_hist == s->hist && s->g_pages == s->pages)
        return OCR_OK;
    if (s->gexec) {
        cudaGraphExecDestroy(s->gexec);
        s->gexec = nullptr;
    }
    cudaStream_t st = s->ctx->stream;
    cudaGraph_t graph;
    OCR_CUDA(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    record_step(s, true, cfg->rp, cfg->window, use_fp, cfg->fp);
    cudaError_t e = cudaStreamEndCapture(st, &graph);
    if (e != cudaSuccess) return cuda_fail(e, "cudaStreamEndCapture(decode step)");
    e = cudaGraphInstantiate(&s->gexec, graph, 0);
    cudaGraphDestroy(graph);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGraphInstantiate(decode step)");
    s->g_rp = cfg->rp;
    s->g_window = cfg->window;
    s->g_use_fp = use_fp;
    s->g_fp = cfg->fp;
    s->g_hist = s->hist;
    s->g_pages = s->pages;
    return OCR_OK;
}

// the shared decode loop: slots [s0, s0 + ns) active, history [ns][n_hist], up to max_new choices each
ocr_status decode_slots(ocr_session* s, int s0, int ns, const ocr_sampler_cfg* cfg, const int32_t* history, int n_hist,
                        ocr_token_cb cb, void* user, int32_t* ids_out, int* n_out) {
    OCR_TRY(check_sampler(cfg));
    const auto& c = s->m->cfg;
    ocr_ctx* ctx = s->ctx;
    cudaStream_t st = ctx->stream;
    const int max_new = cfg->max_new;
    if (n_hist < 0 || (n_hist > 0 && !history)) return fail(OCR_ERR_ARG, "history: bad length or null");
    const int seed = std::min(n_hist, cfg->window);
    for (int k = 0; k < ns; k++) {
        const int b = s0 + k;
        if (!s->has_logits[b]) return fail(OCR_ERR_STATE, "slot " + std::to_string(b) + ": no logits yet (prefill first)");
        if (s->n_past[b] + max_new - 1 > s->n_ctx)
            return fail(OCR_ERR_STATE, std::to_string(max_new) + " choices: slot " + std::to_string(b) + " at " +
                                           std::to_string(s->n_past[b]) + " overflows the session's " + std::to_string(s->n_ctx));
        for (int i = n_hist - seed; i < n_hist; i++) {
            const int32_t t = history[(size_t)k * n_hist + i];
            if (t < 0 || t >= c.n_vocab) return fail(OCR_ERR_ARG, "history token " + std::to_string(t) + " is outside the vocabulary");
        }
    }
    OCR_TRY(ensure_hist(s, seed + max_new));
    if (cfg->fp > 0.0f) OCR_TRY(ensure_counts(s));
    // device-side state: window seeds, lengths, positions, the active mask
    std::vector<int32_t> hseed((size_t)ns * s->hist_cap, 0), len(s->B, 0), pos(s->B, 0), act(s->B, 0);
    for (int b = 0; b < s->B; b++) pos[b] = s->n_past[b];
    for (int k = 0; k < ns; k++) {
        const int b = s0 + k;
        for (int i = 0; i < seed; i++) hseed[(size_t)k * s->hist_cap + i] = history[(size_t)k * n_hist + n_hist - seed + i];
        len[b] = seed;
        act[b] = 1;
    }
    OCR_CUDA(cudaMemcpyAsync(s->hist + (size_t)s0 * s->hist_cap, hseed.data(), hseed.size() * 4, cudaMemcpyHostToDevice, st));
    OCR_CUDA(cudaMemcpyAsync(s->len, len.data(), s->B * 4, cudaMemcpyHostToDevice, st));
    OCR_CUDA(cudaMemcpyAsync(s->pos, pos.data(), s->B * 4, cudaMemcpyHostToDevice, st));
    OCR_CUDA(cudaMemcpyAsync(s->active, act.data(), s->B * 4, cudaMemcpyHostToDevice, st));
    if (cfg->fp > 0.0f) {
        const size_t n = (size_t)ns * c.n_vocab;
        OCR_CUDA(cudaMemsetAsync(s->counts + (size_t)s0 * c.n_vocab, 0, n * 4, st));
        OCR_CUDA(cudaMemsetAsync(s->fpen + (size_t)s0 * c.n_vocab, 0, n * 4, st));
    }
    // choice 0 from the current logits
    LmArgs sa = sampler_args(s, cfg);
    launch_sample(st, s->logits, c.n_vocab, c.n_vocab, sa, ctx->num_sms, s0, ns);
    OCR_CUDA(cudaGetLastError());
    int steps = 0;
    int delivered = 0;
    bool stopped = false;
    const int chunk = 8;
    const int ring = 4 * chunk;
    if (cb && ns == 1 && s->step_ev.empty()) {
        s->step_ev.resize(ring);
        for (auto& e : s->step_ev) OCR_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
    // choices [delivered, upto) of slot s0 to the callback, once the step that made choice upto - 1 is done
    auto deliver = [&](int upto) -> ocr_status {
        if (upto <= delivered) return OCR_OK;
        if (upto - 1 >= 1) OCR_CUDA(cudaEventSynchronize(s->step_ev[(upto - 1) % ring]));
        else OCR_CUDA(cudaStreamSynchronize(st));
        OCR_CUDA(cudaMemcpy(s->h_ids, s->hist + (size_t)s0 * s->hist_cap + seed + delivered,
                            (size_t)(upto - delivered) * 4, cudaMemcpyDeviceToHost));
        for (int i = delivered; i < upto; i++) {
            ids_out[i] = s->h_ids[i - delivered];
            if (!cb(user, ids_out[i])) {
                stopped = true;
                delivered = i + 1;
                return OCR_OK;
            }
        }
        delivered = upto;
        return OCR_OK;
    };
    auto mark = [&](int step) -> ocr_status {
        if (cb && ns == 1) OCR_CUDA(cudaEventRecord(s->step_ev[step % ring], st));
        return OCR_OK;
    };
    if (max_new > 1) {
        // step 1 runs eagerly (it also settles every launcher's one-time setup), then the captured graph
        record_step(s, true, cfg->rp, cfg->window, cfg->fp > 0.0f ? 1 : 0, cfg->fp);
        OCR_CUDA(cudaGetLastError());
        steps = 1;
        OCR_TRY(mark(steps));
        if (max_new > 2) OCR_TRY(capture_graph(s, cfg));
        while (steps < max_new - 1 && !stopped) {
            OCR_CUDA(cudaGraphLaunch(s->gexec, st));
            steps++;
            OCR_TRY(mark(steps));
            // keep 2 chunks queued ahead of the callback (the reference's run-ahead: chunk x depth 2)
            if (cb && ns == 1 && (steps + 1) - delivered >= 3 * chunk) OCR_TRY(deliver(steps + 1 - 2 * chunk));
        }
    }
    OCR_CUDA(cudaStreamSynchronize(st));
    OCR_TRY(check_device_error(ctx));
    if (cb && ns == 1) {
        if (!stopped) OCR_TRY(deliver(max_new));
        if (n_out) *n_out = delivered;
    } else {
        for (int k = 0; k < ns; k++)
            OCR_CUDA(cudaMemcpy(ids_out + (size_t)k * max_new, s->hist + (size_t)(s0 + k) * s->hist_cap + seed,
                                (size_t)max_new * 4, cudaMemcpyDeviceToHost));
        if (n_out) *n_out = max_new;
    }
    for (int k = 0; k < ns; k++) s->n_past[s0 + k] += steps;
    return OCR_OK;
}

// the prefill's scratch for n rows: x, h, qkv, attention output, g (f32), the ids; with the tensor-core contractions
// also the operands of widths dim, n_head x 128 and n_ff for the rows in groups of 32
size_t prefill_x16_bytes(const ocr_session* s, int n, int K) {
    return (size_t)((n + BG_SLOTS - 1) / BG_SLOTS) * x16_group_bytes(K);
}
ocr_status ensure_prefill(ocr_session* s, int n) {
    const auto& c = s->m->cfg;
    const size_t per_row = (size_t)c.dim * 2 + s->qkv_w + s->qd + c.n_ff + 1;
    size_t need = per_row * n * 4 + 4096;
    if (s->m->tc)
        need += prefill_x16_bytes(s, n, c.dim) + prefill_x16_bytes(s, n, s->qd) + prefill_x16_bytes(s, n, c.n_ff) + 1024;
    if (s->pf_bytes >= need) return OCR_OK;
    OCR_CUDA(cudaStreamSynchronize(s->ctx->stream));
    if (s->pf) dfree(s->pf, s->pf_bytes, &s->ctx->mem_work);
    s->pf = nullptr;
    s->pf_bytes = 0;
    OCR_CUDA(dalloc(&s->pf, need, &s->ctx->mem_work));
    s->pf_bytes = need;
    return OCR_OK;
}

}  // namespace

// =====================================================================================================================
// the C ABI
// =====================================================================================================================
void ocr::ctx_release(ocr_ctx* c) {
    if (--c->refs > 0) return;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    if (c->op_scratch) cudaFree(c->op_scratch);
    if (c->h_stage) cudaFreeHost(c->h_stage);
    if (c->d_stage) cudaFree(c->d_stage);
    if (c->d_err) cudaFree(c->d_err);
    cudaStreamDestroy(c->stream);
    delete c;
}

extern "C" {

const char* ocr_last_error(void) { return g_err.c_str(); }
const char* ocr_version(void) { return "libocrcuda 0.1 (sm_100a)"; }

ocr_status ocr_ctx_create(int device, ocr_ctx** out) {
    if (!out) return fail(OCR_ERR_ARG, "out is null");
    int n = 0;
    OCR_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) return fail(OCR_ERR_ARG, "device " + std::to_string(device) + " of " + std::to_string(n));
    OCR_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    OCR_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major < 10) return fail(OCR_ERR_CUDA, std::string("device ") + prop.name + ": sm_100a (B200) required");
    auto* c = new ocr_ctx;
    c->device = device;
    c->num_sms = prop.multiProcessorCount;
    const char* pdl = getenv("OCR_PDL");
    c->pdl = !(pdl && pdl[0] == '0');
    cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = dalloc((void**)&c->d_err, sizeof(int), nullptr);
    if (e != cudaSuccess) {
        delete c;
        return cuda_fail(e, "ocr_ctx_create");
    }
    *out = c;
    return OCR_OK;
}

// Handles may be released in any order (a garbage collector's, say): a context lives while a model made in it does,
// a model while a session of it does; each destroy call releases the caller's reference.

ocr_status ocr_ctx_destroy(ocr_ctx* c) {
    if (c) ctx_release(c);
    return OCR_OK;
}

ocr_status ocr_ctx_sync(ocr_ctx* c) {
    if (!c) return fail(OCR_ERR_ARG, "ctx is null");
    OCR_CUDA(cudaStreamSynchronize(c->stream));
    OCR_CUDA(cudaGetLastError());
    return check_device_error(c);
}

ocr_status ocr_ctx_stream(ocr_ctx* c, void** stream) {
    if (!c || !stream) return fail(OCR_ERR_ARG, "null argument");
    *stream = (void*)c->stream;
    return OCR_OK;
}

ocr_status ocr_ctx_memory(ocr_ctx* c, uint64_t* w, uint64_t* kv, uint64_t* work) {
    if (!c) return fail(OCR_ERR_ARG, "ctx is null");
    if (w) *w = c->mem_weights;
    if (kv) *kv = c->mem_kv;
    if (work) *work = c->mem_work;
    return OCR_OK;
}

ocr_status ocr_model_load_gguf(ocr_ctx* ctx, const char* path, ocr_model** out) {
    if (!ctx || !path || !out) return fail(OCR_ERR_ARG, "null argument");
    std::string msg;
    auto src = file_source(path, msg);
    if (!src) return fail(OCR_ERR_IO, msg);
    Gguf g;
    if (!g.parse(std::move(src), msg)) return fail(OCR_ERR_FORMAT, std::string(path) + " is not a readable GGUF: " + msg);
    return load_gguf(ctx, g, out);
}

ocr_status ocr_model_load_gguf_memory(ocr_ctx* ctx, const void* bytes, size_t n, ocr_model** out) {
    if (!ctx || !bytes || !out) return fail(OCR_ERR_ARG, "null argument");
    std::string msg;
    Gguf g;
    if (!g.parse(memory_source(bytes, n), msg)) return fail(OCR_ERR_FORMAT, "not a readable GGUF: " + msg);
    return load_gguf(ctx, g, out);
}

ocr_status ocr_model_synthetic(ocr_ctx* ctx, const ocr_text_cfg* cfg, uint64_t seed, float sigma_w, float sigma_e,
                               ocr_model** out) {
    if (!ctx || !cfg || !out) return fail(OCR_ERR_ARG, "null argument");
    ocr_model* m = nullptr;
    OCR_TRY(model_alloc(ctx, *cfg, &m));
    // sub-stream k of the model seed per tensor (the CPU generator's numbering: layer * 16 + kind, token_embd 100000,
    // output_norm 100001); the sub-stream seed is output k of SplitMix64 seeded with seed ^ "ocr-b200"
    auto sub = [&](uint64_t k) {
        uint64_t z = (seed ^ 0x6F63722D62323030ull) + (k + 1) * 0x9E3779B97F4A7C15ull;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    cudaStream_t st = ctx->stream;
    for (int l = 0; l < cfg->n_layer; l++)
        for (int k = 0; k < 11; k++) {
            Where w;
            where(m, l, k, w);
            const uint64_t ss = sub((uint64_t)l * 16 + k);
            if (w.is_norm) launch_synth_norm(st, ss, w.n, w.norm);
            else
                launch_synth_q8_0(st, ss, sigma_w, w.rows, w.mat.cols, const_cast<uint8_t*>(w.mat.w), w.row_mul,
                                  w.row_add);
        }
    launch_synth_q8_0(st, sub(100000), sigma_e, cfg->n_vocab, cfg->dim, const_cast<uint8_t*>(m->tok.w), 1, 0);
    launch_synth_norm(st, sub(100001), cfg->dim, m->out_norm);
    derive_weights(m, st);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
        ocr_model_destroy(m);
        return cuda_fail(e, "ocr_model_synthetic");
    }
    *out = m;
    return OCR_OK;
}

ocr_status ocr_model_config(const ocr_model* m, ocr_text_cfg* out) {
    if (!m || !out) return fail(OCR_ERR_ARG, "null argument");
    *out = m->cfg;
    return OCR_OK;
}

ocr_status ocr_model_tensor_gguf(const ocr_model* m, int layer, int kind, void* out, size_t* n_bytes) {
    if (!m || !n_bytes) return fail(OCR_ERR_ARG, "null argument");
    Where w;
    if (!where(m, layer, kind, w)) return fail(OCR_ERR_ARG, "no tensor (layer " + std::to_string(layer) + ", kind " + std::to_string(kind) + ")");
    const size_t need = w.is_norm ? (size_t)w.n * 4 : (size_t)w.rows * (w.mat.cols / 32) * 34;
    if (!out) {
        *n_bytes = need;
        return OCR_OK;
    }
    if (*n_bytes < need) return fail(OCR_ERR_ARG, "output buffer too small");
    ocr_ctx* ctx = m->ctx;
    OCR_CUDA(cudaSetDevice(ctx->device));
    if (w.is_norm) {
        OCR_CUDA(cudaMemcpy(out, w.norm, need, cudaMemcpyDeviceToHost));
    } else {
        void* d = nullptr;
        OCR_CUDA(cudaMalloc(&d, need));
        launch_unpack_q8_0(ctx->stream, w.mat.w, w.rows, w.mat.cols, w.row_mul, w.row_add, (uint8_t*)d);
        cudaError_t e = cudaStreamSynchronize(ctx->stream);
        if (e == cudaSuccess) e = cudaMemcpy(out, d, need, cudaMemcpyDeviceToHost);
        cudaFree(d);
        if (e != cudaSuccess) return cuda_fail(e, "ocr_model_tensor_gguf");
    }
    *n_bytes = need;
    return OCR_OK;
}

ocr_status ocr_model_checksum(const ocr_model* m, uint64_t* out) {
    if (!m || !out) return fail(OCR_ERR_ARG, "null argument");
    std::vector<uint8_t> h(m->mem_bytes);
    OCR_CUDA(cudaSetDevice(m->ctx->device));
    OCR_CUDA(cudaStreamSynchronize(m->ctx->stream));
    OCR_CUDA(cudaMemcpy(h.data(), m->mem, m->mem_bytes, cudaMemcpyDeviceToHost));
    uint64_t x = 0xcbf29ce484222325ull;
    for (uint8_t b : h) x = (x ^ b) * 0x100000001b3ull;
    *out = x;
    return OCR_OK;
}

static void model_release(ocr_model* m) {
    if (--m->refs > 0) return;
    ocr_ctx* ctx = m->ctx;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    dfree(m->mem, m->mem_bytes, &ctx->mem_weights);
    delete m;
    ctx_release(ctx);
}

ocr_status ocr_model_destroy(ocr_model* m) {
    if (m) model_release(m);
    return OCR_OK;
}

ocr_status ocr_session_create(ocr_model* m, int n_ctx, int batch, ocr_session** out) {
    if (!m || !out) return fail(OCR_ERR_ARG, "null argument");
    const auto& c = m->cfg;
    if (n_ctx < 1 || batch < 1) return fail(OCR_ERR_ARG, "n_ctx and batch must be >= 1");
    if (n_ctx > c.n_ctx_train) return fail(OCR_ERR_ARG, std::to_string(n_ctx) + " positions asked, the model was trained on " + std::to_string(c.n_ctx_train));
    ocr_ctx* ctx = m->ctx;
    OCR_CUDA(cudaSetDevice(ctx->device));
    auto* s = new ocr_session;
    s->m = m;
    m->refs++;
    s->ctx = ctx;
    s->n_ctx = n_ctx;
    s->B = batch;
    s->qd = c.n_head * c.d_head;
    s->qkv_w = (c.n_head + 2 * c.n_kv) * c.d_head;
    s->splits = attention_splits(ctx->num_sms, batch, c.n_kv, n_ctx);
    s->n_past.assign(batch, 0);
    s->has_logits.assign(batch, 0);
    s->kv_bytes = (size_t)c.n_layer * batch * c.n_kv * n_ctx * 128 * 2;
    cudaError_t e = dalloc((void**)&s->kc, s->kv_bytes, &ctx->mem_kv);
    if (e == cudaSuccess) e = dalloc((void**)&s->vc, s->kv_bytes, &ctx->mem_kv);
    // work: rope, x, qkv, attn, g, logits, partials, counters, state
    const int lm_grid = std::max(std::max(lm_head_grid(ctx->num_sms, c.n_vocab, c.dim), sample_grid(ctx->num_sms)),
                                 bgemm_grid(ctx->num_sms, c.n_vocab));
    Planner p;
    const size_t o_rope = p.take((size_t)n_ctx * c.d_head * 4);
    const size_t o_x = p.take((size_t)batch * c.dim * 4);
    // the fused layer: the gate/up kernel sums at most MAX_ADD partials, one float4 of the row per consumer thread
    const bool fuse = c.n_kv <= MAX_ADD && c.dim <= 1024;
    const size_t o_x2 = fuse ? p.take((size_t)batch * c.dim * 4) : 0;
    const size_t o_opart = fuse ? p.take((size_t)batch * c.n_kv * c.dim * 4) : 0;
    const bool fuse_ffn = fuse && batch == 1 && m->layers[0].d_s != nullptr;
    const size_t o_dpart = fuse_ffn ? p.take((size_t)FFN_NCLU * c.dim * 4) : 0;
    // batches of more than 8 slots run their contractions on the tensor cores (with the o-projection fused into the
    // attention, whose per-head partials the FFN's operand preparation sums)
    const char* ba_env = getenv("OCR_BATTN");
    const bool ba_on = !(ba_env && ba_env[0] == '0');  // the batched attention (else the cluster kernel, fused o-proj)
    const bool tc = m->tc && batch > 8 && (ba_on || fuse);
    const size_t groups = (size_t)(batch + BG_SLOTS - 1) / BG_SLOTS;
    const size_t o_x16a = tc ? p.take(groups * x16_group_bytes(c.dim)) : 0;
    const size_t o_x16g = tc ? p.take(groups * x16_group_bytes(c.n_ff)) : 0;
    const bool battn = tc && ba_on;
    int ab_split = battn ? attn_batch_split(ctx->num_sms, batch, c.n_kv) : 1;
    const char* abs_env = getenv("OCR_AB_SPLIT");  // the attention's CTAs per (slot, kv head), for comparisons
    if (battn && abs_env && atoi(abs_env) >= 1) ab_split = std::min(AB_MAX_SPLIT, atoi(abs_env));
    const size_t o_x16o = battn ? p.take(groups * x16_group_bytes(c.n_head * c.d_head)) : 0;
    const size_t o_abp = battn && ab_split > 1
                             ? p.take((size_t)batch * c.n_kv * ab_split * (c.n_head / c.n_kv) * 132 * 4) : 0;
    const size_t o_abd = battn ? p.take((size_t)batch * c.n_kv * 4) : 0;
    // the split-K contractions' partials and tickets: the largest of the layer's matrices, per slot group
    size_t bg_floats = 0;
    int bg_tk = 0;
    if (tc) {
        const int qd = c.n_head * c.d_head, rows[4] = {qd + 2 * c.n_kv * c.d_head, c.dim, 2 * c.n_ff, c.dim},
                  cols[4] = {c.dim, qd, c.dim, c.n_ff};
        for (int i = 0; i < 4; i++) {
            bg_floats = std::max(bg_floats, bgemm_part_floats(rows[i], bgemm_ksplit(ctx->num_sms, rows[i], cols[i])));
            bg_tk = std::max(bg_tk, bgemm_tickets(rows[i]));
        }
    }
    const size_t o_bgp = tc ? p.take(groups * bg_floats * 4) : 0;
    // the norms folded into the qkv and gate|up contractions (their operand built in the kernel) when both shapes
    // allow it; OCR_NORM_IN=0 keeps the separate prep kernels
    const char* ni_env = getenv("OCR_NORM_IN");
    const int qkv_rows = c.n_head * c.d_head + 2 * c.n_kv * c.d_head;
    const bool norm_in = tc && ba_on && !(ni_env && ni_env[0] == '0') && c.dim % BG_SLOTS == 0 &&
                         bgemm_norm_in_ok(ctx->num_sms, qkv_rows, c.dim, bgemm_ksplit(ctx->num_sms, qkv_rows, c.dim)) &&
                         bgemm_norm_in_ok(ctx->num_sms, 2 * c.n_ff, c.dim, bgemm_ksplit(ctx->num_sms, 2 * c.n_ff, c.dim));
    const size_t o_ssq = norm_in ? p.take((size_t)(c.dim / 128) * batch * 4) : 0;
    const size_t o_bgt = tc ? p.take(groups * (size_t)bg_tk * 4) : 0;
    const size_t o_qkv = p.take((size_t)batch * s->qkv_w * 4);
    const size_t o_attn = p.take((size_t)batch * s->qd * 4);
    const size_t o_g = p.take((size_t)batch * c.n_ff * 4);
    const size_t o_logits = p.take((size_t)batch * c.n_vocab * 4);
    const size_t o_lmp = p.take(((size_t)batch * lm_grid * 2 + batch) * 4);
    const size_t o_lmd = p.take((size_t)(batch + 64) * 4);
    const size_t o_state = p.take((size_t)batch * 5 * 4);  // pos, len, tok, active, remaining
    if (e == cudaSuccess) e = dalloc(&s->work, p.off, &ctx->mem_work);
    if (e != cudaSuccess) {
        ocr_session_destroy(s);
        return cuda_fail(e, "ocr_session_create (device memory)");
    }
    s->work_bytes = p.off;
    char* w = (char*)s->work;
    s->rope = (float*)(w + o_rope);
    s->x = (float*)(w + o_x);
    if (fuse) {
        s->x2 = (float*)(w + o_x2);
        s->opart = (float*)(w + o_opart);
    }
    if (fuse_ffn) s->dpart = (float*)(w + o_dpart);
    if (tc) {
        s->tc = true;
        s->x16a = (uint8_t*)(w + o_x16a);
        s->x16g = (uint8_t*)(w + o_x16g);
    }
    if (tc) {
        s->bg_part = (float*)(w + o_bgp);
        s->bg_tickets = (uint32_t*)(w + o_bgt);
    }
    if (norm_in) s->ssq = (float*)(w + o_ssq);
    if (battn) {
        s->battn = true;
        s->ab_split = ab_split;
        s->x16o = (uint8_t*)(w + o_x16o);
        s->ab_part = ab_split > 1 ? (float*)(w + o_abp) : nullptr;
        s->ab_done = (uint32_t*)(w + o_abd);
    }
    s->qkv = (float*)(w + o_qkv);
    s->attn = (float*)(w + o_attn);
    s->g = (float*)(w + o_g);
    s->logits = (float*)(w + o_logits);
    s->lm_part = (float*)(w + o_lmp);
    s->lm_done = (uint32_t*)(w + o_lmd);
    s->pos = (int32_t*)(w + o_state);
    s->len = s->pos + batch;
    s->tok = s->len + batch;
    s->active = s->tok + batch;
    s->remaining = s->active + batch;
    const std::vector<float> cs = rope_table(c.rope_base, c.d_head, n_ctx);
    e = cudaMemcpyAsync(s->rope, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e == cudaSuccess) {
        ocr_status st = ensure_hist(s, 4096);
        if (st != OCR_OK) {
            ocr_session_destroy(s);
            return st;
        }
    }
    if (e != cudaSuccess) {
        ocr_session_destroy(s);
        return cuda_fail(e, "ocr_session_create (rope table)");
    }
    *out = s;
    return OCR_OK;
}

ocr_status ocr_session_destroy(ocr_session* s) {
    if (!s) return OCR_OK;
    ocr_ctx* ctx = s->ctx;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (s->gexec) cudaGraphExecDestroy(s->gexec);
    if (s->kc) dfree(s->kc, s->kv_bytes, &ctx->mem_kv);
    if (s->vc) dfree(s->vc, s->kv_bytes, &ctx->mem_kv);
    if (s->work) dfree(s->work, s->work_bytes, &ctx->mem_work);
    if (s->hist) dfree(s->hist, (size_t)s->B * s->hist_cap * 4, &ctx->mem_work);
    if (s->counts) dfree(s->counts, (size_t)s->B * s->m->cfg.n_vocab * 4, &ctx->mem_work);
    if (s->fpen) dfree(s->fpen, (size_t)s->B * s->m->cfg.n_vocab * 4, &ctx->mem_work);
    if (s->pf) dfree(s->pf, s->pf_bytes, &ctx->mem_work);
    if (s->h_ids) cudaFreeHost(s->h_ids);
    for (cudaEvent_t e : s->step_ev) cudaEventDestroy(e);
    ocr_model* m = s->m;
    delete s;
    model_release(m);
    return OCR_OK;
}

ocr_status ocr_session_n_past(const ocr_session* s, int slot, int* out) {
    if (!s || !out) return fail(OCR_ERR_ARG, "null argument");
    if (slot < 0 || slot >= s->B) return fail(OCR_ERR_ARG, "slot out of range");
    *out = s->n_past[slot];
    return OCR_OK;
}

ocr_status ocr_session_rewind(ocr_session* s, int slot, int n_past) {
    if (!s) return fail(OCR_ERR_ARG, "null argument");
    if (slot < 0 || slot >= s->B) return fail(OCR_ERR_ARG, "slot out of range");
    if (n_past < 0 || n_past > s->n_past[slot]) return fail(OCR_ERR_ARG, "rewind beyond the slot's positions");
    s->n_past[slot] = n_past;
    s->has_logits[slot] = 0;
    return OCR_OK;
}

ocr_status ocr_session_kv(const ocr_session* s, int layer, int slot, int row0, int n_rows, uint16_t* k_out,
                          uint16_t* v_out) {
    if (!s || !k_out || !v_out) return fail(OCR_ERR_ARG, "null argument");
    const auto& c = s->m->cfg;
    if (layer < 0 || layer >= c.n_layer || slot < 0 || slot >= s->B) return fail(OCR_ERR_ARG, "layer or slot out of range");
    if (row0 < 0 || n_rows < 0 || row0 + n_rows > s->n_ctx) return fail(OCR_ERR_ARG, "rows outside the cache");
    if (!n_rows) return OCR_OK;
    OCR_CUDA(cudaSetDevice(s->ctx->device));
    OCR_CUDA(cudaStreamSynchronize(s->ctx->stream));
    const size_t row_bytes = (size_t)c.n_kv * 128 * 2;
    for (int j = 0; j < c.n_kv; j++) {
        // the device's [slot][kv head][n_ctx][128] rows of head j → columns j*128 … of the host rows
        const size_t src = (((size_t)slot * c.n_kv + j) * s->n_ctx + row0) * 128;
        OCR_CUDA(cudaMemcpy2D(k_out + (size_t)j * 128, row_bytes, s->kcl(layer) + src, 256, 256, n_rows,
                              cudaMemcpyDeviceToHost));
        OCR_CUDA(cudaMemcpy2D(v_out + (size_t)j * 128, row_bytes, s->vcl(layer) + src, 256, 256, n_rows,
                              cudaMemcpyDeviceToHost));
    }
    return OCR_OK;
}

// A few rows (a prompt's tail, the bench's re-run of the last prefix row) are cheaper as decode steps of this slot
// alone — 5 matvec / attention kernels per layer per row — than through the prefill GEMMs, whose tiles are sized for
// hundreds of rows.
constexpr int SHORT_PREFILL = 4;

ocr_status prefill_short(ocr_session* s, int slot, const int32_t* ids, const float* embd, int n, float* logits_out) {
    const auto& c = s->m->cfg;
    ocr_ctx* ctx = s->ctx;
    cudaStream_t st = ctx->stream;
    std::vector<int32_t> act(s->B, 0), pos(s->B, 0), tok(s->B, -1);
    act[slot] = 1;
    OCR_CUDA(cudaMemcpyAsync(s->active, act.data(), s->B * 4, cudaMemcpyHostToDevice, st));
    for (int i = 0; i < n; i++) {
        const bool given = !ids || ids[i] < 0;
        pos[slot] = s->n_past[slot] + i;
        tok[slot] = given ? -1 : ids[i];
        if (given)
            OCR_CUDA(cudaMemcpyAsync(s->x + (size_t)slot * c.dim, embd + (size_t)i * c.dim, (size_t)c.dim * 4,
                                     cudaMemcpyDefault, st));
        OCR_CUDA(cudaMemcpyAsync(s->tok, tok.data(), s->B * 4, cudaMemcpyHostToDevice, st));
        OCR_CUDA(cudaMemcpyAsync(s->pos, pos.data(), s->B * 4, cudaMemcpyHostToDevice, st));
        record_step(s, false, 1.0f, 1, 0, 0.0f, nullptr, given);
        OCR_CUDA(cudaGetLastError());
    }
    if (logits_out)
        OCR_CUDA(cudaMemcpyAsync(logits_out, s->logits + (size_t)slot * c.n_vocab, (size_t)c.n_vocab * 4,
                                 cudaMemcpyDeviceToHost, st));
    OCR_CUDA(cudaStreamSynchronize(st));
    OCR_TRY(check_device_error(ctx));
    s->n_past[slot] += n;
    s->has_logits[slot] = 1;
    return OCR_OK;
}

ocr_status ocr_prefill(ocr_session* s, int slot, const int32_t* ids, const float* embd, int n, float* logits_out) {
    if (!s) return fail(OCR_ERR_ARG, "null session");
    if (slot < 0 || slot >= s->B) return fail(OCR_ERR_ARG, "slot out of range");
    if (n <= 0) return fail(OCR_ERR_ARG, "empty prompt");
    const auto& c = s->m->cfg;
    ocr_ctx* ctx = s->ctx;
    if (s->n_past[slot] + n > s->n_ctx)
        return fail(OCR_ERR_STATE, std::to_string(s->n_past[slot]) + " + " + std::to_string(n) + " positions overflow the session's " + std::to_string(s->n_ctx));
    bool any_embd = false;
    for (int i = 0; i < n; i++) {
        if (ids && ids[i] >= c.n_vocab) return fail(OCR_ERR_ARG, "token " + std::to_string(ids[i]) + " is outside the vocabulary");
        if (!ids || ids[i] < 0) any_embd = true;
    }
    if (any_embd && !embd) return fail(OCR_ERR_ARG, "embedding rows asked but embd is null");
    OCR_CUDA(cudaSetDevice(ctx->device));
    if (n <= SHORT_PREFILL) return prefill_short(s, slot, ids, embd, n, logits_out);
    OCR_TRY(ensure_prefill(s, n));
    cudaStream_t st = ctx->stream;
    float* x = (float*)s->pf;
    float* h = x + (size_t)n * c.dim;
    float* qkv = h + (size_t)n * c.dim;
    float* a = qkv + (size_t)n * s->qkv_w;
    float* g = a + (size_t)n * s->qd;
    int32_t* d_ids = (int32_t*)(g + (size_t)n * c.n_ff);
    std::vector<int32_t> hid(n);
    for (int i = 0; i < n; i++) hid[i] = ids ? ids[i] : -1;
    if (any_embd) OCR_CUDA(cudaMemcpyAsync(x, embd, (size_t)n * c.dim * 4, cudaMemcpyDefault, st));
    OCR_CUDA(cudaMemcpyAsync(d_ids, hid.data(), (size_t)n * 4, cudaMemcpyHostToDevice, st));
    launch_embed_rows(st, d_ids, n, s->m->tok, x);
    const int pos0 = s->n_past[slot];
    const float scale = 1.0f / sqrtf((float)c.d_head);
    // the tensor-core contractions (k_bgemm.cu) take the rows in groups of 32 like decode slots; the operands after
    // the ids, 256-B aligned
    const bool tc = s->m->tc;
    // the causal attention on the tensor cores with the contractions (OCR_PF_ATTN=0: the f32 kernel)
    const char* pfa_env = getenv("OCR_PF_ATTN");
    const bool pf_attn_tc = tc && c.d_head == 128 && !(pfa_env && pfa_env[0] == '0');
    uint8_t* x16a = (uint8_t*)(((uintptr_t)(d_ids + n) + 255) & ~(uintptr_t)255);
    uint8_t* x16o = x16a + prefill_x16_bytes(s, n, c.dim);
    uint8_t* x16g = x16o + prefill_x16_bytes(s, n, s->qd);
    auto prep = [&](const float* src, int K, const float* nw, uint8_t* x16) {
        PrepArgs p;
        p.x = src;
        p.x_stride = K;
        p.nw = nw;
        p.eps = c.eps;
        p.K = K;
        p.nb = n;
        p.x16 = x16;
        p.err = ctx->d_err;
        launch_xprep(st, p, false);
    };
    auto gemm = [&](const QMat& w, const BgMaps& bq, const uint8_t* x16, int mode, float* y, int y_stride,
                    uint8_t* y16) {
        BgArgs g;
        g.w = w;
        g.x16 = x16;
        g.mode = mode;
        g.y = y;
        g.y_stride = y_stride;
        g.y16 = y16;
        g.nb = n;
        g.wide = 1;  // (three groups of 32 rows per CTA when there are three or more)
        g.err = ctx->d_err;
        launch_bgemm(st, g, bq, ctx->num_sms, false);
    };
    for (int l = 0; l < c.n_layer; l++) {
        const LayerW& L = s->m->layers[l];
        __half* kc = s->kcl(l) + (size_t)slot * c.n_kv * s->n_ctx * 128;
        __half* vc = s->vcl(l) + (size_t)slot * c.n_kv * s->n_ctx * 128;
        if (tc) {
            prep(x, c.dim, L.attn_norm, x16a);
            gemm(L.qkv, L.bq_qkv, x16a, MV_STORE, qkv, s->qkv_w, nullptr);
            launch_qk_norm_rope_store(st, qkv, n, c.n_head, c.n_kv, L.q_norm, L.k_norm, s->rope, pos0, c.eps, kc, vc,
                                      s->n_ctx);
            if (pf_attn_tc)
                launch_attention_prefill_tc(st, qkv, n, c.n_head, c.n_kv, kc, vc, s->n_ctx, pos0, scale, a, ctx->d_err);
            else
                launch_attention_prefill(st, qkv, n, c.n_head, c.n_kv, kc, vc, s->n_ctx, pos0, scale, a);
            prep(a, s->qd, nullptr, x16o);
            gemm(L.o, L.bq_o, x16o, MV_ADD, x, c.dim, nullptr);
            prep(x, c.dim, L.ffn_norm, x16a);
            gemm(L.gu, L.bq_gu, x16a, MV_SWIGLU, nullptr, 0, x16g);
            gemm(L.down, L.bq_down, x16g, MV_ADD, x, c.dim, nullptr);
            continue;
        }
        launch_rmsnorm_rows(st, x, L.attn_norm, h, n, c.dim, c.eps);
        launch_gemm_q8_0(st, h, n, L.qkv, qkv, 0, 0);
        launch_qk_norm_rope_store(st, qkv, n, c.n_head, c.n_kv, L.q_norm, L.k_norm, s->rope, pos0, c.eps, kc, vc, s->n_ctx);
        launch_attention_prefill(st, qkv, n, c.n_head, c.n_kv, kc, vc, s->n_ctx, pos0, scale, a);
        launch_gemm_q8_0(st, a, n, L.o, x, 1, 0);
        launch_rmsnorm_rows(st, x, L.ffn_norm, h, n, c.dim, c.eps);
        launch_gemm_q8_0(st, h, n, L.gu, g, 0, 1);
        launch_gemm_q8_0(st, g, n, L.down, x, 1, 0);
    }
    MvArgs lm;
    lm.w = s->m->tok;
    lm.x = x + (size_t)(n - 1) * c.dim;
    lm.x_stride = c.dim;
    lm.nw = s->m->out_norm;
    lm.eps = c.eps;
    lm.nb = 1;
    lm.mode = MV_LMHEAD;
    lm.y = s->logits + (size_t)slot * c.n_vocab;
    lm.err = ctx->d_err;
    launch_matvec(st, lm, ctx->num_sms, false);
    OCR_CUDA(cudaGetLastError());
    if (logits_out)
        OCR_CUDA(cudaMemcpyAsync(logits_out, s->logits + (size_t)slot * c.n_vocab, (size_t)c.n_vocab * 4, cudaMemcpyDeviceToHost, st));
    OCR_CUDA(cudaStreamSynchronize(st));
    OCR_TRY(check_device_error(ctx));
    s->n_past[slot] += n;
    s->has_logits[slot] = 1;
    return OCR_OK;
}

ocr_status ocr_step(ocr_session* s, const int32_t* tok, float* logits_out) {
    if (!s || !tok) return fail(OCR_ERR_ARG, "null argument");
    const auto& c = s->m->cfg;
    ocr_ctx* ctx = s->ctx;
    std::vector<int32_t> act(s->B), pos(s->B);
    for (int b = 0; b < s->B; b++) {
        if (tok[b] >= c.n_vocab) return fail(OCR_ERR_ARG, "token " + std::to_string(tok[b]) + " is outside the vocabulary");
        act[b] = tok[b] >= 0;
        pos[b] = s->n_past[b];
        if (act[b] && s->n_past[b] + 1 > s->n_ctx) return fail(OCR_ERR_STATE, "slot " + std::to_string(b) + ": the session is full");
    }
    OCR_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    OCR_CUDA(cudaMemcpyAsync(s->tok, tok, s->B * 4, cudaMemcpyHostToDevice, st));
    OCR_CUDA(cudaMemcpyAsync(s->active, act.data(), s->B * 4, cudaMemcpyHostToDevice, st));
    OCR_CUDA(cudaMemcpyAsync(s->pos, pos.data(), s->B * 4, cudaMemcpyHostToDevice, st));
    record_step(s, false, 1.0f, 1, 0, 0.0f);
    OCR_CUDA(cudaGetLastError());
    if (logits_out)
        OCR_CUDA(cudaMemcpyAsync(logits_out, s->logits, (size_t)s->B * c.n_vocab * 4, cudaMemcpyDeviceToHost, st));
    OCR_CUDA(cudaStreamSynchronize(st));
    OCR_TRY(check_device_error(ctx));
    for (int b = 0; b < s->B; b++)
        if (act[b]) {
            s->n_past[b] += 1;
            s->has_logits[b] = 1;
        }
    return OCR_OK;
}

ocr_status ocr_step_embd(ocr_session* s, const int32_t* active, const float* embd, float* logits_out) {
    if (!s || !active || !embd) return fail(OCR_ERR_ARG, "null argument");
    const auto& c = s->m->cfg;
    ocr_ctx* ctx = s->ctx;
    std::vector<int32_t> act(s->B), pos(s->B), tok(s->B, -1);
    for (int b = 0; b < s->B; b++) {
        act[b] = active[b] != 0;
        pos[b] = s->n_past[b];
        if (act[b] && s->n_past[b] + 1 > s->n_ctx) return fail(OCR_ERR_STATE, "slot " + std::to_string(b) + ": the session is full");
    }
    OCR_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    // the active slots' rows into the residual (an inactive slot's row is not read)
    for (int b = 0; b < s->B; b++)
        if (act[b])
            OCR_CUDA(cudaMemcpyAsync(s->x + (size_t)b * c.dim, embd + (size_t)b * c.dim, (size_t)c.dim * 4,
                                     cudaMemcpyHostToDevice, st));
    OCR_CUDA(cudaMemcpyAsync(s->tok, tok.data(), s->B * 4, cudaMemcpyHostToDevice, st));
    OCR_CUDA(cudaMemcpyAsync(s->active, act.data(), s->B * 4, cudaMemcpyHostToDevice, st));
    OCR_CUDA(cudaMemcpyAsync(s->pos, pos.data(), s->B * 4, cudaMemcpyHostToDevice, st));
    record_step(s, false, 1.0f, 1, 0, 0.0f, nullptr, true);
    OCR_CUDA(cudaGetLastError());
    if (logits_out)
        OCR_CUDA(cudaMemcpyAsync(logits_out, s->logits, (size_t)s->B * c.n_vocab * 4, cudaMemcpyDeviceToHost, st));
    OCR_CUDA(cudaStreamSynchronize(st));
    OCR_TRY(check_device_error(ctx));
    for (int b = 0; b < s->B; b++)
        if (act[b]) {
            s->n_past[b] += 1;
            s->has_logits[b] = 1;
        }
    return OCR_OK;
}

ocr_status ocr_profile_step(ocr_session* s, const int32_t* tok, ocr_kernel_time* out, int cap, int* n) {
    if (!s || !tok || !out || !n) return fail(OCR_ERR_ARG, "null argument");
    const auto& c = s->m->cfg;
    ocr_ctx* ctx = s->ctx;
    std::vector<int32_t> act(s->B), pos(s->B);
    Prof prof;
    for (int b = 0; b < s->B; b++) {
        if (tok[b] >= c.n_vocab) return fail(OCR_ERR_ARG, "token " + std::to_string(tok[b]) + " is outside the vocabulary");
        act[b] = tok[b] >= 0;
        pos[b] = s->n_past[b];
        if (act[b] && s->n_past[b] + 1 > s->n_ctx) return fail(OCR_ERR_STATE, "slot " + std::to_string(b) + ": the session is full");
        if (act[b]) prof.pos.push_back(s->n_past[b]);
    }
    OCR_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    OCR_CUDA(cudaMemcpyAsync(s->tok, tok, s->B * 4, cudaMemcpyHostToDevice, st));
    OCR_CUDA(cudaMemcpyAsync(s->active, act.data(), s->B * 4, cudaMemcpyHostToDevice, st));
    OCR_CUDA(cudaMemcpyAsync(s->pos, pos.data(), s->B * 4, cudaMemcpyHostToDevice, st));
    prof.st = st;
    cudaEvent_t e0;
    OCR_CUDA(cudaEventCreate(&e0));
    OCR_CUDA(cudaEventRecord(e0, st));
    record_step(s, false, 1.0f, 1, 0, 0.0f, &prof);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaEvent_t prev = e0;
    const int k = std::min<int>(cap, (int)prof.rec.size());
    for (int i = 0; i < (int)prof.rec.size(); i++) {
        float ms = 0.0f;
        if (e == cudaSuccess) cudaEventElapsedTime(&ms, prev, prof.ev[i]);
        prof.rec[i].us = ms * 1000.0f;
        if (i < k) out[i] = prof.rec[i];
        prev = prof.ev[i];
    }
    for (cudaEvent_t ev : prof.ev) cudaEventDestroy(ev);
    cudaEventDestroy(e0);
    if (e != cudaSuccess) return cuda_fail(e, "ocr_profile_step");
    OCR_TRY(check_device_error(ctx));
    for (int b = 0; b < s->B; b++)
        if (act[b]) {
            s->n_past[b] += 1;
            s->has_logits[b] = 1;
        }
    *n = k;
    return OCR_OK;
}

ocr_status ocr_timeline_step(ocr_session* s, const int32_t* tok, int reps, ocr_kernel_time* out, int cap, int* n) {
    if (!s || !tok || !out || !n) return fail(OCR_ERR_ARG, "null argument");
    if (reps < 2 || reps > 16 || cap < 1) return fail(OCR_ERR_ARG, "reps must be 2..16 and cap at least 1");
    const auto& c = s->m->cfg;
    ocr_ctx* ctx = s->ctx;
    std::vector<int32_t> act(s->B), pos(s->B);
    Prof prof;
    for (int b = 0; b < s->B; b++) {
        if (tok[b] >= c.n_vocab) return fail(OCR_ERR_ARG, "token " + std::to_string(tok[b]) + " is outside the vocabulary");
        act[b] = tok[b] >= 0;
        pos[b] = s->n_past[b];
        if (act[b] && s->n_past[b] + 1 > s->n_ctx) return fail(OCR_ERR_STATE, "slot " + std::to_string(b) + ": the session is full");
        if (act[b]) prof.pos.push_back(s->n_past[b]);
    }
    OCR_CUDA(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->stream;
    const int per_rep = 8 * c.n_layer + 8;  // an upper bound on the launches of one step (slots beyond it: an error)
    const size_t slots = (size_t)reps * per_rep;
    TlSlot* d_tl = nullptr;
    OCR_CUDA(cudaMalloc((void**)&d_tl, slots * sizeof(TlSlot)));
    cudaError_t e = cudaMemsetAsync(d_tl, 0, slots * sizeof(TlSlot), st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s->tok, tok, s->B * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s->active, act.data(), s->B * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s->pos, pos.data(), s->B * 4, cudaMemcpyHostToDevice, st);
    prof.st = st;
    prof.tl = d_tl;
    prof.tl_cap = (int)slots;
    // the step `reps` times back to back in one graph, chained as the decode's graph chains its launches (each step's
    // first launch waits for the whole step before it, as between two replays of the decode's graph)
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    if (e == cudaSuccess) e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
    if (e == cudaSuccess) {
        for (int r = 0; r < reps; r++) record_step(s, false, 1.0f, 1, 0, 0.0f, &prof);
        e = cudaStreamEndCapture(st, &graph);
    }
    if (e == cudaSuccess) e = cudaGraphInstantiate(&exec, graph, 0);
    if (e == cudaSuccess) e = cudaGraphLaunch(exec, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    std::vector<TlSlot> h(prof.rec.size());
    if (e == cudaSuccess && (int)prof.rec.size() > prof.tl_cap) e = cudaErrorInvalidValue;
    if (e == cudaSuccess) e = cudaMemcpy(h.data(), d_tl, h.size() * sizeof(TlSlot), cudaMemcpyDeviceToHost);
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    cudaFree(d_tl);
    if (e != cudaSuccess) return cuda_fail(e, "ocr_timeline_step");
    OCR_TRY(check_device_error(ctx));
    // the last repetition: each launch's in-chain time (its latest CTA end less the previous launch's)
    const int per = (int)prof.rec.size() / reps, first = (reps - 1) * per;
    const int k = std::min(cap, per);
    for (int i = 0; i < k; i++) {
        const int g = first + i;
        ocr_kernel_time r = prof.rec[g];
        const unsigned long long prev = h[g - 1].end, end = h[g].end;
        r.us = (h[g].end && prev && end > prev) ? (float)((double)(end - prev) * 1e-3) : 0.0f;
        out[i] = r;
    }
    for (int b = 0; b < s->B; b++)
        if (act[b]) {
            s->n_past[b] += 1;
            s->has_logits[b] = 1;
        }
    *n = k;
    return OCR_OK;
}

ocr_status ocr_decode(ocr_session* s, int slot, const ocr_sampler_cfg* cfg, const int32_t* history, int n_hist,
                      ocr_token_cb on_token, void* user, int32_t* ids_out, int* n_out) {
    if (!s || !ids_out) return fail(OCR_ERR_ARG, "null argument");
    if (slot < 0 || slot >= s->B) return fail(OCR_ERR_ARG, "slot out of range");
    OCR_CUDA(cudaSetDevice(s->ctx->device));
    int n = 0;
    OCR_TRY(decode_slots(s, slot, 1, cfg, history, n_hist, on_token, user, ids_out, &n));
    if (n_out) *n_out = n;
    return OCR_OK;
}

ocr_status ocr_decode_batch(ocr_session* s, const ocr_sampler_cfg* cfg, const int32_t* history, int n_hist,
                            int32_t* ids_out) {
    if (!s || !ids_out) return fail(OCR_ERR_ARG, "null argument");
    OCR_CUDA(cudaSetDevice(s->ctx->device));
    return decode_slots(s, 0, s->B, cfg, history, n_hist, nullptr, nullptr, ids_out, nullptr);
}

// The page engine: Engine::read_text's per-page loop (app/crates/ocr-wgpu/src/engine.rs:447-524) over many pages at
// once. The session's slots hold pages at different stages: between chunks of decode steps, every free slot takes the
// next page (prefill of its rows, the window seeded, choice 0 from the prefill's logits), and each page's token budget
// counts down on the device, its slot going idle after its last choice — so one captured step serves any mix of pages.
ocr_status ocr_read_pages(ocr_session* s, const ocr_sampler_cfg* cfg, int chunk, const ocr_page_io* io) {
    if (!s || !io || !io->next || !io->done) return fail(OCR_ERR_ARG, "null argument");
    OCR_TRY(check_sampler(cfg));
    if (chunk < 1 || chunk > 4096) return fail(OCR_ERR_ARG, "chunk must be in [1, 4096]");
    const auto& c = s->m->cfg;
    ocr_ctx* ctx = s->ctx;
    cudaStream_t st = ctx->stream;
    const int B = s->B;
    OCR_CUDA(cudaSetDevice(ctx->device));
    OCR_TRY(ensure_hist(s, cfg->window + cfg->max_new));
    if (cfg->fp > 0.0f) OCR_TRY(ensure_counts(s));
    const int cap = s->hist_cap;
    // host mirrors of the device state block: pos, len, tok, active, remaining (5 x B ints, contiguous)
    std::vector<int32_t> mir((size_t)5 * B, 0);
    auto M = [&](int field, int b) -> int32_t& { return mir[(size_t)field * B + b]; };
    auto upload = [&]() -> ocr_status {
        OCR_CUDA(cudaMemcpyAsync(s->pos, mir.data(), mir.size() * 4, cudaMemcpyHostToDevice, st));
        return OCR_OK;
    };
    auto readback = [&]() -> ocr_status {
        OCR_CUDA(cudaMemcpyAsync(mir.data(), s->pos, mir.size() * 4, cudaMemcpyDeviceToHost, st));
        OCR_CUDA(cudaStreamSynchronize(st));
        return check_device_error(ctx);
    };
    struct Slot {
        bool busy = false;
        ocr_page pg{};
        int seed = 0, made = 0;
    };
    std::vector<Slot> sl(B);
    for (int b = 0; b < B; b++) M(0, b) = s->n_past[b];
    OCR_TRY(upload());  // every slot idle
    // a page's ids so far, from the slot's history, to the caller's buffer
    auto collect = [&](int b) -> ocr_status {
        Slot& x = sl[b];
        const int n = M(1, b) - x.seed - x.made;
        if (n < 0 || x.made + n > x.pg.max_new)
            return fail(OCR_ERR_DEVICE, "page " + std::to_string(x.pg.id) + ": the slot's history holds " +
                                            std::to_string(x.made + n) + " choices, its budget is " +
                                            std::to_string(x.pg.max_new));
        if (n > 0) {
            OCR_CUDA(cudaMemcpy(x.pg.ids_out + x.made, s->hist + (size_t)b * cap + x.seed + x.made, (size_t)n * 4,
                                cudaMemcpyDeviceToHost));
            x.made += n;
        }
        return OCR_OK;
    };
    bool more = true, stop = false;
    ocr_status rc = OCR_OK;
    auto begin = [&](int b, const ocr_page& pg) -> ocr_status {
        if (pg.n_rows < 1 || pg.max_new < 1 || pg.max_new > cfg->max_new || !pg.ids_out || pg.n_hist < 0 ||
            (pg.n_hist > 0 && !pg.history))
            return fail(OCR_ERR_ARG, "page " + std::to_string(pg.id) + ": bad rows, budget, history or output");
        if (pg.n_rows + pg.max_new - 1 > s->n_ctx)
            return fail(OCR_ERR_STATE, "page " + std::to_string(pg.id) + ": " + std::to_string(pg.n_rows) + " rows + " +
                                           std::to_string(pg.max_new) + " tokens overflow the session's " +
                                           std::to_string(s->n_ctx));
        const int seed = std::min(pg.n_hist, cfg->window);
        for (int i = pg.n_hist - seed; i < pg.n_hist; i++)
            if (pg.history[i] < 0 || pg.history[i] >= c.n_vocab)
                return fail(OCR_ERR_ARG, "page " + std::to_string(pg.id) + ": history token outside the vocabulary");
        s->n_past[b] = 0;
        s->has_logits[b] = 0;
        OCR_TRY(ocr_prefill(s, b, pg.ids, pg.embd, pg.n_rows, nullptr));
        // (a prefill of a few rows runs as a step of this slot alone and rewrites every slot's state: restore it)
        M(0, b) = s->n_past[b];
        M(1, b) = seed;
        M(3, b) = 1;
        M(4, b) = pg.max_new - 1;
        s->pages = false;  // choice 0 spends no budget
        OCR_TRY(upload());
        OCR_CUDA(cudaMemcpyAsync(s->hist + (size_t)b * cap, pg.history + (pg.n_hist - seed), (size_t)seed * 4,
                                 cudaMemcpyHostToDevice, st));
        if (cfg->fp > 0.0f) {
            OCR_CUDA(cudaMemsetAsync(s->counts + (size_t)b * c.n_vocab, 0, (size_t)c.n_vocab * 4, st));
            OCR_CUDA(cudaMemsetAsync(s->fpen + (size_t)b * c.n_vocab, 0, (size_t)c.n_vocab * 4, st));
        }
        LmArgs sa = sampler_args(s, cfg);
        launch_sample(st, s->logits, c.n_vocab, c.n_vocab, sa, ctx->num_sms, b, 1);
        OCR_CUDA(cudaGetLastError());
        s->pages = true;
        OCR_TRY(readback());
        Slot& x = sl[b];
        x.busy = true;
        x.pg = pg;
        x.seed = seed;
        x.made = 0;
        if (pg.max_new == 1) {  // choice 0 was the page's only token
            M(3, b) = 0;
            OCR_TRY(upload());
        }
        return OCR_OK;
    };
    // a finished page goes back to the caller and frees its slot
    auto finish = [&](int b) -> ocr_status {
        Slot& x = sl[b];
        OCR_TRY(collect(b));
        x.pg.n_out = x.made;
        x.busy = false;
        if (!io->done(io->user, &x.pg)) stop = true;
        return OCR_OK;
    };
    s->pages = true;
    bool captured = false;
    while (rc == OCR_OK && !stop) {
        for (int b = 0; b < B && more && rc == OCR_OK && !stop; b++) {
            if (sl[b].busy) continue;
            ocr_page pg{};
            if (!io->next(io->user, &pg)) {
                more = false;
                break;
            }
            rc = begin(b, pg);
            if (rc == OCR_OK && M(3, b) == 0) rc = finish(b);
        }
        if (rc != OCR_OK || stop) break;
        int busy = 0, steps = 0;
        for (int b = 0; b < B; b++)
            if (sl[b].busy) {
                busy++;
                steps = std::max(steps, M(4, b));
            }
        if (!busy) break;
        steps = std::min(steps, chunk);
        // the chunk: the captured step, replayed (slots whose budget runs out go idle on the device); the first step
        // ever runs eagerly, settling every launcher's one-time setup before the capture
        int i = 0;
        if (!captured) {
            record_step(s, true, cfg->rp, cfg->window, cfg->fp > 0.0f ? 1 : 0, cfg->fp);
            const cudaError_t e = cudaGetLastError();
            if (e != cudaSuccess) rc = cuda_fail(e, "page step");
            i = 1;
            captured = true;
        }
        if (rc == OCR_OK && i < steps) rc = capture_graph(s, cfg);
        for (; i < steps && rc == OCR_OK; i++) {
            const cudaError_t e = cudaGraphLaunch(s->gexec, st);
            if (e != cudaSuccess) rc = cuda_fail(e, "cudaGraphLaunch(page step)");
        }
        if (rc == OCR_OK) rc = readback();
        for (int b = 0; b < B && rc == OCR_OK; b++) {
            if (!sl[b].busy) continue;
            s->n_past[b] = M(0, b);
            rc = M(3, b) == 0 ? finish(b) : collect(b);
        }
    }
    s->pages = false;
    // every slot idle again, positions as the pages left them
    for (int b = 0; b < B; b++) {
        M(3, b) = 0;
        s->has_logits[b] = 0;
    }
    if (rc == OCR_OK) rc = upload();
    if (rc == OCR_OK) OCR_CUDA(cudaStreamSynchronize(st));
    return rc;
}

ocr_status ocr_sample_logits(ocr_ctx* ctx, const float* d_logits, int n_vocab, const ocr_sampler_cfg* cfg,
                             const int32_t* history, int n_hist, const int32_t* count_tok, const uint32_t* count_n,
                             int n_counts, int32_t* tok) {
    if (!ctx || !d_logits || !cfg || !tok) return fail(OCR_ERR_ARG, "null argument");
    if (cfg->rp != 1.0f && !(std::isnormal(cfg->rp) && cfg->rp > 0.0f))
        return fail(OCR_ERR_ARG, "the repetition penalty is no positive normal f32");
    if (cfg->window < 1) return fail(OCR_ERR_ARG, "repetition window must be >= 1");
    if (n_vocab < 1 || n_hist < 0 || n_counts < 0) return fail(OCR_ERR_ARG, "bad sizes");
    for (int i = 0; i < n_hist; i++)
        if (history[i] < 0 || history[i] >= n_vocab) return fail(OCR_ERR_ARG, "history token " + std::to_string(history[i]) + " is outside the vocabulary");
    const bool use_fp = cfg->fp > 0.0f && n_counts > 0;
    for (int i = 0; use_fp && i < n_counts; i++)
        if (count_tok[i] < 0 || count_tok[i] >= n_vocab) return fail(OCR_ERR_ARG, "count token outside the vocabulary");
    OCR_CUDA(cudaSetDevice(ctx->device));
    const int grid = sample_grid(ctx->num_sms);
    const size_t o_part = 0, o_done = ((size_t)grid * 2 + 1) * 4 + 256, o_state = o_done + 256,
                 o_hist = o_state + 256, o_counts = o_hist + ((size_t)n_hist + 1) * 4 + 256,
                 o_fpen = o_counts + (use_fp ? (size_t)n_vocab * 4 + 256 : 0),
                 total = o_fpen + (use_fp ? (size_t)n_vocab * 4 : 0) + 256;
    OCR_TRY(ensure_op_scratch(ctx, total));
    char* w = (char*)ctx->op_scratch;
    cudaStream_t st = ctx->stream;
    int32_t state[2] = {n_hist, 0};
    OCR_CUDA(cudaMemcpyAsync(w + o_state, state, 8, cudaMemcpyHostToDevice, st));
    if (n_hist) OCR_CUDA(cudaMemcpyAsync(w + o_hist, history, (size_t)n_hist * 4, cudaMemcpyHostToDevice, st));
    OCR_CUDA(cudaMemsetAsync(w + o_done, 0, 4, st));
    std::vector<uint32_t> hc;
    std::vector<float> hf;
    if (use_fp) {
        hc.assign(n_vocab, 0);
        hf.assign(n_vocab, 0.0f);
        for (int i = 0; i < n_counts; i++) {
            hc[count_tok[i]] = count_n[i];
            hf[count_tok[i]] = cfg->fp * (float)count_n[i];
        }
        OCR_CUDA(cudaMemcpyAsync(w + o_counts, hc.data(), (size_t)n_vocab * 4, cudaMemcpyHostToDevice, st));
        OCR_CUDA(cudaMemcpyAsync(w + o_fpen, hf.data(), (size_t)n_vocab * 4, cudaMemcpyHostToDevice, st));
    }
    LmArgs a;
    a.nb = 1;
    a.sample = 1;
    a.rp = cfg->rp;
    a.window = cfg->window;
    a.use_fp = use_fp ? 1 : 0;
    a.fp = cfg->fp;
    a.hist = (int32_t*)(w + o_hist);
    a.hist_cap = n_hist + 1;
    a.len = (int32_t*)(w + o_state);
    a.tok = (int32_t*)(w + o_state) + 1;
    a.counts = use_fp ? (uint32_t*)(w + o_counts) : nullptr;
    a.fpen = use_fp ? (float*)(w + o_fpen) : nullptr;
    a.part = (float*)(w + o_part);
    a.done = (uint32_t*)(w + o_done);
    a.err = ctx->d_err;
    launch_sample(st, d_logits, n_vocab, n_vocab, a, ctx->num_sms, 0, 1);
    OCR_CUDA(cudaGetLastError());
    OCR_CUDA(cudaMemcpyAsync(state, w + o_state, 8, cudaMemcpyDeviceToHost, st));
    OCR_CUDA(cudaStreamSynchronize(st));
    OCR_TRY(check_device_error(ctx));
    *tok = state[1];
    return OCR_OK;
}

int ocr_q8_row_bytes(int cols) { return cols > 0 && cols % 32 == 0 ? q8_stride(cols) : 0; }

ocr_status ocr_op_repack_q8_0(ocr_ctx* ctx, const void* d_blocks, int rows, int cols, uint8_t* d_rows) {
    if (!ctx || !d_blocks || !d_rows) return fail(OCR_ERR_ARG, "null argument");
    if (rows < 1 || cols < 32 || cols % 32) return fail(OCR_ERR_ARG, "rows >= 1, cols a positive multiple of 32");
    if (((uintptr_t)d_blocks & 1) || ((uintptr_t)d_rows & 15))
        return fail(OCR_ERR_ARG, "alignment: blocks 2 B, rows 16 B");
    OCR_CUDA(cudaSetDevice(ctx->device));
    launch_repack_q8_0(ctx->stream, (const uint8_t*)d_blocks, rows, cols, d_rows, 1, 0);
    OCR_CUDA(cudaGetLastError());
    return OCR_OK;
}

ocr_status ocr_op_matvec_q8_0(ocr_ctx* ctx, const uint8_t* d_w, int rows, int cols, const float* d_x,
                              const float* d_norm_w, float eps, int nb, float* d_y, int accumulate) {
    if (!ctx || !d_w || !d_x || !d_y) return fail(OCR_ERR_ARG, "null argument");
    if (rows < 1 || cols < 32 || cols % 32 || nb < 1) return fail(OCR_ERR_ARG, "bad shape");
    if ((uintptr_t)d_w & 15) return fail(OCR_ERR_ARG, "the rows must start 16-B aligned");
    OCR_CUDA(cudaSetDevice(ctx->device));
    if (nb > 8 && bgemm_shape_ok(rows, cols)) {
        // a batch: the tensor-core contraction (operand prep, then k_bgemm) — the decode step's batched path
        QMat w;
        w.w = d_w;
        w.rows = rows;
        w.cols = cols;
        w.stride = q8_stride(cols);
        const size_t groups = (size_t)(nb + BG_SLOTS - 1) / BG_SLOTS;
        const int ksplit = bgemm_ksplit(ctx->num_sms, rows, cols);
        const size_t xb = groups * x16_group_bytes(cols), pb = groups * bgemm_part_floats(rows, ksplit) * 4,
                     tb = (groups * (size_t)bgemm_tickets(rows) * 4 + 255) / 256 * 256, wb = bgemm_tiled_bytes(rows, cols);
        OCR_TRY(ensure_op_scratch(ctx, xb + pb + tb + wb));
        OCR_CUDA(cudaMemsetAsync((char*)ctx->op_scratch + xb + pb, 0, tb, ctx->stream));
        // the matrix's tile-major copy, in the scratch
        BgMaps maps;
        maps.tiles = (const uint8_t*)ctx->op_scratch + xb + pb + tb;
        launch_tile_q8_0(ctx->stream, w, const_cast<uint8_t*>(maps.tiles));
        PrepArgs p;
        p.x = d_x;
        p.x_stride = cols;
        p.nw = d_norm_w;
        p.eps = eps;
        p.K = cols;
        p.nb = nb;
        p.x16 = (uint8_t*)ctx->op_scratch;
        p.err = ctx->d_err;
        launch_xprep(ctx->stream, p, false);
        BgArgs g;
        g.w = w;
        g.x16 = (const uint8_t*)ctx->op_scratch;
        g.mode = accumulate ? MV_ADD : MV_STORE;
        g.y = d_y;
        g.y_stride = rows;
        g.nb = nb;
        g.err = ctx->d_err;
        g.ksplit = ksplit;
        g.part = (float*)((char*)ctx->op_scratch + xb);
        g.tickets = (uint32_t*)((char*)ctx->op_scratch + xb + pb);
        launch_bgemm(ctx->stream, g, maps, ctx->num_sms, false);
        OCR_CUDA(cudaGetLastError());
        return OCR_OK;
    }
    if ((size_t)((cols + 511) / 512) * 512 * 4 * std::min(nb, 8) > 96 * 1024)
        return fail(OCR_ERR_ARG, "nb x cols too large for the staged activations");
    MvArgs a;
    a.w.w = d_w;
    a.w.rows = rows;
    a.w.cols = cols;
    a.w.stride = q8_stride(cols);
    a.x = d_x;
    a.x_stride = cols;
    a.nw = d_norm_w;
    a.eps = eps;
    a.y = d_y;
    a.y_stride = rows;
    a.mode = accumulate ? MV_ADD : MV_STORE;
    a.nb = nb;
    a.err = ctx->d_err;
    launch_matvec(ctx->stream, a, ctx->num_sms, false);
    OCR_CUDA(cudaGetLastError());
    return OCR_OK;
}

ocr_status ocr_op_lm_head_sample(ocr_ctx* ctx, const uint8_t* d_w, int n_vocab, int dim, const float* d_x,
                                 const float* d_norm_w, float eps, float rp, int window, int32_t* d_hist,
                                 int32_t* d_len, int32_t* d_tok, float* d_logits) {
    if (!ctx || !d_w || !d_x || !d_hist || !d_len || !d_tok) return fail(OCR_ERR_ARG, "null argument");
    if (n_vocab < 1 || dim < 32 || dim % 32) return fail(OCR_ERR_ARG, "bad shape");
    if ((uintptr_t)d_w & 15) return fail(OCR_ERR_ARG, "the rows must start 16-B aligned");
    if (rp != 1.0f && !(std::isnormal(rp) && rp > 0.0f)) return fail(OCR_ERR_ARG, "the repetition penalty is no positive normal f32");
    if (window < 1) return fail(OCR_ERR_ARG, "repetition window must be >= 1");
    OCR_CUDA(cudaSetDevice(ctx->device));
    const int grid = lm_head_grid(ctx->num_sms, n_vocab, dim);
    const size_t o_done = ((size_t)grid * 2 + 1) * 4 + 256;
    OCR_TRY(ensure_op_scratch(ctx, o_done + 256));
    char* w = (char*)ctx->op_scratch;
    MvArgs a;
    a.w.w = d_w;
    a.w.rows = n_vocab;
    a.w.cols = dim;
    a.w.stride = q8_stride(dim);
    a.x = d_x;
    a.x_stride = dim;
    a.nw = d_norm_w;
    a.eps = eps;
    a.nb = 1;
    a.mode = MV_LMHEAD;
    a.y = d_logits;
    a.err = ctx->d_err;
    a.lm.sample = 1;
    a.lm.rp = rp;
    a.lm.window = window;
    a.lm.hist = d_hist;
    a.lm.hist_cap = 1 << 30;
    a.lm.len = d_len;
    a.lm.tok = d_tok;
    a.lm.part = (float*)w;
    a.lm.done = (uint32_t*)(w + o_done);
    a.lm.nb = 1;
    a.lm.err = ctx->d_err;
    OCR_CUDA(cudaMemsetAsync(a.lm.done, 0, 4, ctx->stream));
    launch_matvec(ctx->stream, a, ctx->num_sms, false);
    OCR_CUDA(cudaGetLastError());
    return OCR_OK;
}

ocr_status ocr_op_attention_decode(ocr_ctx* ctx, float* d_qkv, const float* d_q_norm, const float* d_k_norm,
                                   const float* d_rope, uint16_t* d_k_cache, uint16_t* d_v_cache, int n_head, int n_kv,
                                   int n_ctx, int pos, float eps, float* d_out) {
    if (!ctx || !d_qkv || !d_q_norm || !d_k_norm || !d_rope || !d_k_cache || !d_v_cache || !d_out)
        return fail(OCR_ERR_ARG, "null argument");
    if (n_kv < 1 || n_head % n_kv) return fail(OCR_ERR_ARG, "n_head must be a multiple of n_kv");
    const int g = n_head / n_kv;
    if (g != 1 && g != 2 && g != 4 && g != 8) return fail(OCR_ERR_ARG, "GQA groups of 1, 2, 4 or 8 only");
    if (pos < 0 || pos >= n_ctx) return fail(OCR_ERR_ARG, "pos outside the cache");
    OCR_CUDA(cudaSetDevice(ctx->device));
    AttnArgs a;
    a.splits = attention_splits(ctx->num_sms, 1, n_kv, n_ctx);
    OCR_TRY(ensure_op_scratch(ctx, 256));
    char* w = (char*)ctx->op_scratch;
    cudaStream_t st = ctx->stream;
    OCR_CUDA(cudaMemcpyAsync(w, &pos, 4, cudaMemcpyHostToDevice, st));
    a.qkv = d_qkv;
    a.qkv_stride = (n_head + 2 * n_kv) * 128;
    a.q_norm = d_q_norm;
    a.k_norm = d_k_norm;
    a.rope = d_rope;
    a.kc = (__half*)d_k_cache;
    a.vc = (__half*)d_v_cache;
    a.pos = (const int32_t*)w;
    a.n_head = n_head;
    a.n_kv = n_kv;
    a.n_ctx = n_ctx;
    a.eps = eps;
    a.scale = 1.0f / sqrtf(128.0f);
    a.out = d_out;
    a.out_stride = n_head * 128;
    a.nb = 1;
    a.err = ctx->d_err;
    launch_attention_decode(st, a, false);
    OCR_CUDA(cudaGetLastError());
    return OCR_OK;
}


// ---- GGUF reader, host only ---------------------------------------------------------------------------------------
struct ocr_gguf {
    Gguf g;
};

ocr_status ocr_gguf_open(const char* path, ocr_gguf** out) {
    if (!path || !out) return fail(OCR_ERR_ARG, "null argument");
    std::string msg;
    auto src = file_source(path, msg);
    if (!src) return fail(OCR_ERR_IO, msg);
    auto* h = new ocr_gguf;
    if (!h->g.parse(std::move(src), msg)) {
        delete h;
        return fail(OCR_ERR_FORMAT, std::string(path) + " is not a readable GGUF: " + msg);
    }
    *out = h;
    return OCR_OK;
}

ocr_status ocr_gguf_open_memory(const void* bytes, size_t n, ocr_gguf** out) {
    if ((!bytes && n) || !out) return fail(OCR_ERR_ARG, "null argument");
    static const uint8_t empty = 0;
    std::string msg;
    auto* h = new ocr_gguf;
    if (!h->g.parse(memory_source(bytes ? bytes : &empty, n), msg)) {
        delete h;
        return fail(OCR_ERR_FORMAT, "not a readable GGUF: " + msg);
    }
    *out = h;
    return OCR_OK;
}

ocr_status ocr_gguf_close(ocr_gguf* g) {
    delete g;
    return OCR_OK;
}

ocr_status ocr_gguf_header(const ocr_gguf* h, uint32_t* version, uint64_t* n_tensors, uint64_t* alignment,
                           uint64_t* data_offset) {
    if (!h) return fail(OCR_ERR_ARG, "null argument");
    if (version) *version = h->g.version;
    if (n_tensors) *n_tensors = h->g.tensors.size();
    if (alignment) *alignment = h->g.alignment;
    if (data_offset) *data_offset = h->g.data_offset;
    return OCR_OK;
}

ocr_status ocr_gguf_get_u32(const ocr_gguf* h, const char* key, uint32_t* out) {
    if (!h || !key || !out) return fail(OCR_ERR_ARG, "null argument");
    std::string msg;
    if (!h->g.get_u32(key, *out, msg)) return fail(OCR_ERR_FORMAT, msg);
    return OCR_OK;
}

ocr_status ocr_gguf_get_f32(const ocr_gguf* h, const char* key, float* out) {
    if (!h || !key || !out) return fail(OCR_ERR_ARG, "null argument");
    std::string msg;
    if (!h->g.get_f32(key, *out, msg)) return fail(OCR_ERR_FORMAT, msg);
    return OCR_OK;
}

ocr_status ocr_gguf_get_str(const ocr_gguf* h, const char* key, char* out, size_t cap) {
    if (!h || !key || !out || !cap) return fail(OCR_ERR_ARG, "null argument");
    std::string msg, v;
    if (!h->g.get_str(key, v, msg)) return fail(OCR_ERR_FORMAT, msg);
    if (v.size() + 1 > cap) return fail(OCR_ERR_ARG, key + std::string(": string longer than the buffer"));
    memcpy(out, v.c_str(), v.size() + 1);
    return OCR_OK;
}

ocr_status ocr_gguf_f32_array(const ocr_gguf* h, const char* key, float* out, size_t cap, size_t* n) {
    if (!h || !key || !n) return fail(OCR_ERR_ARG, "null argument");
    auto it = h->g.meta.find(key);
    if (it == h->g.meta.end()) return fail(OCR_ERR_FORMAT, std::string("GGUF has no metadata key ") + key);
    if (it->second.type != 9) return fail(OCR_ERR_FORMAT, std::string(key) + " is not an array");
    const auto& a = it->second.arr;
    for (const auto& v : a)
        if (v.type != 6) return fail(OCR_ERR_FORMAT, std::string(key) + " holds a non-f32 value");
    *n = a.size();
    if (out) {
        if (cap < a.size()) return fail(OCR_ERR_ARG, "output buffer too small");
        for (size_t i = 0; i < a.size(); i++) out[i] = (float)a[i].f;
    }
    return OCR_OK;
}

ocr_status ocr_gguf_tensor(const ocr_gguf* h, const char* name, int* ggml_type, uint64_t shape[4], int* n_dims,
                           uint64_t* file_offset) {
    if (!h || !name) return fail(OCR_ERR_ARG, "null argument");
    const GTensor* t = h->g.info(name);
    if (!t) return fail(OCR_ERR_FORMAT, std::string("GGUF has no tensor ") + name);
    if (ggml_type) *ggml_type = t->type == GType::F32 ? 0 : t->type == GType::F16 ? 1 : t->type == GType::Q8_0 ? 8 : 30;
    if (shape)
        for (int i = 0; i < 4; i++) shape[i] = i < (int)t->shape.size() ? t->shape[i] : 1;
    if (n_dims) *n_dims = (int)t->shape.size();
    if (file_offset) *file_offset = t->file_offset;
    return OCR_OK;
}

ocr_status ocr_gguf_to_f32(const ocr_gguf* h, const char* name, float* out, size_t cap, size_t* n) {
    if (!h || !name || !n) return fail(OCR_ERR_ARG, "null argument");
    const GTensor* t = h->g.info(name);
    if (!t) return fail(OCR_ERR_FORMAT, std::string("GGUF has no tensor ") + name);
    if (t->n_bytes() > (1u << 20))
        return fail(OCR_ERR_ARG, std::string(name) + ": " + std::to_string(t->n_bytes()) + " bytes is not small");
    *n = (size_t)t->n_elements();
    if (!out) return OCR_OK;
    if (cap < *n) return fail(OCR_ERR_ARG, "output buffer too small");
    std::vector<uint8_t> d((size_t)t->n_bytes());
    std::string msg;
    if (!h->g.src->read_at(t->file_offset, d.data(), d.size(), msg)) return fail(OCR_ERR_IO, msg);
    auto h2f = [](uint16_t x) { return __half2float(__ushort_as_half(x)); };
    switch (t->type) {
    case GType::F32: memcpy(out, d.data(), *n * 4); break;
    case GType::F16:
        for (size_t i = 0; i < *n; i++) out[i] = h2f((uint16_t)(d[2 * i] | (d[2 * i + 1] << 8)));
        break;
    case GType::BF16:
        for (size_t i = 0; i < *n; i++) {
            const uint32_t b = (uint32_t)(d[2 * i] | (d[2 * i + 1] << 8)) << 16;
            memcpy(&out[i], &b, 4);
        }
        break;
    case GType::Q8_0:
        for (size_t b = 0; b < *n / 32; b++) {
            const uint8_t* blk = d.data() + b * 34;
            const float s = h2f((uint16_t)(blk[0] | (blk[1] << 8)));
            for (int j = 0; j < 32; j++) out[b * 32 + j] = (float)(int8_t)blk[2 + j] * s;
        }
        break;
    }
    return OCR_OK;
}

ocr_status ocr_gguf_text_config(const ocr_gguf* h, ocr_text_cfg* out) {
    if (!h || !out) return fail(OCR_ERR_ARG, "null argument");
    ocr_text_cfg c{};
    OCR_TRY(validate_gguf(h->g, c));
    *out = c;
    return OCR_OK;
}

ocr_status ocr_gguf_vision_config(const ocr_gguf* h, ocr_vision_cfg* out) {
    if (!h || !out) return fail(OCR_ERR_ARG, "null argument");
    const Gguf& g = h->g;
    std::string msg, proj;
    if (!g.get_str("clip.projector_type", proj, msg)) return fail(OCR_ERR_FORMAT, msg);
    if (proj != "lightonocr") return fail(OCR_ERR_FORMAT, "projector \"" + proj + "\": this engine runs lightonocr only");
    auto it = g.meta.find("clip.use_silu");
    if (it == g.meta.end()) return fail(OCR_ERR_FORMAT, "GGUF has no metadata key clip.use_silu");
    if (it->second.type != 7) return fail(OCR_ERR_FORMAT, "clip.use_silu is not a bool");
    if (!it->second.u) return fail(OCR_ERR_FORMAT, "clip.use_silu is false: the encoder's FFN would not be SwiGLU");
    ocr_vision_cfg c{};
    const char* keys[] = {"clip.vision.embedding_length", "clip.vision.attention.head_count", "clip.vision.block_count",
                          "clip.vision.feed_forward_length", "clip.vision.patch_size",
                          "clip.vision.spatial_merge_size", "clip.vision.image_size", "clip.vision.projection_dim"};
    uint32_t v[8];
    for (int i = 0; i < 8; i++)
        if (!g.get_u32(keys[i], v[i], msg)) return fail(OCR_ERR_FORMAT, msg);
    if (v[1] == 0 || v[0] % v[1] != 0 || v[0] / v[1] != 64)
        return fail(OCR_ERR_FORMAT, "head dim " + std::to_string(v[0]) + "/" + std::to_string(v[1]) +
                                        ": the attention kernel is written for 64");
    c.dim = (int32_t)v[0];
    c.n_head = (int32_t)v[1];
    c.n_layer = (int32_t)v[2];
    c.n_ff = (int32_t)v[3];
    c.patch = (int32_t)v[4];
    c.merge = (int32_t)v[5];
    c.image_size = (int32_t)v[6];
    c.proj_dim = (int32_t)v[7];
    if (!g.get_f32("clip.vision.attention.layer_norm_epsilon", c.eps, msg)) return fail(OCR_ERR_FORMAT, msg);
    c.rope_theta = 10000.0f;  // clip.cpp sets it in code for this projector; the GGUF carries no key (vision.rs:30-31)
    for (int k = 0; k < 2; k++) {
        const char* key = k == 0 ? "clip.vision.image_mean" : "clip.vision.image_std";
        float* dst = k == 0 ? c.mean : c.std;
        auto a = g.meta.find(key);
        if (a == g.meta.end()) return fail(OCR_ERR_FORMAT, std::string("GGUF has no metadata key ") + key);
        if (a->second.type != 9) return fail(OCR_ERR_FORMAT, std::string(key) + " is not an array");
        if (a->second.arr.size() != 3)
            return fail(OCR_ERR_FORMAT, std::string(key) + " has " + std::to_string(a->second.arr.size()) + " values");
        for (int i = 0; i < 3; i++) {
            if (a->second.arr[i].type != 6) return fail(OCR_ERR_FORMAT, std::string(key) + " holds a non-f32 value");
            dst[i] = (float)a->second.arr[i].f;
        }
    }
    *out = c;
    return OCR_OK;
}

ocr_status ocr_op_wait_probe(ocr_ctx* ctx, int tries, int* waited_out) {
    if (!ctx || !waited_out) return fail(OCR_ERR_ARG, "null argument");
    if (tries < 1 || tries > 100000) return fail(OCR_ERR_ARG, "tries must be in [1, 100000]");
    OCR_CUDA(cudaSetDevice(ctx->device));
    OCR_TRY(ensure_op_scratch(ctx, 256));
    int* d_out = (int*)ctx->op_scratch;
    OCR_CUDA(cudaMemsetAsync(d_out, 0, 4, ctx->stream));
    launch_wait_probe(ctx->stream, ctx->d_err, (uint32_t)tries, d_out);
    OCR_CUDA(cudaGetLastError());
    OCR_CUDA(cudaMemcpyAsync(waited_out, d_out, 4, cudaMemcpyDeviceToHost, ctx->stream));
    OCR_CUDA(cudaStreamSynchronize(ctx->stream));
    return OCR_OK;  // the device error flag stays set: ocr_ctx_sync reports (and clears) it
}

ocr_status ocr_op_penalize(ocr_ctx* ctx, float* d_logits, int n_vocab, float rp, int window, const int32_t* d_hist,
                           int n_hist) {
    if (!ctx || !d_logits || (!d_hist && n_hist)) return fail(OCR_ERR_ARG, "null argument");
    if (rp != 1.0f && !(std::isnormal(rp) && rp > 0.0f)) return fail(OCR_ERR_ARG, "the repetition penalty is no positive normal f32");
    if (window < 1 || n_vocab < 1 || n_hist < 0) return fail(OCR_ERR_ARG, "bad sizes");
    OCR_CUDA(cudaSetDevice(ctx->device));
    OCR_TRY(ensure_op_scratch(ctx, 256));
    OCR_CUDA(cudaMemcpyAsync(ctx->op_scratch, &n_hist, 4, cudaMemcpyHostToDevice, ctx->stream));
    LmArgs a;
    a.nb = 1;
    a.sample = 1;
    a.rp = rp;
    a.window = window;
    a.hist = const_cast<int32_t*>(d_hist);
    a.hist_cap = n_hist;
    a.len = (int32_t*)ctx->op_scratch;
    launch_penalize(ctx->stream, d_logits, n_vocab, a, ctx->num_sms);
    OCR_CUDA(cudaGetLastError());
    return OCR_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------------------------------
// the LM head + choice with no allocation
// ---------------------------------------------------------------------------------------------------------------------
// Some callers cannot let a library allocate device memory mid-run: a serving loop that plans every byte of HBM up
// front and runs under a fixed budget, a caller whose allocator owns the device and forbids hidden cudaMalloc calls,
// or a latency-critical path where cudaMalloc/cudaFree would synchronise the device. ocr_op_lm_head_sample grows a
// per-context scratch buffer on its first call; this variant instead keeps its scratch (the CTAs' partial maxima and
// the completion ticket) in a file-scope device array that exists from module load on, so the call allocates
// nothing. The array is one per device: two calls that can run at the same time on one device (different contexts
// or streams) race on it; calls queued on one context's stream are ordered and safe.
namespace {

constexpr size_t NOALLOC_SCRATCH_BYTES = 16384;
// the ticket sits on its own 256 B after the partials (8 B per CTA, plus one NaN flag and the 256 B gap): the CTA count
// the array holds, 2015
constexpr int NOALLOC_MAX_CTAS = (int)((NOALLOC_SCRATCH_BYTES - 264) / 8);
static __device__ __align__(256) unsigned char g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

constexpr int NOALLOC_MAX_DEVICES = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_addr[NOALLOC_MAX_DEVICES] = {};

// the array's device address on `device`, looked up once per device with that device current (the first call on a
// device does this setup — make it before any stream capture)
ocr_status noalloc_scratch(int device, void** out) {
    if (device < 0 || device >= NOALLOC_MAX_DEVICES) return fail(OCR_ERR_ARG, "device index out of range");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_addr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
        g_noalloc_addr[device] = p;
    }
    *out = g_noalloc_addr[device];
    return OCR_OK;
}

}  // namespace

ocr_status ocr_op_lm_head_sample_noalloc(ocr_ctx* ctx, const uint8_t* d_w, int n_vocab, int dim, const float* d_x,
                                         const float* d_norm_w, float eps, float rp, int window, int32_t* d_hist,
                                         int32_t* d_len, int32_t* d_tok, float* d_logits) {
    if (!ctx || !d_w || !d_x || !d_hist || !d_len || !d_tok) return fail(OCR_ERR_ARG, "null argument");
    if (n_vocab < 1 || dim < 32 || dim % 32) return fail(OCR_ERR_ARG, "bad shape");
    if ((uintptr_t)d_w & 15) return fail(OCR_ERR_ARG, "the rows must start 16-B aligned");
    if (rp != 1.0f && !(std::isnormal(rp) && rp > 0.0f)) return fail(OCR_ERR_ARG, "the repetition penalty is no positive normal f32");
    if (window < 1) return fail(OCR_ERR_ARG, "repetition window must be >= 1");
    const int grid = lm_head_grid(ctx->num_sms, n_vocab, dim);
    const size_t o_done = ((size_t)grid * 2 + 1) * 4 + 256;  // partials, then the ticket on its own 256 B
    if (grid > NOALLOC_MAX_CTAS || o_done + 4 > NOALLOC_SCRATCH_BYTES)
        return fail(OCR_ERR_ARG, "the LM head would run " + std::to_string(grid) + " CTAs; the static scratch holds the partials of at most " +
                                     std::to_string(NOALLOC_MAX_CTAS));
    OCR_CUDA(cudaSetDevice(ctx->device));
    void* scratch = nullptr;
    OCR_TRY(noalloc_scratch(ctx->device, &scratch));
    char* w = (char*)scratch;
    MvArgs a;
    a.w.w = d_w;
    a.w.rows = n_vocab;
    a.w.cols = dim;
    a.w.stride = q8_stride(dim);
    a.x = d_x;
    a.x_stride = dim;
    a.nw = d_norm_w;
    a.eps = eps;
    a.nb = 1;
    a.mode = MV_LMHEAD;
    a.y = d_logits;
    a.err = ctx->d_err;
    a.lm.sample = 1;
    a.lm.rp = rp;
    a.lm.window = window;
    a.lm.hist = d_hist;
    a.lm.hist_cap = 1 << 30;
    a.lm.len = d_len;
    a.lm.tok = d_tok;
    a.lm.part = (float*)w;
    a.lm.done = (uint32_t*)(w + o_done);
    a.lm.nb = 1;
    a.lm.err = ctx->d_err;
    // the completion ticket must start at zero (the kernel's last CTA resets it, but an earlier call that failed
    // part way may not have); the partials need no clearing, every CTA writes its own before the ticket
    OCR_CUDA(cudaMemsetAsync(a.lm.done, 0, 4, ctx->stream));
    launch_matvec(ctx->stream, a, ctx->num_sms, false);
    OCR_CUDA(cudaGetLastError());
    return OCR_OK;
}
