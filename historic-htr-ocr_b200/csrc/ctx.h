// ctx.h — the context handle and the device-memory helpers shared by the runtime's translation units (runtime.cu:
// the text decoder; vision.cu: the vision encoder). Internal: not part of the C ABI.
#pragma once

#include <cuda_runtime.h>

#include <string>

#include "ocr_cuda.h"

namespace ocr {
void set_error(const std::string& m);
ocr_status fail(ocr_status c, const std::string& m);
ocr_status cuda_fail(cudaError_t e, const char* what);
}  // namespace ocr

// ---- the context ----
struct ocr_ctx {
    int refs = 1;  // the caller's handle + one per live model: freed when the last is released
    int device = 0;
    cudaStream_t stream = nullptr;
    int num_sms = 148;
    bool pdl = true;
    int* d_err = nullptr;
    uint64_t mem_weights = 0, mem_kv = 0, mem_work = 0;
    // scratch of the low-level ops (grown on demand, freed with the context)
    void* op_scratch = nullptr;
    size_t op_scratch_bytes = 0;
    // pinned staging for uploads
    void* h_stage = nullptr;
    void* d_stage = nullptr;
    size_t stage_bytes = 0;
};

namespace ocr {
// device memory, zeroed (and the zeroing complete) before it is returned; ctr (nullable) counts the bytes
cudaError_t dalloc(void** p, size_t n, uint64_t* ctr);
void dfree(void* p, size_t n, uint64_t* ctr);
// the context's device error flag: OCR_ERR_DEVICE with its message when a kernel set it (the flag is then cleared)
ocr_status check_device_error(ocr_ctx* ctx);
// drops one reference to the context (a model or vision encoder holds one while it lives); the last frees it
void ctx_release(ocr_ctx* c);
}  // namespace ocr
