// k_weights.cu — q8_0 device layout: repack from GGUF blocks, the seeded synthetic generator, unpack for export.
//
// Row layout (kernels.cuh): int8 quants [cols] | f16 scales [cols/32] | pad, stride q8_stride(cols).
// The synthetic generator's arithmetic is integer-only up to one f32 multiply, an IEEE division and the f16 RNE
// store, each written with the _rn intrinsics so no contraction changes a rounding: the host test generator of the
// same seed gives the same bits.
#include "kernels.cuh"

namespace ocr {

// ---- the GGUF q8_0 block (ocr-gguf/src/lib.rs:129-135): f16 d (little endian) + 32 x int8 ---------------------------
__global__ void k_repack_q8_0(const uint8_t* __restrict__ blocks, int rows, int cols, uint8_t* __restrict__ w,
                              int row_mul, int row_add) {
    const int nbr = cols / 32, stride = q8_stride(cols);
    const long nblk = (long)rows * nbr;
    for (long b = blockIdx.x * (long)blockDim.x + threadIdx.x; b < nblk; b += (long)gridDim.x * blockDim.x) {
        const int r = (int)(b / nbr), c = (int)(b % nbr);
        const uint8_t* src = blocks + b * 34;
        // 34-byte blocks start on 2-byte boundaries: read 17 half-words
        const uint16_t* s16 = reinterpret_cast<const uint16_t*>(src);
        uint32_t v[8];
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = (uint32_t)s16[1 + 2 * k] | ((uint32_t)s16[2 + 2 * k] << 16);
        uint8_t* row = w + ((long)r * row_mul + row_add) * stride;
        uint4* dst = reinterpret_cast<uint4*>(row + c * 32);
        dst[0] = make_uint4(v[0], v[1], v[2], v[3]);
        dst[1] = make_uint4(v[4], v[5], v[6], v[7]);
        reinterpret_cast<uint16_t*>(row + cols)[c] = s16[0];
    }
}

__global__ void k_unpack_q8_0(const uint8_t* __restrict__ w, int rows, int cols, int row_mul, int row_add,
                              uint8_t* __restrict__ blocks) {
    const int nbr = cols / 32, stride = q8_stride(cols);
    const long nblk = (long)rows * nbr;
    for (long b = blockIdx.x * (long)blockDim.x + threadIdx.x; b < nblk; b += (long)gridDim.x * blockDim.x) {
        const int r = (int)(b / nbr), c = (int)(b % nbr);
        const uint8_t* row = w + ((long)r * row_mul + row_add) * stride;
        uint8_t* dst = blocks + b * 34;
        const uint16_t h = reinterpret_cast<const uint16_t*>(row + cols)[c];
        dst[0] = (uint8_t)(h & 0xff);
        dst[1] = (uint8_t)(h >> 8);
        for (int k = 0; k < 32; k++) dst[2 + k] = row[c * 32 + k];
    }
}

// ---- SplitMix64 addressed by output index (ocr-decode sampling.rs:24-35's generator) ---------------------------------
__device__ __forceinline__ uint64_t splitmix64_at(uint64_t seed, uint64_t i) {
    uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ int u16sum4(uint64_t z) {
    return (int)(z & 0xffff) + (int)((z >> 16) & 0xffff) + (int)((z >> 32) & 0xffff) + (int)(z >> 48);
}

// N(0,1) stand-in: Irwin–Hall sum of 12 uniform u16, centred, scaled by 2^-16 (exact)
__device__ __forceinline__ float gauss(uint64_t seed, uint64_t i) {
    const int s = u16sum4(splitmix64_at(seed, 3 * i)) + u16sum4(splitmix64_at(seed, 3 * i + 1)) +
                  u16sum4(splitmix64_at(seed, 3 * i + 2)) - 6 * 65535;
    return __fmul_rn((float)s, 1.0f / 65536.0f);
}

__device__ __forceinline__ int8_t sat_i8(float v) {
    if (v != v) return 0;
    if (v >= 127.0f) return 127;
    if (v <= -128.0f) return -128;
    return (int8_t)v;
}

// one q8_0 block of generated values, quantized as ggml's quantize_row_q8_0_ref (text.rs:676-691)
__global__ void k_synth_q8_0(uint64_t seed, float sigma, int rows, int cols, int valid, uint8_t* __restrict__ w,
                             int row_mul, int row_add) {
    const int nbr = cols / 32, stride = q8_stride(cols);
    const long nblk = (long)rows * nbr;
    for (long b = blockIdx.x * (long)blockDim.x + threadIdx.x; b < nblk; b += (long)gridDim.x * blockDim.x) {
        float x[32];
        float amax = 0.0f;
        const int r = (int)(b / nbr), c = (int)(b % nbr);
#pragma unroll
        for (int j = 0; j < 32; j++) {
            // value (r, col) = sigma * gauss(r * valid + col) for col < valid, zero past it (valid == cols: the flat
            // index b * 32 + j)
            const int col = c * 32 + j;
            x[j] = col < valid ? __fmul_rn(sigma, gauss(seed, (uint64_t)r * valid + col)) : 0.0f;
            const float a = fabsf(x[j]);
            if (a > amax) amax = a;
        }
        const float dv = __fdiv_rn(amax, 127.0f);
        const float id = dv != 0.0f ? __fdiv_rn(1.0f, dv) : 0.0f;
        uint8_t* row = w + ((long)r * row_mul + row_add) * stride;
        uint32_t v[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
            uint32_t u = 0;
#pragma unroll
            for (int m = 0; m < 4; m++) u |= ((uint32_t)(uint8_t)sat_i8(roundf(__fmul_rn(x[4 * k + m], id)))) << (8 * m);
            v[k] = u;
        }
        uint4* dst = reinterpret_cast<uint4*>(row + c * 32);
        dst[0] = make_uint4(v[0], v[1], v[2], v[3]);
        dst[1] = make_uint4(v[4], v[5], v[6], v[7]);
        reinterpret_cast<__half*>(row + cols)[c] = __float2half_rn(dv);
    }
}

// 1 + 0.01 u, u = the top 24 bits of output i mapped to [-1, 1) (the tests' norm weights, text.rs:1304)
__global__ void k_synth_norm(uint64_t seed, int n, float* __restrict__ out) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float u = (float)(splitmix64_at(seed, (uint64_t)i) >> 40) * (1.0f / 16777216.0f) * 2.0f - 1.0f;
        out[i] = __fadd_rn(1.0f, __fmul_rn(0.01f, u));
    }
}

// one CTA per (row, slice): quants as 32-bit words, then the slice's scales, then zeros to the stride
__global__ void k_slice_o(const uint8_t* __restrict__ w, int cols, int parts, uint8_t* __restrict__ out) {
    const int r = blockIdx.x, j = blockIdx.y, rows = gridDim.x;
    const int sc = cols / parts, ss = q8_stride(sc);
    const uint8_t* src = w + (size_t)r * q8_stride(cols);
    uint8_t* dst = out + ((size_t)j * rows + r) * ss;
    for (int i = threadIdx.x; i < sc / 4; i += blockDim.x)
        reinterpret_cast<uint32_t*>(dst)[i] = reinterpret_cast<const uint32_t*>(src + (size_t)j * sc)[i];
    const uint16_t* scales = reinterpret_cast<const uint16_t*>(src + cols) + (size_t)j * (sc / 32);
    for (int i = threadIdx.x; i < sc / 32; i += blockDim.x) reinterpret_cast<uint16_t*>(dst + sc)[i] = scales[i];
    for (int i = sc + sc / 16 + threadIdx.x; i < ss; i += blockDim.x) dst[i] = 0;
}

static int grid_for(long n, int threads) {
    long g = (n + threads - 1) / threads;
    return (int)(g < 1 ? 1 : (g > 65535 * 8 ? 65535 * 8 : g));
}

void launch_repack_q8_0(cudaStream_t st, const uint8_t* blocks, int rows, int cols, uint8_t* w, int row_mul,
                        int row_add) {
    const long n = (long)rows * (cols / 32);
    k_repack_q8_0<<<grid_for(n, 256), 256, 0, st>>>(blocks, rows, cols, w, row_mul, row_add);
}

void launch_unpack_q8_0(cudaStream_t st, const uint8_t* w, int rows, int cols, int row_mul, int row_add,
                        uint8_t* blocks) {
    const long n = (long)rows * (cols / 32);
    k_unpack_q8_0<<<grid_for(n, 256), 256, 0, st>>>(w, rows, cols, row_mul, row_add, blocks);
}

void launch_synth_q8_0(cudaStream_t st, uint64_t seed, float sigma, int rows, int cols, uint8_t* w, int row_mul,
                       int row_add, int valid) {
    const long n = (long)rows * (cols / 32);
    k_synth_q8_0<<<grid_for(n, 128), 128, 0, st>>>(seed, sigma, rows, cols, valid > 0 ? valid : cols, w, row_mul,
                                                   row_add);
}

void launch_synth_norm(cudaStream_t st, uint64_t seed, int n, float* out) {
    k_synth_norm<<<grid_for(n, 256), 256, 0, st>>>(seed, n, out);
}

void launch_slice_o(cudaStream_t st, const uint8_t* w, int rows, int cols, int parts, uint8_t* out) {
    k_slice_o<<<dim3((unsigned)rows, (unsigned)parts), 128, 0, st>>>(w, cols, parts, out);
}

}  // namespace ocr
