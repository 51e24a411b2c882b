// k_vision.cu — the vision encoder's small kernels around its tensor-core contractions and attention: the bake's pad
// and the patch im2col (straight into the patch embedding's operand), the 2D RoPE with the f16 head-major K / V, the
// projector's norm + 2x2 unfold, and the GELU. Each writes the next contraction's operand (x16: groups of 32 rows,
// each value split exactly into f16 hi + lo, the layout of kernels.cuh) directly, so no f32 copy of it is made.
//
// Reference (b-straub/historic-htr-ocr): patchify.wgsl:22-38, rope2d.wgsl:25-45, heads_f16.wgsl, unfold2x2.wgsl:23-32,
// gelu.wgsl:22-27, rms_norm.wgsl; the graph in app/crates/ocr-wgpu/src/vision.rs:266-317, 405-423; the bake's white
// pad in app/crates/ocr-core/src/imageops.rs:318-323.
#include "kernels.cuh"

namespace ocr {

namespace {

__device__ __forceinline__ uint32_t h2_bits(float a, float b) {
    const __half2 h = __halves2half2(__float2half_rn(a), __float2half_rn(b));
    return *reinterpret_cast<const uint32_t*>(&h);
}

// 8 consecutive columns [k0, k0 + 8) of row n of an x16 group, split hi / lo
__device__ __forceinline__ void put8(uint8_t* g, int n, int k0, const float* v) {
    float h[8];
#pragma unroll
    for (int i = 0; i < 8; i++) h[i] = __half2float(__float2half_rn(v[i]));
    *reinterpret_cast<uint4*>(g + x16_offset(n, k0)) =
        make_uint4(h2_bits(h[0], h[1]), h2_bits(h[2], h[3]), h2_bits(h[4], h[5]), h2_bits(h[6], h[7]));
    *reinterpret_cast<uint4*>(g + x16_offset(BG_SLOTS + n, k0)) =
        make_uint4(h2_bits(v[0] - h[0], v[1] - h[1]), h2_bits(v[2] - h[2], v[3] - h[3]),
                   h2_bits(v[4] - h[4], v[5] - h[5]), h2_bits(v[6] - h[6], v[7] - h[7]));
}

}  // namespace

// one thread per (patch, 8-column piece); rows past the patches in the last group of 32 get zeros
__global__ void __launch_bounds__(256) k_patchify(const uint8_t* __restrict__ rgb, Placement pl, int patch,
                                                  const float* __restrict__ lut, int K, int n, int px,
                                                  uint8_t* __restrict__ x16) {
    __shared__ float slut[768];
    for (int i = threadIdx.x; i < 768; i += blockDim.x) slut[i] = lut[i];
    __syncthreads();
    const int pieces = K / 8, pp = patch * patch;
    const long total = (long)(n + BG_SLOTS - 1) / BG_SLOTS * BG_SLOTS * pieces;
    for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total; e += (long)gridDim.x * blockDim.x) {
        const int t = (int)(e / pieces), k0 = (int)(e % pieces) * 8;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int col = k0 + i;
            float val = 0.0f;
            if (t < n && col < 3 * pp) {
                const int ch = col / pp, r = col % pp, ky = r / patch, kx = r % patch;
                const int x = (t % px) * patch + kx - pl.left, y = (t / px) * patch + ky - pl.top;
                int byte = 255;  // the bake's white pad
                if (x >= 0 && x < pl.img_w && y >= 0 && y < pl.img_h) byte = rgb[((size_t)y * pl.img_w + x) * 3 + ch];
                val = slut[ch * 256 + byte];
            }
            v[i] = val;
        }
        put8(x16 + (size_t)(t / BG_SLOTS) * x16_group_bytes(K), t % BG_SLOTS, k0, v);
    }
}

void launch_patchify(cudaStream_t st, const uint8_t* rgb, const Placement& pl, int patch, const float* lut, int K,
                     uint8_t* x16) {
    const int px = pl.width / patch, n = px * (pl.height / patch);
    const long total = (long)(n + BG_SLOTS - 1) / BG_SLOTS * BG_SLOTS * (K / 8);
    const int blocks = (int)std::min<long>((total + 255) / 256, 148L * 16);
    k_patchify<<<blocks, 256, 0, st>>>(rgb, pl, patch, lut, K, n, px, x16);
}

// The attention's operands as they land in shared memory: per head, per tile of 64 keys, 8 KB of K (key row r, the
// 16-byte piece p of its 64 dims at r * 128 + ((p ^ (r % 8)) << 4): K-major with the 128-byte swizzle) and 8 KB of V
// transposed (dim row d, the piece q of keys 8q … 8q + 7 at d * 128 + ((q ^ (d % 8)) << 4)), so one bulk copy of a
// tile is a tensor-core operand. Keys past n are zero.
__device__ __forceinline__ size_t k_tiled(int h, int n_pad, int t, int d) {
    const int r = t & 63;
    return ((size_t)h * n_pad + (t & ~63)) * 64 + r * 64 + ((((d >> 3) ^ (r & 7))) << 3) + (d & 7);
}
__device__ __forceinline__ size_t vt_tiled(int h, int n_pad, int t, int d) {
    const int j = t & 63;
    return ((size_t)h * n_pad + (t & ~63)) * 64 + d * 64 + ((((j >> 3) ^ (d & 7))) << 3) + (j & 7);
}

// one thread per (row, head, rotation pair); the pair (2k, 2k + 1) of half `hf` (dims [0, d/2) by the patch row, [d/2,
// d) by the patch column) rotated in q (in place) and k; k and v stored f16 in the attention's tiled layouts
__global__ void __launch_bounds__(256) k_rope2d_heads(float* __restrict__ qkv, int n, int n_head, int d_head, int px,
                                                      const float* __restrict__ cs, int max_pos,
                                                      __half* __restrict__ kh, __half* __restrict__ vh, int n_pad) {
    const int pairs = d_head / 2, nk = d_head / 4, dim = n_head * d_head;
    const long total = (long)n_pad * n_head * pairs;
    for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total; e += (long)gridDim.x * blockDim.x) {
        const int j = (int)(e % pairs), h = (int)((e / pairs) % n_head), t = (int)(e / ((long)pairs * n_head));
        const int hf = j / nk, k = j % nk, o = hf * (d_head / 2) + 2 * k;
        __half2* kd = reinterpret_cast<__half2*>(kh + k_tiled(h, n_pad, t, o));
        __half* v0 = vh + vt_tiled(h, n_pad, t, o);
        __half* v1 = vh + vt_tiled(h, n_pad, t, o + 1);
        if (t >= n) {
            *kd = __floats2half2_rn(0.0f, 0.0f);
            *v0 = *v1 = __float2half_rn(0.0f);
            continue;
        }
        const int pos = hf == 0 ? t / px : t % px;
        const float c = cs[((size_t)(hf * max_pos + pos) * nk + k) * 2], s = cs[((size_t)(hf * max_pos + pos) * nk + k) * 2 + 1];
        float* row = qkv + (size_t)t * 3 * dim + h * d_head + o;
        const float q0 = row[0], q1 = row[1];
        row[0] = __fsub_rn(__fmul_rn(q0, c), __fmul_rn(q1, s));
        row[1] = __fadd_rn(__fmul_rn(q0, s), __fmul_rn(q1, c));
        const float k0 = row[dim], k1 = row[dim + 1];
        *kd = __floats2half2_rn(__fsub_rn(__fmul_rn(k0, c), __fmul_rn(k1, s)), __fadd_rn(__fmul_rn(k0, s), __fmul_rn(k1, c)));
        *v0 = __float2half_rn(row[2 * dim]);
        *v1 = __float2half_rn(row[2 * dim + 1]);
    }
}

void launch_rope2d_heads(cudaStream_t st, float* qkv, int n, int n_head, int d_head, int px, const float* cs,
                         int max_pos, __half* kh, __half* vh, int n_pad) {
    const long total = (long)n_pad * n_head * (d_head / 2);
    const int blocks = (int)std::min<long>((total + 255) / 256, 148L * 16);
    k_rope2d_heads<<<blocks, 256, 0, st>>>(qkv, n, n_head, d_head, px, cs, max_pos, kh, vh, n_pad);
}

// one CTA per merged token: the 4 source rows' RMS scales (f32 sums of squares, warp sums added in warp order), then
// the 4·dim unfolded columns, 8 per piece (channels c, c + 1 with their 4 kernel positions)
constexpr int UP_THREADS = 256;
__global__ void __launch_bounds__(UP_THREADS) k_unfold_prep(const float* __restrict__ x, const float* __restrict__ w,
                                                            float eps, int px, int n_out, int dim,
                                                            uint8_t* __restrict__ x16) {
    __shared__ float part[4][UP_THREADS / 32];
    __shared__ float scale[4];
    const int o = blockIdx.x, K = 4 * dim;
    uint8_t* g = x16 + (size_t)(o / BG_SLOTS) * x16_group_bytes(K);
    const int n = o % BG_SLOTS;
    if (o >= n_out) {
        const float z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int p = threadIdx.x; p < K / 8; p += UP_THREADS) put8(g, n, p * 8, z);
        return;
    }
    const int oxn = px / 2, oy = o / oxn, ox = o % oxn;
    const float* src[4];
#pragma unroll
    for (int q = 0; q < 4; q++) src[q] = x + ((size_t)(2 * oy + (q >> 1)) * px + 2 * ox + (q & 1)) * dim;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        float s = 0.0f;
        for (int c = threadIdx.x; c < dim; c += UP_THREADS) s = __fadd_rn(s, __fmul_rn(src[q][c], src[q][c]));
#pragma unroll
        for (int m = 16; m; m >>= 1) s += __shfl_xor_sync(0xffffffffu, s, m);
        if (lane == 0) part[q][warp] = s;
    }
    __syncthreads();
    if (threadIdx.x < 4) {
        float s = 0.0f;
        for (int i = 0; i < UP_THREADS / 32; i++) s += part[threadIdx.x][i];
        scale[threadIdx.x] = 1.0f / sqrtf(s / (float)dim + eps);
    }
    __syncthreads();
    for (int p = threadIdx.x; p < K / 8; p += UP_THREADS) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int col = p * 8 + i, c = col >> 2, q = col & 3;  // q = ky * 2 + kx
            v[i] = __fmul_rn(__fmul_rn(src[q][c], scale[q]), w[c]);
        }
        put8(g, n, p * 8, v);
    }
}

void launch_unfold_prep(cudaStream_t st, const float* x, const float* w, float eps, int px, int py, int dim,
                        uint8_t* x16) {
    const int n_out = (px / 2) * (py / 2);
    k_unfold_prep<<<(n_out + BG_SLOTS - 1) / BG_SLOTS * BG_SLOTS, UP_THREADS, 0, st>>>(x, w, eps, px, n_out, dim, x16);
}

// ---- the bake's Lanczos-3 resize (imageops::resize of the `image` crate 0.25, Lanczos3): separable, a vertical pass
// into f32, then a horizontal pass into bytes. The taps and their normalised weights per output row / column come from
// the host (the same f32 arithmetic as the CPU restatement); every sum runs tap by tap in order, each product rounded
// before the add (no fused multiply-add), as the reference's Rust evaluates it.
__global__ void __launch_bounds__(256) k_resize_v(const uint8_t* __restrict__ rgb, int w0, int h, const int* __restrict__ left,
                                                  const int* __restrict__ cnt, const float* __restrict__ wt, int maxn,
                                                  float* __restrict__ tmp) {
    const long total = (long)h * w0 * 3;
    for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total; e += (long)gridDim.x * blockDim.x) {
        const int y = (int)(e / ((long)w0 * 3)), xc = (int)(e % ((long)w0 * 3));
        const int l = left[y], n = cnt[y];
        const float* w = wt + (size_t)y * maxn;
        float t = 0.0f;
        for (int i = 0; i < n; i++) t = __fadd_rn(t, __fmul_rn((float)rgb[(size_t)(l + i) * w0 * 3 + xc], w[i]));
        tmp[e] = t;
    }
}

__global__ void __launch_bounds__(256) k_resize_h(const float* __restrict__ tmp, int w0, int h, int w,
                                                  const int* __restrict__ left, const int* __restrict__ cnt,
                                                  const float* __restrict__ wt, int maxn, uint8_t* __restrict__ out) {
    const long total = (long)h * w * 3;
    for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total; e += (long)gridDim.x * blockDim.x) {
        const int c = (int)(e % 3), x = (int)((e / 3) % w), y = (int)(e / (3L * w));
        const int l = left[x], n = cnt[x];
        const float* ww = wt + (size_t)x * maxn;
        const float* row = tmp + (size_t)y * w0 * 3 + c;
        float t = 0.0f;
        for (int i = 0; i < n; i++) t = __fadd_rn(t, __fmul_rn(row[(size_t)(l + i) * 3], ww[i]));
        t = fminf(fmaxf(t, 0.0f), 255.0f);
        out[e] = (uint8_t)roundf(t);  // half away from zero, as Rust's f32::round
    }
}

void launch_resize(cudaStream_t st, const uint8_t* rgb, int w0, int h0, int w, int h, const int* vleft,
                   const int* vcnt, const float* vw, int vmax, const int* hleft, const int* hcnt, const float* hw,
                   int hmax, float* tmp, uint8_t* out) {
    (void)h0;
    const long tv = (long)h * w0 * 3, th = (long)h * w * 3;
    k_resize_v<<<(int)std::min<long>((tv + 255) / 256, 148L * 32), 256, 0, st>>>(rgb, w0, h, vleft, vcnt, vw, vmax, tmp);
    k_resize_h<<<(int)std::min<long>((th + 255) / 256, 148L * 32), 256, 0, st>>>(tmp, w0, h, w, hleft, hcnt, hw, hmax, out);
}

// the baked canvas: the (scaled) image at (left, top) of a white fw x fh canvas
__global__ void __launch_bounds__(256) k_bake_place(const uint8_t* __restrict__ src, int sw, int sh, int left, int top,
                                                    int fw, int fh, uint8_t* __restrict__ out) {
    const long total = (long)fw * fh * 3;
    for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total; e += (long)gridDim.x * blockDim.x) {
        const int c = (int)(e % 3), x = (int)((e / 3) % fw) - left, y = (int)(e / (3L * fw)) - top;
        out[e] = (x >= 0 && x < sw && y >= 0 && y < sh) ? src[((size_t)y * sw + x) * 3 + c] : (uint8_t)255;
    }
}

void launch_bake_place(cudaStream_t st, const uint8_t* src, int sw, int sh, int left, int top, int fw, int fh,
                       uint8_t* out) {
    const long total = (long)fw * fh * 3;
    k_bake_place<<<(int)std::min<long>((total + 255) / 256, 148L * 32), 256, 0, st>>>(src, sw, sh, left, top, fw, fh, out);
}

// gelu.wgsl:22-26: 0.5 x (1 + tanh(sqrt(2/pi) x (1 + 0.044715 x²))), the tanh argument clamped to ±15
__device__ __forceinline__ float gelu_tanh(float x) {
    float t = __fmul_rn(__fmul_rn(0.7978845608028654f, x), __fadd_rn(1.0f, __fmul_rn(__fmul_rn(0.044715f, x), x)));
    t = fminf(fmaxf(t, -15.0f), 15.0f);
    return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, tanhf(t)));
}

// one thread per (row, 8-column piece); rows past n in the last group get zeros
__global__ void __launch_bounds__(256) k_act_prep(const float* __restrict__ y, int n, int K, int act,
                                                  uint8_t* __restrict__ x16) {
    const int pieces = K / 8;
    const long total = (long)(n + BG_SLOTS - 1) / BG_SLOTS * BG_SLOTS * pieces;
    for (long e = blockIdx.x * (long)blockDim.x + threadIdx.x; e < total; e += (long)gridDim.x * blockDim.x) {
        const int r = (int)(e / pieces), k0 = (int)(e % pieces) * 8;
        float v[8];
        if (r < n) {
            const float4* s = reinterpret_cast<const float4*>(y + (size_t)r * K + k0);
            const float4 a = s[0], b = s[1];
            v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
            if (act) {
#pragma unroll
                for (int i = 0; i < 8; i++) v[i] = gelu_tanh(v[i]);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) v[i] = 0.0f;
        }
        put8(x16 + (size_t)(r / BG_SLOTS) * x16_group_bytes(K), r % BG_SLOTS, k0, v);
    }
}

void launch_act_prep(cudaStream_t st, const float* y, int n, int K, int act, uint8_t* x16) {
    const long total = (long)(n + BG_SLOTS - 1) / BG_SLOTS * BG_SLOTS * (K / 8);
    const int blocks = (int)std::min<long>((total + 255) / 256, 148L * 16);
    k_act_prep<<<blocks, 256, 0, st>>>(y, n, K, act, x16);
}

}  // namespace ocr
