// kt_decode.cu -- the device-resident decode step around the quantized
// matmul: Transformer.decode (Engine/kotensor/src/main/kotlin/Transformer.kt:
// 141-154) -> TransformerBlock.decodeInto (TransformerBlock.kt:40-47) ->
// Attention.decodeInto (Attention.kt:207-239, attendHead :295-328), with
// RMSNorm.forwardInto (RMSNorm.kt:71-90), RoPE.applyInPlace (RoPE.kt:117-137),
// SwiGLU.forwardInto (SwiGLU.kt:19-25, Tensor.siluInPlace Tensor.kt:231-237),
// the quantized / tied embedding lookups (Embedding.kt:96-101, :129-135) and
// the greedy argmax (Transformer.kt:255-266).
//
// Every kernel reads the token position (and token id) from device memory so
// a whole step can be captured once into a CUDA graph and replayed.  The KV
// cache is the reference's: fp32 keys / values [layers][kvHeads][maxSeq][headDim].
#include <cfloat>

#include "kt_internal.h"

namespace kt {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();  // red may still be read by a previous call
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) t += red[i];  // fixed order
    return t;
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = -FLT_MAX;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) t = fmaxf(t, red[i]);
    return t;
}

// out[r] = x[r] * (1 / sqrt(mean(x[r]^2) + eps)) * weight, one block per row (RMSNorm.kt:71-90).
__global__ void __launch_bounds__(kThreads) rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                          float* __restrict__ out, int dim, float eps) {
    __shared__ float red[32];
    const float* xr = x + static_cast<int64_t>(blockIdx.x) * dim;
    float* orow = out + static_cast<int64_t>(blockIdx.x) * dim;
    float ss = 0.0f;
    for (int d = threadIdx.x; d < dim; d += blockDim.x) ss = fmaf(xr[d], xr[d], ss);
    ss = block_sum(ss, red);
    const float r = 1.0f / sqrtf(ss / static_cast<float>(dim) + eps);
    for (int d = threadIdx.x; d < dim; d += blockDim.x) orow[d] = xr[d] * r * w[d];
}

// RoPE.applyInPlace at position *pos (+ row): pairs (i, i + half) of every head.
__global__ void rope_kernel(float* __restrict__ v, int rows, int width, int head_dim, const float* __restrict__ inv_freq,
                            const int32_t* __restrict__ pos) {
    const int half = head_dim / 2;
    const int heads = width / head_dim;
    const int64_t total = static_cast<int64_t>(rows) * heads * half;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int i = static_cast<int>(idx % half);
        const int64_t hr = idx / half;
        const int h = static_cast<int>(hr % heads);
        const int r = static_cast<int>(hr / heads);
        const float theta = static_cast<float>(*pos + r) * inv_freq[i];
        float s, c;
        sincosf(theta, &s, &c);
        float* p = v + static_cast<int64_t>(r) * width + h * head_dim;
        const float x1 = p[i], x2 = p[i + half];
        p[i] = x1 * c - x2 * s;
        p[i + half] = x1 * s + x2 * c;
    }
}

// cache[layer][h][pos + r][d] = kv[r][h * hd + d]
__global__ void kv_store_kernel(const float* __restrict__ k, const float* __restrict__ v, float* __restrict__ kc,
                                float* __restrict__ vc, int rows, int kv_heads, int head_dim, int max_seq, int layer,
                                const int32_t* __restrict__ pos) {
    const int width = kv_heads * head_dim;
    const int64_t total = static_cast<int64_t>(rows) * width;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int r = static_cast<int>(idx / width);
        const int e = static_cast<int>(idx % width);
        const int h = e / head_dim, d = e % head_dim;
        const int64_t off = ((static_cast<int64_t>(layer) * kv_heads + h) * max_seq + (*pos + r)) * head_dim + d;
        kc[off] = k[idx];
        vc[off] = v[idx];
    }
}

// attendHead (Attention.kt:295-328) for one query row at position *pos: one
// block per query head; scores over 0..pos kept in global scratch
// [heads][max_seq]; softmax with the reference's max; context = sum w_j v_j.
__global__ void __launch_bounds__(kThreads) attention_decode_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc, float* __restrict__ ctx,
    float* __restrict__ scores, int heads, int kv_heads, int head_dim, int max_seq, int layer, float scale,
    const int32_t* __restrict__ pos) {
    __shared__ float red[32];
    extern __shared__ float qs[];  // head_dim
    const int h = blockIdx.x;
    const int group = heads / kv_heads;
    const int position = *pos;
    const float* qh = q + static_cast<int64_t>(h) * head_dim;
    for (int d = threadIdx.x; d < head_dim; d += blockDim.x) qs[d] = qh[d];
    __syncthreads();
    const int64_t base = ((static_cast<int64_t>(layer) * kv_heads + h / group) * max_seq) * head_dim;
    float* sc = scores + static_cast<int64_t>(h) * max_seq;
    // scores: one warp per position
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int j = warp; j <= position; j += nw) {
        const float* kr = kc + base + static_cast<int64_t>(j) * head_dim;
        float s = 0.0f;
        for (int d = lane; d < head_dim; d += 32) s = fmaf(qs[d], kr[d], s);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) sc[j] = s * scale;
    }
    __syncthreads();
    float mx = -1e9f;  // the reference's initial maximum
    for (int j = threadIdx.x; j <= position; j += blockDim.x) mx = fmaxf(mx, sc[j]);
    mx = block_max(mx, red);
    float sum = 0.0f;
    for (int j = threadIdx.x; j <= position; j += blockDim.x) {
        const float e = expf(sc[j] - mx);
        sc[j] = e;
        sum += e;
    }
    sum = block_sum(sum, red);
    const float inv = 1.0f / sum;
    __syncthreads();
    // context: thread per head dimension, positions in order
    for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
        float acc = 0.0f;
        for (int j = 0; j <= position; ++j) acc = fmaf(sc[j] * inv, vc[base + static_cast<int64_t>(j) * head_dim + d], acc);
        ctx[static_cast<int64_t>(h) * head_dim + d] = acc;
    }
}

// gate = silu(gate) * up (Tensor.siluInPlace then mulInPlace)
__global__ void silu_mul_kernel(float* __restrict__ gate, const float* __restrict__ up, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float x = gate[i];
        gate[i] = x / (1.0f + expf(-x)) * up[i];
    }
}

__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ y, int64_t n) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        x[i] += y[i];
}

// Greedy pick of one row (argmaxOfLastToken, Transformer.kt:255-266): the
// largest logit above -1e9, the lowest index among equal ones, 0 if none.
__global__ void __launch_bounds__(kThreads) argmax_kernel(const float* __restrict__ logits, int n,
                                                          int32_t* __restrict__ out) {
    __shared__ float bv[kThreads];
    __shared__ int bi[kThreads];
    float best = -1e9f;
    int idx = 0x7fffffff;
    for (int v = threadIdx.x; v < n; v += blockDim.x) {
        const float x = logits[static_cast<int64_t>(blockIdx.x) * n + v];
        if (x > best) {  // strictly greater: the first (lowest) index of a tie stays
            best = x;
            idx = v;
        }
    }
    bv[threadIdx.x] = best;
    bi[threadIdx.x] = idx;
    __syncthreads();
    for (int s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            const float ov = bv[threadIdx.x + s];
            const int oi = bi[threadIdx.x + s];
            if (ov > bv[threadIdx.x] || (ov == bv[threadIdx.x] && oi < bi[threadIdx.x])) {
                bv[threadIdx.x] = ov;
                bi[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) out[blockIdx.x] = bi[0] == 0x7fffffff ? 0 : bi[0];
}

// dequantizeColumn(token) of a weight [K x N] (the tied embedding lookup):
// out[k] = value(k, *col) for k < K.
__global__ void dequantize_column_kernel(QView w, const int32_t* __restrict__ col, float* __restrict__ out,
                                         int32_t* __restrict__ status) {
    const int c = *col;
    if (c < 0 || c >= w.columns) {
        if (blockIdx.x == 0 && threadIdx.x == 0 && status != nullptr) atomicOr(status, KT_ERR_INVALID_ARGUMENT);
        return;
    }
    for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < w.rows; k += gridDim.x * blockDim.x) {
        const int64_t g = static_cast<int64_t>(k / w.group_size) * w.columns + c;
        float v;
        if (w.bits == 8) {
            v = __fmul_rn(w.scales[g], static_cast<float>(static_cast<int8_t>(w.q[static_cast<int64_t>(k) * w.bytes_per_row + c])));
        } else {
            const int half = w.bytes_per_row;
            const uint8_t b = w.q[static_cast<int64_t>(k) * half + (c < half ? c : c - half)];
            const int q = c < half ? (b & 15) : (b >> 4);
            v = __fmul_rn(w.scales[g], static_cast<float>(q - static_cast<int>(w.zeros[g])));
        }
        out[k] = v;
    }
}

__global__ void increment_kernel(int32_t* p, int32_t delta) { *p += delta; }

int grid_for(int64_t n) { return static_cast<int>(std::min<int64_t>((n + kThreads - 1) / kThreads, 148 * 8)); }

}  // namespace

cudaError_t launch_rmsnorm(const float* x, const float* w, float* out, int rows, int dim, float eps, cudaStream_t s) {
    rmsnorm_kernel<<<rows, kThreads, 0, s>>>(x, w, out, dim, eps);
    return cudaGetLastError();
}
cudaError_t launch_rope(float* v, int rows, int width, int head_dim, const float* inv_freq, const int32_t* pos,
                        cudaStream_t s) {
    rope_kernel<<<grid_for(static_cast<int64_t>(rows) * width / 2), kThreads, 0, s>>>(v, rows, width, head_dim,
                                                                                       inv_freq, pos);
    return cudaGetLastError();
}
cudaError_t launch_kv_store(const float* k, const float* v, float* kc, float* vc, int rows, int kv_heads, int head_dim,
                            int max_seq, int layer, const int32_t* pos, cudaStream_t s) {
    kv_store_kernel<<<grid_for(static_cast<int64_t>(rows) * kv_heads * head_dim), kThreads, 0, s>>>(
        k, v, kc, vc, rows, kv_heads, head_dim, max_seq, layer, pos);
    return cudaGetLastError();
}
cudaError_t launch_attention_decode(const float* q, const float* kc, const float* vc, float* ctx, float* scores,
                                    int heads, int kv_heads, int head_dim, int max_seq, int layer, float scale,
                                    const int32_t* pos, cudaStream_t s) {
    attention_decode_kernel<<<heads, kThreads, head_dim * sizeof(float), s>>>(q, kc, vc, ctx, scores, heads, kv_heads,
                                                                              head_dim, max_seq, layer, scale, pos);
    return cudaGetLastError();
}
cudaError_t launch_silu_mul(float* gate, const float* up, int64_t n, cudaStream_t s) {
    silu_mul_kernel<<<grid_for(n), kThreads, 0, s>>>(gate, up, n);
    return cudaGetLastError();
}
cudaError_t launch_add(float* x, const float* y, int64_t n, cudaStream_t s) {
    add_kernel<<<grid_for(n), kThreads, 0, s>>>(x, y, n);
    return cudaGetLastError();
}
cudaError_t launch_argmax(const float* logits, int rows, int n, int32_t* out, cudaStream_t s) {
    argmax_kernel<<<rows, kThreads, 0, s>>>(logits, n, out);
    return cudaGetLastError();
}
cudaError_t launch_dequantize_column(const QView& w, const int32_t* col, float* out, int32_t* status, cudaStream_t s) {
    dequantize_column_kernel<<<grid_for(w.rows), kThreads, 0, s>>>(w, col, out, status);
    return cudaGetLastError();
}
cudaError_t launch_increment(int32_t* p, int32_t delta, cudaStream_t s) {
    increment_kernel<<<1, 1, 0, s>>>(p, delta);
    return cudaGetLastError();
}

}  // namespace kt
