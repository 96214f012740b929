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
#include <algorithm>
#include <atomic>
#include <cfloat>
#include <cstdlib>

#include "kt_device.cuh"
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
    dev::pdl_wait();  // inputs may come from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
    __shared__ float red[32];
    const float* xr = x + static_cast<int64_t>(blockIdx.x) * dim;
    float* orow = out + static_cast<int64_t>(blockIdx.x) * dim;
    float ss = 0.0f;
    for (int d = threadIdx.x; d < dim; d += blockDim.x) ss = fmaf(xr[d], xr[d], ss);
    ss = block_sum(ss, red);
    const float r = 1.0f / sqrtf(ss / static_cast<float>(dim) + eps);
    for (int d = threadIdx.x; d < dim; d += blockDim.x) orow[d] = xr[d] * r * w[d];
}

constexpr int kRowRegs = 16;  // rows of up to kThreads * 16 values are normalised from registers

// x += y, then out = RMSNorm(x) (the residual add of TransformerBlock.decodeInto
// followed by the next norm), one block per row.
__global__ void __launch_bounds__(kThreads) add_rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ y,
                                                              const float* __restrict__ w, float* __restrict__ out,
                                                              int dim, float eps) {
    dev::pdl_wait();  // inputs may come from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
    __shared__ float red[32];
    float* xr = x + static_cast<int64_t>(blockIdx.x) * dim;
    const float* yr = y + static_cast<int64_t>(blockIdx.x) * dim;
    float* orow = out + static_cast<int64_t>(blockIdx.x) * dim;
    float ss = 0.0f;
    if (dim <= kThreads * kRowRegs) {
        // the row stays in registers between the sum of squares and the scaling
        float v[kRowRegs];
#pragma unroll
        for (int i = 0; i < kRowRegs; ++i) {
            const int d = threadIdx.x + i * kThreads;
            v[i] = d < dim ? xr[d] + yr[d] : 0.0f;
            if (d < dim) xr[d] = v[i];
            ss = fmaf(v[i], v[i], ss);
        }
        ss = block_sum(ss, red);
        const float r = 1.0f / sqrtf(ss / static_cast<float>(dim) + eps);
#pragma unroll
        for (int i = 0; i < kRowRegs; ++i) {
            const int d = threadIdx.x + i * kThreads;
            if (d < dim) orow[d] = v[i] * r * w[d];
        }
        return;
    }
    for (int d = threadIdx.x; d < dim; d += blockDim.x) {
        const float v = xr[d] + yr[d];
        xr[d] = v;
        ss = fmaf(v, v, ss);
    }
    ss = block_sum(ss, red);  // its barriers also order the x writes before the reads below
    const float r = 1.0f / sqrtf(ss / static_cast<float>(dim) + eps);
    for (int d = threadIdx.x; d < dim; d += blockDim.x) orow[d] = xr[d] * r * w[d];
}

// RoPE on the q and k parts of fused q|k|v rows (row r at position *pos + r),
// then the k and v parts into the cache (Attention.decodeInto / prefillInto,
// Attention.kt:222-232, :256-276).  blockIdx.y = row.
__global__ void rope_kv_kernel(float* __restrict__ qkv, int q_width, int kv_heads, int head_dim,
                               const float* __restrict__ inv_freq, float* __restrict__ kc, float* __restrict__ vc,
                               int max_seq, int layer, const int32_t* __restrict__ pos, int rows_per_seq,
                               int64_t cache_stride) {
    dev::pdl_wait();  // inputs may come from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
    const int half = head_dim / 2;
    const int kv_width = kv_heads * head_dim;
    const int rope_pairs = (q_width + kv_width) / 2;  // pairs over the q heads then the k heads
    const int r = blockIdx.y;
    const int seq = r / rows_per_seq;
    const int p = *pos + (r - seq * rows_per_seq);
    kc += seq * cache_stride;
    vc += seq * cache_stride;
    float* row = qkv + static_cast<int64_t>(r) * (q_width + 2 * kv_width);
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < rope_pairs + kv_width; idx += gridDim.x * blockDim.x) {
        if (idx < rope_pairs) {
            const int head = idx / half, i = idx % half;
            float* v = row + head * head_dim;  // q heads, then k heads (contiguous)
            const float theta = static_cast<float>(p) * inv_freq[i];
            float sn, cs;
            sincosf(theta, &sn, &cs);
            const float x1 = v[i], x2 = v[i + half];
            v[i] = x1 * cs - x2 * sn;
            v[i + half] = x1 * sn + x2 * cs;
            if (head * head_dim >= q_width) {  // a key: store both rotated halves
                const int kh = (head * head_dim - q_width) / head_dim;
                const int64_t off = ((static_cast<int64_t>(layer) * kv_heads + kh) * max_seq + p) * head_dim;
                kc[off + i] = v[i];
                kc[off + i + half] = v[i + half];
            }
        } else {
            const int e = idx - rope_pairs;  // a value element
            const int vh = e / head_dim, d = e % head_dim;
            const int64_t off = ((static_cast<int64_t>(layer) * kv_heads + vh) * max_seq + p) * head_dim + d;
            vc[off] = row[q_width + kv_width + e];
        }
    }
}

// RoPE.applyInPlace at position *pos (+ row): pairs (i, i + half) of every head.
__global__ void rope_kernel(float* __restrict__ v, int rows, int width, int head_dim, const float* __restrict__ inv_freq,
                            const int32_t* __restrict__ pos) {
    dev::pdl_wait();  // inputs may come from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
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
    dev::pdl_wait();  // inputs may come from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
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

// attendHead (Attention.kt:295-328) for one query row at position *pos, split
// over the positions (the reference's single softmax restated as a
// log-sum-exp merge): block (head, s) takes positions [s*kSpan, s*kSpan +
// kSpan) up to pos and leaves in scratch[head][s][0 .. head_dim + 2) its local maximum
// m, sum l of exp(score - m) and the unnormalised context acc[d]; the merge
// kernel combines the splits in order: M = max m_s (at least -1e9, the
// reference's initial maximum), ctx = sum acc_s e^(m_s - M) / sum l_s e^(m_s - M).
constexpr int kMaxHeadDim = 254;
constexpr int kSpan = 64;  // positions per block
constexpr int kMaxFusedSplits = 256;  // position blocks the fused decode kernel merges (max_seq <= 16384)

__global__ void __launch_bounds__(kThreads) attention_partial_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
    float* __restrict__ scratch, int heads, int kv_heads, int head_dim, int max_seq, int layer, float scale,
    int q_stride, const int32_t* __restrict__ pos, int rows_per_seq, int64_t cache_stride) {
    dev::pdl_wait();  // inputs may come from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
    __shared__ float red[32];
    // query row t: sequence t / rows_per_seq (its cache cache_stride floats further),
    // position *pos + t % rows_per_seq, attending to 0..that position
    const int t = blockIdx.z;
    const int seq = t / rows_per_seq;
    const int tp = t - seq * rows_per_seq;
    kc += seq * cache_stride;
    vc += seq * cache_stride;
    __shared__ float qs[kMaxHeadDim + 2];
    __shared__ float sc[kSpan];
    __shared__ float part[kThreads / 32][kMaxHeadDim + 2];
    const int h = blockIdx.x, split = blockIdx.y;
    const int j0 = split * kSpan;
    const int j1 = min(j0 + kSpan, *pos + tp + 1);
    if (j0 >= j1) return;  // past the current position: the merge skips this split
    const int group = heads / kv_heads;
    const float* qh = q + static_cast<int64_t>(t) * q_stride + static_cast<int64_t>(h) * head_dim;
    for (int d = threadIdx.x; d < head_dim; d += blockDim.x) qs[d] = qh[d];
    __syncthreads();
    const int64_t base = ((static_cast<int64_t>(layer) * kv_heads + h / group) * max_seq) * head_dim;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    float mx = -FLT_MAX;
    for (int j = j0 + warp; j < j1; j += nw) {
        const float* kr = kc + base + static_cast<int64_t>(j) * head_dim;
        float sdot = 0.0f;
        for (int d = lane; d < head_dim; d += 32) sdot = fmaf(qs[d], kr[d], sdot);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sdot += __shfl_xor_sync(0xffffffffu, sdot, o);
        sdot *= scale;
        if (lane == 0) sc[j - j0] = sdot;
        mx = fmaxf(mx, sdot);
    }
    mx = block_max(mx, red);  // its barriers also publish sc[]
    float sum = 0.0f;
    for (int j = j0 + threadIdx.x; j < j1; j += blockDim.x) {
        const float e = expf(sc[j - j0] - mx);
        sc[j - j0] = e;
        sum += e;
    }
    sum = block_sum(sum, red);
    __syncthreads();
    constexpr int kPer = (kMaxHeadDim + 2 + 31) / 32;
    float acc[kPer];
#pragma unroll
    for (int i = 0; i < kPer; ++i) acc[i] = 0.0f;
    for (int j = j0 + warp; j < j1; j += nw) {
        const float wj = sc[j - j0];
        const float* vr = vc + base + static_cast<int64_t>(j) * head_dim;
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int d = lane + 32 * i;
            if (d < head_dim) acc[i] = fmaf(wj, vr[d], acc[i]);
        }
    }
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
        const int d = lane + 32 * i;
        if (d < head_dim) part[warp][d] = acc[i];
    }
    __syncthreads();
    // this split's partial: scratch[(h * splits + split) * (head_dim + 2) ..]
    const int64_t splits = (max_seq + kSpan - 1) / kSpan;
    float* out = scratch + ((static_cast<int64_t>(t) * heads + h) * splits + split) * (head_dim + 2);
    for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
        float v = 0.0f;
        for (int w = 0; w < nw; ++w) v += part[w][d];
        out[2 + d] = v;
    }
    if (threadIdx.x == 0) {
        out[0] = mx;
        out[1] = sum;
    }
}

// The same partials for the G query heads that share one key/value head
// (grouped-query attention, head h -> kv head h / G), one block per (kv head,
// split, row): each key and value row is read once for the G heads instead of
// once per head.  Warps take positions; a lane holds KPER dims of the G query
// vectors in registers; warp w finishes head w's softmax statistics.
template <int G, int KPER>
__global__ void __launch_bounds__(kThreads) attention_group_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
    float* __restrict__ scratch, int heads, int kv_heads, int head_dim, int max_seq, int layer, float scale,
    int q_stride, const int32_t* __restrict__ pos, int rows_per_seq, int64_t cache_stride) {
    dev::pdl_wait();  // inputs may come from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
    constexpr int kWarps = kThreads / 32;
    static_assert(G <= kWarps, "one warp per query head finishes the statistics");
    __shared__ float sc[G][kSpan];
    __shared__ float stat[G][2];  // max, sum of exponentials
    __shared__ float part[kWarps][G][KPER * 32];
    const int kvh = blockIdx.x, split = blockIdx.y, t = blockIdx.z;
    const int seq = t / rows_per_seq;
    const int tp = t - seq * rows_per_seq;
    kc += seq * cache_stride;
    vc += seq * cache_stride;
    const int j0 = split * kSpan;
    const int j1 = min(j0 + kSpan, *pos + tp + 1);
    if (j0 >= j1) return;  // past the current position: the merge skips this split
    const int n = j1 - j0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float qv[G][KPER];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const float* qh = q + static_cast<int64_t>(t) * q_stride + static_cast<int64_t>(kvh * G + g) * head_dim;
#pragma unroll
        for (int i = 0; i < KPER; ++i) {
            const int d = lane + 32 * i;
            qv[g][i] = d < head_dim ? qh[d] : 0.0f;
        }
    }
    const int64_t base = ((static_cast<int64_t>(layer) * kv_heads + kvh) * max_seq) * head_dim;
    // four of the warp's positions per round: their key rows are loaded before
    // any is used (more bytes in flight per warp on long, many-sequence steps)
    constexpr int kRound = 4;
    for (int jb = j0 + warp; jb < j1; jb += kWarps * kRound) {
        float kv[kRound][KPER];
#pragma unroll
        for (int r = 0; r < kRound; ++r) {
            const int j = jb + kWarps * r;
            const float* kr = kc + base + static_cast<int64_t>(j) * head_dim;
#pragma unroll
            for (int i = 0; i < KPER; ++i) {
                const int d = lane + 32 * i;
                kv[r][i] = j < j1 && d < head_dim ? kr[d] : 0.0f;
            }
        }
#pragma unroll
        for (int r = 0; r < kRound; ++r) {
            const int j = jb + kWarps * r;
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float dot = 0.0f;
#pragma unroll
                for (int i = 0; i < KPER; ++i) dot = fmaf(qv[g][i], kv[r][i], dot);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
                if (lane == 0 && j < j1) sc[g][j - j0] = dot * scale;
            }
        }
    }
    __syncthreads();
    if (warp < G) {  // head `warp`: max and sum of exponentials over this split
        const float s0 = lane < n ? sc[warp][lane] : -FLT_MAX;
        const float s1 = lane + 32 < n ? sc[warp][lane + 32] : -FLT_MAX;
        float mx = fmaxf(s0, s1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float e0 = lane < n ? expf(s0 - mx) : 0.0f;
        const float e1 = lane + 32 < n ? expf(s1 - mx) : 0.0f;
        if (lane < n) sc[warp][lane] = e0;
        if (lane + 32 < n) sc[warp][lane + 32] = e1;
        float sum = e0 + e1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) {
            stat[warp][0] = mx;
            stat[warp][1] = sum;
        }
    }
    __syncthreads();
    float acc[G][KPER];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < KPER; ++i) acc[g][i] = 0.0f;
    for (int jb = j0 + warp; jb < j1; jb += kWarps * kRound) {
        float vv[kRound][KPER];
#pragma unroll
        for (int r = 0; r < kRound; ++r) {
            const int j = jb + kWarps * r;
            const float* vr = vc + base + static_cast<int64_t>(j) * head_dim;
#pragma unroll
            for (int i = 0; i < KPER; ++i) {
                const int d = lane + 32 * i;
                vv[r][i] = j < j1 && d < head_dim ? vr[d] : 0.0f;
            }
        }
#pragma unroll
        for (int r = 0; r < kRound; ++r) {
            const int j = jb + kWarps * r;
            if (j < j1) {
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float w = sc[g][j - j0];
#pragma unroll
                    for (int i = 0; i < KPER; ++i) acc[g][i] = fmaf(w, vv[r][i], acc[g][i]);
                }
            }
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < KPER; ++i) part[warp][g][lane + 32 * i] = acc[g][i];
    __syncthreads();
    const int64_t splits = (max_seq + kSpan - 1) / kSpan;
    for (int idx = threadIdx.x; idx < G * head_dim; idx += kThreads) {
        const int g = idx / head_dim, d = idx - g * head_dim;
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += part[w][g][d];
        float* out = scratch + ((static_cast<int64_t>(t) * heads + kvh * G + g) * splits + split) * (head_dim + 2);
        out[2 + d] = v;
        if (d == 0) {
            out[0] = stat[g][0];
            out[1] = stat[g][1];
        }
    }
}

// The same partials as attention_group_kernel for head_dim 64 and 128 with
// 16-byte aligned cache rows, the split's key and value rows staged in shared
// memory by bulk copies issued before any arithmetic (64 positions: 32 or 64
// KB in flight per block at once, where register loads keep a few KB per
// warp), one block per (kv head, split, row).  Scores: lane l of a warp takes
// position l of its half of the split and a quarter of the dims (the key rows
// land 4 floats apart, so 32 lanes reading one column offset hit every bank
// once per wavefront; the query is a broadcast), the four quarters summed in
// order.  Values: warp w takes positions w, w + 8, ..., a lane holds HD / 32
// dims of the G heads.  Waits on the copies are bounded: on a timeout the
// block sets the error word, drains its copies (again bounded) and returns.
template <int HD>
struct StagedAttention {
    // head_dim 128: the key tile arrives as one bulk copy (rows 512 bytes apart)
    // and lane l reads float4 chunk (i + l) mod 8 of its quarter row at step i, so
    // 8 consecutive lanes cover all 32 banks; head_dim 64 (quarters of 4 chunks):
    // one copy per row, rows landing 4 floats apart
    static constexpr bool kRot = HD == 128;
    static constexpr int kPad = kRot ? HD : HD + 4;  // floats between staged key rows
    static constexpr int kQuarter = HD / 4;
    __device__ static int chunk(int c, int lane) {
        return kRot ? (((c >> 2) + lane) & (kQuarter / 4 - 1)) << 2 : c;
    }
    template <int G>
    static constexpr size_t smem_bytes() {
        return sizeof(float) * (static_cast<size_t>(kSpan) * kPad + kSpan * HD + G * HD + 4 * G * kSpan + kSpan * G);
    }
};

template <int G, int HD>
__global__ void __launch_bounds__(kThreads) attention_group_staged_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
    float* __restrict__ scratch, int heads, int kv_heads, int max_seq, int layer, float scale, int q_stride,
    const int32_t* __restrict__ pos, int rows_per_seq, int64_t cache_stride, int32_t* __restrict__ err) {
    using S = StagedAttention<HD>;
    constexpr int kWarps = kThreads / 32;
    static_assert(G <= kWarps && G * HD <= kSpan * S::kPad / kWarps, "one warp per head; partials fit the key area");
    extern __shared__ __align__(16) float sm[];
    float* ks = sm;                         // [kSpan][kPad]
    float* vs = ks + kSpan * S::kPad;       // [kSpan][HD]
    float* qs = vs + kSpan * HD;            // [G][HD]
    float* sp = qs + G * HD;                // [4][G][kSpan] score quarters
    float* pw = sp + 4 * G * kSpan;         // [kSpan][G] exp(score - max)
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ float stat[G][2];
    dev::pdl_wait();  // the cache rows and q may come from the previous kernel
    dev::pdl_launch_dependents();
    const int kvh = blockIdx.x, split = blockIdx.y, t = blockIdx.z;
    const int seq = t / rows_per_seq;
    const int tp = t - seq * rows_per_seq;
    const int j0 = split * kSpan;
    const int j1 = min(j0 + kSpan, *pos + tp + 1);
    if (j0 >= j1) return;  // past the current position: the merge skips this split
    const int n = j1 - j0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t base =
        seq * cache_stride + ((static_cast<int64_t>(layer) * kv_heads + kvh) * max_seq + j0) * HD;
    const uint32_t bar_k = dev::smem_u32(&bars[0]), bar_v = dev::smem_u32(&bars[1]);
    if (threadIdx.x == 0) {
        dev::mbar_init(bar_k, 1);
        dev::mbar_init(bar_v, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (warp == 0) {
        if (lane == 0) {
            dev::mbar_expect_tx(bar_k, static_cast<uint32_t>(n * HD * sizeof(float)));
            dev::mbar_expect_tx(bar_v, static_cast<uint32_t>(n * HD * sizeof(float)));
            dev::bulk_load(dev::smem_u32(vs), vc + base, static_cast<uint32_t>(n * HD * sizeof(float)), bar_v);
        }
        __syncwarp();
        if constexpr (S::kRot) {
            if (lane == 0)
                dev::bulk_load(dev::smem_u32(ks), kc + base, static_cast<uint32_t>(n * HD * sizeof(float)), bar_k);
        } else {
            for (int j = lane; j < n; j += 32)
                dev::bulk_load(dev::smem_u32(ks + j * S::kPad), kc + base + static_cast<int64_t>(j) * HD,
                               HD * sizeof(float), bar_k);
        }
    }
    const float* qh = q + static_cast<int64_t>(t) * q_stride + static_cast<int64_t>(kvh) * G * HD;
    for (int i = threadIdx.x; i < G * HD; i += kThreads) qs[i] = qh[i];
    __syncthreads();  // qs
    bool ok = dev::mbar_wait_bounded(bar_k, 0);
    if (__syncthreads_or(!ok)) {
        if (threadIdx.x == 0) {
            atomicOr(err, 1);
            dev::mbar_wait_bounded(bar_k, 0);  // copies still in flight land before the block exits
            dev::mbar_wait_bounded(bar_v, 0);
        }
        return;
    }
    {   // score quarters: lane -> position, warp -> (half of the positions, quarter of the dims)
        // four running sums per head (dims 4i, 4i+1, 4i+2, 4i+3 of the quarter),
        // added pairwise at the end: short dependency chains, and rounding
        // closer to a tree sum than one chain of HD / 4
        const int j = (warp & 1) * 32 + lane, dq = warp >> 1;
        float acc[G][4];
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[g][e] = 0.0f;
        if (j < n) {
            const float* kr = ks + j * S::kPad + dq * S::kQuarter;
            const float* qq = qs + dq * S::kQuarter;
#pragma unroll
            for (int c = 0; c < S::kQuarter; c += 4) {
                const int cc = S::chunk(c, lane);
                const float4 k4 = *reinterpret_cast<const float4*>(kr + cc);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float4 q4 = *reinterpret_cast<const float4*>(qq + g * HD + cc);
                    acc[g][0] = fmaf(q4.x, k4.x, acc[g][0]);
                    acc[g][1] = fmaf(q4.y, k4.y, acc[g][1]);
                    acc[g][2] = fmaf(q4.z, k4.z, acc[g][2]);
                    acc[g][3] = fmaf(q4.w, k4.w, acc[g][3]);
                }
            }
#pragma unroll
            for (int g = 0; g < G; ++g)
                sp[(dq * G + g) * kSpan + j] = (acc[g][0] + acc[g][1]) + (acc[g][2] + acc[g][3]);
        }
    }
    __syncthreads();
    if (warp < G) {  // head `warp`: max and sum of exponentials over this split
        const int g = warp;
        auto score = [&](int j) {
            return (((sp[(0 * G + g) * kSpan + j] + sp[(1 * G + g) * kSpan + j]) + sp[(2 * G + g) * kSpan + j]) +
                    sp[(3 * G + g) * kSpan + j]) * scale;
        };
        const float s0 = lane < n ? score(lane) : -FLT_MAX;
        const float s1 = lane + 32 < n ? score(lane + 32) : -FLT_MAX;
        float mx = fmaxf(s0, s1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float e0 = lane < n ? expf(s0 - mx) : 0.0f;
        const float e1 = lane + 32 < n ? expf(s1 - mx) : 0.0f;
        pw[lane * G + g] = e0;
        pw[(lane + 32) * G + g] = e1;
        float sum = e0 + e1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) {
            stat[g][0] = mx;
            stat[g][1] = sum;
        }
    }
    ok = dev::mbar_wait_bounded(bar_v, 0);
    if (__syncthreads_or(!ok)) {  // also publishes pw and stat
        if (threadIdx.x == 0) {
            atomicOr(err, 1);
            dev::mbar_wait_bounded(bar_v, 0);
        }
        return;
    }
    constexpr int kDims = HD / 32;  // per lane: 2 or 4 consecutive dims
    float acc[G][kDims];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < kDims; ++i) acc[g][i] = 0.0f;
    for (int j = warp; j < n; j += kWarps) {
        float v[kDims];
        if constexpr (kDims == 4) {
            const float4 v4 = *reinterpret_cast<const float4*>(vs + j * HD + 4 * lane);
            v[0] = v4.x, v[1] = v4.y, v[2] = v4.z, v[3] = v4.w;
        } else {
            const float2 v2 = *reinterpret_cast<const float2*>(vs + j * HD + 2 * lane);
            v[0] = v2.x, v[1] = v2.y;
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float w = pw[j * G + g];
#pragma unroll
            for (int i = 0; i < kDims; ++i) acc[g][i] = fmaf(w, v[i], acc[g][i]);
        }
    }
    float* part = ks;  // [kWarps][G][HD]; the key rows are no longer read
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < kDims; ++i) part[(warp * G + g) * HD + kDims * lane + i] = acc[g][i];
    __syncthreads();
    const int64_t splits = (max_seq + kSpan - 1) / kSpan;
    for (int idx = threadIdx.x; idx < G * HD; idx += kThreads) {
        const int g = idx / HD, d = idx - g * HD;
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += part[(w * G + g) * HD + d];
        float* out = scratch + ((static_cast<int64_t>(t) * heads + kvh * G + g) * splits + split) * (HD + 2);
        out[2 + d] = v;
        if (d == 0) {
            out[0] = stat[g][0];
            out[1] = stat[g][1];
        }
    }
}

// One decode token per sequence (row t = sequence t, at position *pos), the
// whole of Attention.decodeInto's middle in one launch: each block (kv head,
// split, row) applies RoPE to its G query heads (RoPE.applyInPlace, RoPE.kt:
// 117-137, the rope kernel's arithmetic), the block whose split holds the
// current position also rotates this kv head's key and stores key and value in
// the cache (KVCache layout) before reading it, every active block writes its
// split's partials (max, sum of exponentials, weighted values), and the last
// active block of the (kv head, row) to finish -- an acq_rel ticket -- merges
// the splits in split order into the context (deterministic).  Every ticket is
// back at zero when the launch ends.  Rows of one sequence that attend to each
// other's new keys (a prefill) keep the separate rope / store and attention
// kernels.
template <int G, int HD>
__global__ void __launch_bounds__(kThreads) attention_decode_fused_kernel(
    const float* __restrict__ qkv, int q_width, const float* __restrict__ inv_freq, float* __restrict__ kc,
    float* __restrict__ vc, float* __restrict__ scratch, int32_t* __restrict__ tickets, float* __restrict__ ctx,
    int heads, int kv_heads, int head_dim, int max_seq, int layer, float scale, const int32_t* __restrict__ pos,
    int64_t cache_stride) {
    dev::pdl_wait();  // qkv comes from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
    constexpr int kWarps = kThreads / 32;
    static_assert(G <= kWarps, "one warp per query head finishes the statistics");
    static_assert(HD % 4 == 0 && HD <= 128 && kThreads % HD == 0, "head_dim layout");
    constexpr int kQ = HD / 4;                 // dims of a key row per thread (4 threads per position)
    constexpr int kPG = kThreads / HD;         // position groups of the value pass
    __shared__ __align__(16) float qs[G][HD];  // the rotated query heads
    __shared__ float sc[G][kSpan];
    __shared__ float stat[G][2];               // max, sum of exponentials
    __shared__ float part[kPG][G][HD];
    __shared__ int s_last;
    const int kvh = blockIdx.x, split = blockIdx.y, t = blockIdx.z;
    const int p = *pos;
    const int j0 = split * kSpan;
    const int j1 = min(j0 + kSpan, p + 1);
    if (j0 >= j1) return;  // past the current position
    kc += t * cache_stride;
    vc += t * cache_stride;
    const int n = j1 - j0;
    constexpr int half = HD / 2;
    const int kv_width = kv_heads * HD;
    const float* row = qkv + static_cast<int64_t>(t) * (q_width + 2 * kv_width);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t base = ((static_cast<int64_t>(layer) * kv_heads + kvh) * max_seq) * HD;
    // RoPE of element d of a head vector v at position p (the rope kernel's arithmetic)
    auto rotated = [&](const float* v, int d) {
        const int i = d < half ? d : d - half;
        float s1, c1;
        sincosf(static_cast<float>(p) * __ldg(inv_freq + i), &s1, &c1);
        const float x1 = v[i], x2 = v[i + half];
        return d < half ? x1 * c1 - x2 * s1 : x1 * s1 + x2 * c1;
    };
    if (j1 == p + 1) {  // this split holds the current position: its key and value into the cache
        const float* kr = row + q_width + kvh * HD;
        const float* vr = row + q_width + kv_width + kvh * HD;
        const int64_t off = base + static_cast<int64_t>(p) * HD;
        for (int d = threadIdx.x; d < HD; d += kThreads) {
            kc[off + d] = rotated(kr, d);
            vc[off + d] = vr[d];
        }
    }
    for (int idx = threadIdx.x; idx < G * HD; idx += kThreads) {
        const int g = idx / HD, d = idx - g * HD;
        qs[g][d] = rotated(row + static_cast<int64_t>(kvh * G + g) * HD, d);
    }
    __syncthreads();  // the query heads, and the block's own cache stores, visible to the block
    // scores: four threads per position, each a quarter of the key row
    {
        const int jp = threadIdx.x >> 2, qd = threadIdx.x & 3;
        const int j = j0 + jp;
        float kq[kQ];
        const float* kr = kc + base + static_cast<int64_t>(j) * HD + qd * kQ;
#pragma unroll
        for (int i = 0; i < kQ; i += 4) {
            const float4 k4 = j < j1 ? *reinterpret_cast<const float4*>(kr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            kq[i] = k4.x;
            kq[i + 1] = k4.y;
            kq[i + 2] = k4.z;
            kq[i + 3] = k4.w;
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float dot = 0.0f;
#pragma unroll
            for (int i = 0; i < kQ; ++i) dot = fmaf(qs[g][qd * kQ + i], kq[i], dot);
            dot += __shfl_xor_sync(0xffffffffu, dot, 1);
            dot += __shfl_xor_sync(0xffffffffu, dot, 2);
            if (qd == 0 && j < j1) sc[g][jp] = dot * scale;
        }
    }
    __syncthreads();
    if (warp < G) {  // head `warp`: max and sum of exponentials over this split
        const float s0 = lane < n ? sc[warp][lane] : -FLT_MAX;
        const float s1 = lane + 32 < n ? sc[warp][lane + 32] : -FLT_MAX;
        float mx = fmaxf(s0, s1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float e0 = lane < n ? expf(s0 - mx) : 0.0f;
        const float e1 = lane + 32 < n ? expf(s1 - mx) : 0.0f;
        if (lane < n) sc[warp][lane] = e0;
        if (lane + 32 < n) sc[warp][lane + 32] = e1;
        float sum = e0 + e1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) {
            stat[warp][0] = mx;
            stat[warp][1] = sum;
        }
    }
    __syncthreads();
    // weighted values: thread (position group pg, dim d) over positions j0 + pg + kPG i
    {
        const int d = threadIdx.x % HD, pg = threadIdx.x / HD;
        float acc[G];
#pragma unroll
        for (int g = 0; g < G; ++g) acc[g] = 0.0f;
        constexpr int kPer = kSpan / kPG;
        float vv[kPer];
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int j = j0 + pg + kPG * i;
            vv[i] = j < j1 ? vc[base + static_cast<int64_t>(j) * HD + d] : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
            const int jl = pg + kPG * i;
            if (j0 + jl < j1) {
#pragma unroll
                for (int g = 0; g < G; ++g) acc[g] = fmaf(sc[g][jl], vv[i], acc[g]);
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) part[pg][g][d] = acc[g];
    }
    __syncthreads();
    const int64_t splits = (max_seq + kSpan - 1) / kSpan;
    for (int idx = threadIdx.x; idx < G * HD; idx += kThreads) {
        const int g = idx / HD, d = idx - g * HD;
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kPG; ++w) v += part[w][g][d];  // fixed order
        float* out = scratch + ((static_cast<int64_t>(t) * heads + kvh * G + g) * splits + split) * (HD + 2);
        out[2 + d] = v;
        if (d == 0) {
            out[0] = stat[g][0];
            out[1] = stat[g][1];
        }
    }
    // the last of the row's active splits to arrive merges them (the barrier
    // orders every thread's partial stores before thread 0's acq_rel ticket)
    const int active = p / kSpan + 1;
    __syncthreads();
    if (threadIdx.x == 0) {
        int32_t* ticket = tickets + static_cast<int64_t>(t) * kv_heads + kvh;
        s_last = active == 1 || dev::atomic_add_acq_rel(ticket, 1) == active - 1;
        if (s_last && active > 1) *ticket = 0;  // every split has arrived: ready for the next launch
    }
    __syncthreads();
    if (!s_last) return;
    // merge: warp g loads head g's split statistics, takes the maximum and the
    // sum of exponentials (fixed reduction order) and keeps each split's factor
    // in shared memory; then each thread sums the splits' values for its
    // outputs with every load of a chunk of 8 splits in flight at once
    constexpr int stride = HD + 2;
    __shared__ float coef[G][kMaxFusedSplits];
    __shared__ float inv_l[G];
    if (warp < G) {
        const float* hb = scratch + (static_cast<int64_t>(t) * heads + kvh * G + warp) * splits * stride;
        float m = -1e9f;
        for (int s2 = lane; s2 < active; s2 += 32) m = fmaxf(m, __ldcg(hb + s2 * stride));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int s2 = lane; s2 < active; s2 += 32) {
            const float e = expf(__ldcg(hb + s2 * stride) - m);
            coef[warp][s2] = e;
            l = fmaf(__ldcg(hb + s2 * stride + 1), e, l);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) inv_l[warp] = 1.0f / l;
    }
    __syncthreads();
    constexpr int kOuts = (G * HD + kThreads - 1) / kThreads;  // outputs per thread
    float vsum[kOuts];
#pragma unroll
    for (int o2 = 0; o2 < kOuts; ++o2) vsum[o2] = 0.0f;
    for (int s0 = 0; s0 < active; s0 += 8) {
        float u[kOuts][8];
#pragma unroll
        for (int o2 = 0; o2 < kOuts; ++o2) {
            const int idx = threadIdx.x + kThreads * o2;
            const int g = idx / HD, d = idx - g * HD;
            const float* hv = scratch + (static_cast<int64_t>(t) * heads + kvh * G + g) * splits * stride + 2 + d;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                u[o2][j] = idx < G * HD && s0 + j < active ? __ldcg(hv + (s0 + j) * stride) : 0.0f;
        }
#pragma unroll
        for (int o2 = 0; o2 < kOuts; ++o2) {
            const int g = min((threadIdx.x + kThreads * o2) / HD, G - 1);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (s0 + j < active) vsum[o2] = fmaf(u[o2][j], coef[g][s0 + j], vsum[o2]);
        }
    }
#pragma unroll
    for (int o2 = 0; o2 < kOuts; ++o2) {
        const int idx = threadIdx.x + kThreads * o2;
        if (idx < G * HD) {
            const int g = idx / HD, d = idx - g * HD;
            ctx[(static_cast<int64_t>(t) * heads + kvh * G + g) * HD + d] = vsum[o2] * inv_l[g];
        }
    }
}

// The same for head_dim 128 with a warp per position (a lane holds KPER dims
// of the G query vectors in registers; key and value rows of the warp's
// positions loaded together), measured faster than the kernel above there.
template <int G, int KPER>
__global__ void __launch_bounds__(kThreads) attention_decode_fused_wide_kernel(
    const float* __restrict__ qkv, int q_width, const float* __restrict__ inv_freq, float* __restrict__ kc,
    float* __restrict__ vc, float* __restrict__ scratch, int32_t* __restrict__ tickets, float* __restrict__ ctx,
    int heads, int kv_heads, int head_dim, int max_seq, int layer, float scale, const int32_t* __restrict__ pos,
    int64_t cache_stride) {
    dev::pdl_wait();  // qkv comes from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
    constexpr int kWarps = kThreads / 32;
    static_assert(G <= kWarps, "one warp per query head finishes the statistics");
    __shared__ float sc[G][kSpan];
    __shared__ float stat[G][2];  // max, sum of exponentials
    __shared__ float part[kWarps][G][KPER * 32];
    __shared__ int s_last;
    const int kvh = blockIdx.x, split = blockIdx.y, t = blockIdx.z;
    const int p = *pos;
    const int j0 = split * kSpan;
    const int j1 = min(j0 + kSpan, p + 1);
    if (j0 >= j1) return;  // past the current position
    kc += t * cache_stride;
    vc += t * cache_stride;
    const int n = j1 - j0;
    const int half = head_dim / 2;
    const int kv_width = kv_heads * head_dim;
    const float* row = qkv + static_cast<int64_t>(t) * (q_width + 2 * kv_width);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t base = ((static_cast<int64_t>(layer) * kv_heads + kvh) * max_seq) * head_dim;
    // RoPE factors of this lane's dims d = lane + 32 i (they depend on the dim only)
    float cs[KPER], sn[KPER];
#pragma unroll
    for (int i = 0; i < KPER; ++i) {
        const int d = lane + 32 * i;
        const int fi = d < half ? d : d - half;
        cs[i] = 1.0f;
        sn[i] = 0.0f;
        if (d < head_dim) sincosf(static_cast<float>(p) * __ldg(inv_freq + fi), &sn[i], &cs[i]);
    }
    if (j1 == p + 1) {  // this split holds the current position: its key and value into the cache
        const float* kr = row + q_width + kvh * head_dim;
        const float* vr = row + q_width + kv_width + kvh * head_dim;
        const int64_t off = base + static_cast<int64_t>(p) * head_dim;
        for (int d = threadIdx.x; d < head_dim; d += kThreads) {
            const int i = d < half ? d : d - half;
            float s1, c1;
            sincosf(static_cast<float>(p) * __ldg(inv_freq + i), &s1, &c1);
            const float x1 = kr[i], x2 = kr[i + half];
            kc[off + d] = d < half ? x1 * c1 - x2 * s1 : x1 * s1 + x2 * c1;
            vc[off + d] = vr[d];
        }
        __syncthreads();  // the block's stores are visible to its own reads below
    }
    // the G query vectors: every load issued first (no load waits on another),
    // then the rotation pairs (d, d + half) -- in this lane's registers when
    // half is a multiple of 32, else loaded beside them
    float qv[G][KPER], qp[G][KPER];
    const bool in_lane = (half & 31) == 0;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const float* qh = row + static_cast<int64_t>(kvh * G + g) * head_dim;
#pragma unroll
        for (int i = 0; i < KPER; ++i) {
            const int d = lane + 32 * i;
            qv[g][i] = d < head_dim ? qh[d] : 0.0f;
            qp[g][i] = !in_lane && d < head_dim ? qh[d < half ? d + half : d - half] : 0.0f;
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float rq[KPER];
#pragma unroll
        for (int i = 0; i < KPER; ++i) {
            const int d = lane + 32 * i;
            const int sh = half >> 5;  // partner element index offset when in_lane
            const float partner = in_lane ? qv[g][d < half ? min(i + sh, KPER - 1) : max(i - sh, 0)] : qp[g][i];
            const float x1 = d < half ? qv[g][i] : partner, x2 = d < half ? partner : qv[g][i];
            rq[i] = d < head_dim ? (d < half ? x1 * cs[i] - x2 * sn[i] : x1 * sn[i] + x2 * cs[i]) : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < KPER; ++i) qv[g][i] = rq[i];
    }
    // a warp's positions j0 + warp + 8 jj: their key and value rows are loaded
    // together (one memory round trip), the value rows kept in registers until
    // the softmax weights are known
    constexpr int kPer = kSpan / kWarps;  // positions per warp
    float kr_[kPer][KPER], vr_[kPer][KPER];
#pragma unroll
    for (int jj = 0; jj < kPer; ++jj) {
        const int j = j0 + warp + kWarps * jj;
        const float* kr = kc + base + static_cast<int64_t>(j) * head_dim;
        const float* vr = vc + base + static_cast<int64_t>(j) * head_dim;
#pragma unroll
        for (int i = 0; i < KPER; ++i) {
            const int d = lane + 32 * i;
            const bool ok = j < j1 && d < head_dim;
            kr_[jj][i] = ok ? kr[d] : 0.0f;
            vr_[jj][i] = ok ? vr[d] : 0.0f;
        }
    }
#pragma unroll
    for (int jj = 0; jj < kPer; ++jj) {
        const int j = j0 + warp + kWarps * jj;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float dot = 0.0f;
#pragma unroll
            for (int i = 0; i < KPER; ++i) dot = fmaf(qv[g][i], kr_[jj][i], dot);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            if (lane == 0 && j < j1) sc[g][j - j0] = dot * scale;
        }
    }
    __syncthreads();
    if (warp < G) {  // head `warp`: max and sum of exponentials over this split
        const float s0 = lane < n ? sc[warp][lane] : -FLT_MAX;
        const float s1 = lane + 32 < n ? sc[warp][lane + 32] : -FLT_MAX;
        float mx = fmaxf(s0, s1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float e0 = lane < n ? expf(s0 - mx) : 0.0f;
        const float e1 = lane + 32 < n ? expf(s1 - mx) : 0.0f;
        if (lane < n) sc[warp][lane] = e0;
        if (lane + 32 < n) sc[warp][lane + 32] = e1;
        float sum = e0 + e1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) {
            stat[warp][0] = mx;
            stat[warp][1] = sum;
        }
    }
    __syncthreads();
    float acc[G][KPER];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < KPER; ++i) acc[g][i] = 0.0f;
#pragma unroll
    for (int jj = 0; jj < kPer; ++jj) {
        const int j = j0 + warp + kWarps * jj;
        if (j < j1) {
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float w = sc[g][j - j0];
#pragma unroll
                for (int i = 0; i < KPER; ++i) acc[g][i] = fmaf(w, vr_[jj][i], acc[g][i]);
            }
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < KPER; ++i) part[warp][g][lane + 32 * i] = acc[g][i];
    __syncthreads();
    const int64_t splits = (max_seq + kSpan - 1) / kSpan;
    for (int idx = threadIdx.x; idx < G * head_dim; idx += kThreads) {
        const int g = idx / head_dim, d = idx - g * head_dim;
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += part[w][g][d];
        float* out = scratch + ((static_cast<int64_t>(t) * heads + kvh * G + g) * splits + split) * (head_dim + 2);
        out[2 + d] = v;
        if (d == 0) {
            out[0] = stat[g][0];
            out[1] = stat[g][1];
        }
    }
    // the last of the row's active splits to arrive merges them (the barrier
    // orders every thread's partial stores before thread 0's acq_rel ticket)
    const int active = p / kSpan + 1;
    __syncthreads();
    if (threadIdx.x == 0) {
        int32_t* ticket = tickets + static_cast<int64_t>(t) * kv_heads + kvh;
        s_last = active == 1 || dev::atomic_add_acq_rel(ticket, 1) == active - 1;
        if (s_last && active > 1) *ticket = 0;  // every split has arrived: ready for the next launch
    }
    __syncthreads();
    if (!s_last) return;
    // merge: warp g loads head g's split statistics (32 splits per lane
    // round), takes the maximum and the sum of exponentials (fixed reduction
    // order) and keeps each split's factor in shared memory; then each thread
    // sums the splits' values for its outputs with every load of a chunk of 8
    // splits in flight at once
    const int stride = head_dim + 2;
    __shared__ float coef[G][kMaxFusedSplits];
    __shared__ float inv_l[G];
    if (warp < G) {
        const float* hb = scratch + (static_cast<int64_t>(t) * heads + kvh * G + warp) * splits * stride;
        float m = -1e9f;
        for (int s2 = lane; s2 < active; s2 += 32) m = fmaxf(m, __ldcg(hb + s2 * stride));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int s2 = lane; s2 < active; s2 += 32) {
            const float e = expf(__ldcg(hb + s2 * stride) - m);
            coef[warp][s2] = e;
            l = fmaf(__ldcg(hb + s2 * stride + 1), e, l);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) inv_l[warp] = 1.0f / l;
    }
    __syncthreads();
    constexpr int kOuts = (G * KPER * 32 + kThreads - 1) / kThreads;  // outputs per thread
    float vsum[kOuts];
#pragma unroll
    for (int o2 = 0; o2 < kOuts; ++o2) vsum[o2] = 0.0f;
    for (int s0 = 0; s0 < active; s0 += 8) {
        float u[kOuts][8];
#pragma unroll
        for (int o2 = 0; o2 < kOuts; ++o2) {
            const int idx = threadIdx.x + kThreads * o2;
            const int g = idx / head_dim, d = idx - g * head_dim;
            const float* hv =
                scratch + (static_cast<int64_t>(t) * heads + kvh * G + g) * splits * stride + 2 + d;
#pragma unroll
            for (int j = 0; j < 8; ++j) u[o2][j] = idx < G * head_dim && s0 + j < active ? __ldcg(hv + (s0 + j) * stride) : 0.0f;
        }
#pragma unroll
        for (int o2 = 0; o2 < kOuts; ++o2) {
            const int g = min((threadIdx.x + kThreads * o2) / head_dim, G - 1);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (s0 + j < active) vsum[o2] = fmaf(u[o2][j], coef[g][s0 + j], vsum[o2]);
        }
    }
#pragma unroll
    for (int o2 = 0; o2 < kOuts; ++o2) {
        const int idx = threadIdx.x + kThreads * o2;
        if (idx < G * head_dim) {
            const int g = idx / head_dim, d = idx - g * head_dim;
            ctx[(static_cast<int64_t>(t) * heads + kvh * G + g) * head_dim + d] = vsum[o2] * inv_l[g];
        }
    }
}

// The fused decode step of attention_decode_fused_kernel (RoPE of the query
// heads, the current key / value into the cache, the split partials, the
// last block's merge) with the split's key and value rows staged in shared
// memory by bulk copies, as attention_group_staged_kernel: the copies of the
// cached rows start before anything else; the block holding the current
// position writes that row into the cache and into its staged tile itself.
// Waits on the copies are bounded (error word, drain, return).
template <int G, int HD>
__global__ void __launch_bounds__(kThreads) attention_decode_staged_kernel(
    const float* __restrict__ qkv, int q_width, const float* __restrict__ inv_freq, float* __restrict__ kc,
    float* __restrict__ vc, float* __restrict__ scratch, int32_t* __restrict__ tickets, float* __restrict__ ctx,
    int heads, int kv_heads, int max_seq, int layer, float scale, const int32_t* __restrict__ pos,
    int64_t cache_stride, int32_t* __restrict__ err) {
    using S = StagedAttention<HD>;
    constexpr int kWarps = kThreads / 32;
    static_assert(G <= kWarps && G * HD <= kSpan * S::kPad / kWarps, "one warp per head; partials fit the key area");
    static_assert(G * kMaxFusedSplits + G <= kSpan * S::kPad, "merge factors fit the key area");
    extern __shared__ __align__(16) float sm[];
    float* ks = sm;                         // [kSpan][kPad]
    float* vs = ks + kSpan * S::kPad;       // [kSpan][HD]
    float* qs = vs + kSpan * HD;            // [G][HD] rotated query heads
    float* sp = qs + G * HD;                // [4][G][kSpan] score quarters
    float* pw = sp + 4 * G * kSpan;         // [kSpan][G] exp(score - max)
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ float stat[G][2];
    __shared__ int s_last;
    dev::pdl_wait();  // qkv comes from the previous kernel; the cache rows from earlier steps
    dev::pdl_launch_dependents();
    const int kvh = blockIdx.x, split = blockIdx.y, t = blockIdx.z;
    const int p = *pos;
    const int j0 = split * kSpan;
    const int j1 = min(j0 + kSpan, p + 1);
    if (j0 >= j1) return;  // past the current position
    const int n = j1 - j0;
    const bool holds_current = j1 == p + 1;
    const int n_old = holds_current ? n - 1 : n;  // rows already in the cache
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t base = t * cache_stride + ((static_cast<int64_t>(layer) * kv_heads + kvh) * max_seq + j0) * HD;
    const uint32_t bar_k = dev::smem_u32(&bars[0]), bar_v = dev::smem_u32(&bars[1]);
    if (threadIdx.x == 0) {
        dev::mbar_init(bar_k, 1);
        dev::mbar_init(bar_v, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (warp == 0) {
        const uint32_t bytes = static_cast<uint32_t>(n_old * HD * sizeof(float));
        if (lane == 0) {
            dev::mbar_expect_tx(bar_k, bytes);
            dev::mbar_expect_tx(bar_v, bytes);
            if (n_old > 0) dev::bulk_load(dev::smem_u32(vs), vc + base, bytes, bar_v);
        }
        __syncwarp();
        if constexpr (S::kRot) {
            if (lane == 0 && n_old > 0) dev::bulk_load(dev::smem_u32(ks), kc + base, bytes, bar_k);
        } else {
            for (int j = lane; j < n_old; j += 32)
                dev::bulk_load(dev::smem_u32(ks + j * S::kPad), kc + base + static_cast<int64_t>(j) * HD,
                               HD * sizeof(float), bar_k);
        }
    }
    constexpr int half = HD / 2;
    const int kv_width = kv_heads * HD;
    const float* row = qkv + static_cast<int64_t>(t) * (q_width + 2 * kv_width);
    // RoPE of element d of a head vector v at position p (the rope kernel's arithmetic)
    auto rotated = [&](const float* v, int d) {
        const int i = d < half ? d : d - half;
        float s1, c1;
        sincosf(static_cast<float>(p) * __ldg(inv_freq + i), &s1, &c1);
        const float x1 = v[i], x2 = v[i + half];
        return d < half ? x1 * c1 - x2 * s1 : x1 * s1 + x2 * c1;
    };
    if (holds_current) {  // this step's key and value: into the cache and the staged tile
        const float* kr = row + q_width + kvh * HD;
        const float* vr = row + q_width + kv_width + kvh * HD;
        const int64_t off = base + static_cast<int64_t>(n - 1) * HD;
        for (int d = threadIdx.x; d < HD; d += kThreads) {
            const float kd = rotated(kr, d), vd = vr[d];
            kc[off + d] = kd;
            vc[off + d] = vd;
            ks[(n - 1) * S::kPad + d] = kd;
            vs[(n - 1) * HD + d] = vd;
        }
    }
    for (int idx = threadIdx.x; idx < G * HD; idx += kThreads) {
        const int g = idx / HD, d = idx - g * HD;
        qs[idx] = rotated(row + static_cast<int64_t>(kvh * G + g) * HD, d);
    }
    bool ok = dev::mbar_wait_bounded(bar_k, 0);
    if (__syncthreads_or(!ok)) {  // also publishes qs and the current row
        if (threadIdx.x == 0) {
            atomicOr(err, 1);
            dev::mbar_wait_bounded(bar_k, 0);
            dev::mbar_wait_bounded(bar_v, 0);
        }
        return;
    }
    {   // score quarters: lane -> position, warp -> (half of the positions, quarter of the dims)
        const int j = (warp & 1) * 32 + lane, dq = warp >> 1;
        float acc[G][4];
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[g][e] = 0.0f;
        if (j < n) {
            const float* kr = ks + j * S::kPad + dq * S::kQuarter;
            const float* qq = qs + dq * S::kQuarter;
#pragma unroll
            for (int c = 0; c < S::kQuarter; c += 4) {
                const int cc = S::chunk(c, lane);
                const float4 k4 = *reinterpret_cast<const float4*>(kr + cc);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float4 q4 = *reinterpret_cast<const float4*>(qq + g * HD + cc);
                    acc[g][0] = fmaf(q4.x, k4.x, acc[g][0]);
                    acc[g][1] = fmaf(q4.y, k4.y, acc[g][1]);
                    acc[g][2] = fmaf(q4.z, k4.z, acc[g][2]);
                    acc[g][3] = fmaf(q4.w, k4.w, acc[g][3]);
                }
            }
#pragma unroll
            for (int g = 0; g < G; ++g)
                sp[(dq * G + g) * kSpan + j] = (acc[g][0] + acc[g][1]) + (acc[g][2] + acc[g][3]);
        }
    }
    __syncthreads();
    if (warp < G) {  // head `warp`: max and sum of exponentials over this split
        const int g = warp;
        auto score = [&](int j) {
            return (((sp[(0 * G + g) * kSpan + j] + sp[(1 * G + g) * kSpan + j]) + sp[(2 * G + g) * kSpan + j]) +
                    sp[(3 * G + g) * kSpan + j]) * scale;
        };
        const float s0 = lane < n ? score(lane) : -FLT_MAX;
        const float s1 = lane + 32 < n ? score(lane + 32) : -FLT_MAX;
        float mx = fmaxf(s0, s1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float e0 = lane < n ? expf(s0 - mx) : 0.0f;
        const float e1 = lane + 32 < n ? expf(s1 - mx) : 0.0f;
        pw[lane * G + g] = e0;
        pw[(lane + 32) * G + g] = e1;
        float sum = e0 + e1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) {
            stat[g][0] = mx;
            stat[g][1] = sum;
        }
    }
    ok = dev::mbar_wait_bounded(bar_v, 0);
    if (__syncthreads_or(!ok)) {  // also publishes pw and stat
        if (threadIdx.x == 0) {
            atomicOr(err, 1);
            dev::mbar_wait_bounded(bar_v, 0);
        }
        return;
    }
    constexpr int kDims = HD / 32;  // per lane: 2 or 4 consecutive dims
    float acc[G][kDims];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < kDims; ++i) acc[g][i] = 0.0f;
    for (int j = warp; j < n; j += kWarps) {
        float v[kDims];
        if constexpr (kDims == 4) {
            const float4 v4 = *reinterpret_cast<const float4*>(vs + j * HD + 4 * lane);
            v[0] = v4.x, v[1] = v4.y, v[2] = v4.z, v[3] = v4.w;
        } else {
            const float2 v2 = *reinterpret_cast<const float2*>(vs + j * HD + 2 * lane);
            v[0] = v2.x, v[1] = v2.y;
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const float w = pw[j * G + g];
#pragma unroll
            for (int i = 0; i < kDims; ++i) acc[g][i] = fmaf(w, v[i], acc[g][i]);
        }
    }
    float* part = ks;  // [kWarps][G][HD]; the key rows are no longer read
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int i = 0; i < kDims; ++i) part[(warp * G + g) * HD + kDims * lane + i] = acc[g][i];
    __syncthreads();
    const int64_t splits = (max_seq + kSpan - 1) / kSpan;
    for (int idx = threadIdx.x; idx < G * HD; idx += kThreads) {
        const int g = idx / HD, d = idx - g * HD;
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += part[(w * G + g) * HD + d];
        float* out = scratch + ((static_cast<int64_t>(t) * heads + kvh * G + g) * splits + split) * (HD + 2);
        out[2 + d] = v;
        if (d == 0) {
            out[0] = stat[g][0];
            out[1] = stat[g][1];
        }
    }
    // the last of the row's active splits to arrive merges them (the barrier
    // orders every thread's partial stores before thread 0's acq_rel ticket)
    const int active = p / kSpan + 1;
    __syncthreads();
    if (threadIdx.x == 0) {
        int32_t* ticket = tickets + static_cast<int64_t>(t) * kv_heads + kvh;
        s_last = active == 1 || dev::atomic_add_acq_rel(ticket, 1) == active - 1;
        if (s_last && active > 1) *ticket = 0;  // every split has arrived: ready for the next launch
    }
    __syncthreads();
    if (!s_last) return;
    // merge (attention_decode_fused_kernel's): split factors in the key area
    constexpr int stride = HD + 2;
    float* coef = ks;                         // [G][kMaxFusedSplits]
    float* inv_l = ks + G * kMaxFusedSplits;  // [G]
    if (warp < G) {
        const float* hb = scratch + (static_cast<int64_t>(t) * heads + kvh * G + warp) * splits * stride;
        float m = -1e9f;
        for (int s2 = lane; s2 < active; s2 += 32) m = fmaxf(m, __ldcg(hb + s2 * stride));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int s2 = lane; s2 < active; s2 += 32) {
            const float e = expf(__ldcg(hb + s2 * stride) - m);
            coef[warp * kMaxFusedSplits + s2] = e;
            l = fmaf(__ldcg(hb + s2 * stride + 1), e, l);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) inv_l[warp] = 1.0f / l;
    }
    __syncthreads();
    constexpr int kOuts = (G * HD + kThreads - 1) / kThreads;  // outputs per thread
    float vsum[kOuts];
#pragma unroll
    for (int o2 = 0; o2 < kOuts; ++o2) vsum[o2] = 0.0f;
    for (int s0 = 0; s0 < active; s0 += 8) {
        float u[kOuts][8];
#pragma unroll
        for (int o2 = 0; o2 < kOuts; ++o2) {
            const int idx = threadIdx.x + kThreads * o2;
            const int g = idx / HD, d = idx - g * HD;
            const float* hv = scratch + (static_cast<int64_t>(t) * heads + kvh * G + g) * splits * stride + 2 + d;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                u[o2][j] = idx < G * HD && s0 + j < active ? __ldcg(hv + (s0 + j) * stride) : 0.0f;
        }
#pragma unroll
        for (int o2 = 0; o2 < kOuts; ++o2) {
            const int g = min((threadIdx.x + kThreads * o2) / HD, G - 1);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (s0 + j < active) vsum[o2] = fmaf(u[o2][j], coef[g * kMaxFusedSplits + s0 + j], vsum[o2]);
        }
    }
#pragma unroll
    for (int o2 = 0; o2 < kOuts; ++o2) {
        const int idx = threadIdx.x + kThreads * o2;
        if (idx < G * HD) {
            const int g = idx / HD, d = idx - g * HD;
            ctx[(static_cast<int64_t>(t) * heads + kvh * G + g) * HD + d] = vsum[o2] * inv_l[g];
        }
    }
}

// Causal attention for a prompt (rows_per_seq > 1), the partials of
// attention_partial_kernel for a tile of query rows at once: one block per (kv
// head, split of 64 positions, tile of 64 / G rows of one sequence), so the
// split's key and value rows -- staged in shared memory by bulk copies with the
// tile's query rows -- are read once per tile instead of once per row.  Scores:
// thread (tq, tj) forms the 4 x 4 products of query vectors tq + 16a (vector
// r G + g: row r, head g of the group) and positions tj + 16b, one fp32 chain
// over the head dims; a position past a row's own (causal) is masked out.  Warp
// w takes the softmax statistics of query vectors 8w .. 8w + 7; then thread
// (tq, td) sums the weighted value rows for its four query vectors and HD / 16
// dims.  A row with no position in this split writes nothing (the merge reads
// only the splits up to each row's position).  Waits on the copies are bounded.
template <int G, int HD>
struct PrefillAttention {
    static constexpr int QT = 64 / G;     // query rows per block
    static constexpr int QV = QT * G;     // query vectors per block (<= 64)
    static constexpr int kPad = HD + 4;   // floats between staged key rows
    static constexpr int kPp = kSpan + 4; // floats between rows of exp(score - max)
    static constexpr int kQArea = 64 * HD > 64 * kPp ? 64 * HD : 64 * kPp;
    __host__ __device__ static constexpr size_t smem_bytes() {
        return sizeof(float) * (static_cast<size_t>(kSpan) * kPad + kSpan * HD + kQArea);
    }
};

template <int G, int HD>
__global__ void __launch_bounds__(kThreads) attention_prefill_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
    float* __restrict__ scratch, int heads, int kv_heads, int max_seq, int layer, float scale, int q_stride,
    const int32_t* __restrict__ pos, int rows_per_seq, int64_t cache_stride, int32_t* __restrict__ err) {
    using S = PrefillAttention<G, HD>;
    constexpr int QT = S::QT, QV = S::QV;
    static_assert(kThreads == 256 && QV <= 64, "16 x 16 threads over 64 query vectors x 64 positions");
    extern __shared__ __align__(16) float sm[];
    float* ks = sm;                         // [kSpan][kPad]
    float* vs = ks + kSpan * S::kPad;       // [kSpan][HD]
    float* qs = vs + kSpan * HD;            // [QV][HD], then ps [64][kPp]
    float* ps = qs;
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ float stat[64][2];
    dev::pdl_wait();  // q and the cache rows come from the previous kernels
    dev::pdl_launch_dependents();
    const int kvh = blockIdx.x, split = blockIdx.y, tile = blockIdx.z;
    const int tiles_per_seq = (rows_per_seq + QT - 1) / QT;
    const int seq = tile / tiles_per_seq;
    const int r0 = (tile - seq * tiles_per_seq) * QT;  // first row of the tile inside its sequence
    const int nr = min(QT, rows_per_seq - r0);
    const int p0 = *pos;
    const int j0 = split * kSpan;
    const int last = p0 + r0 + nr - 1;  // the position of the tile's last row
    if (j0 > last) return;              // no row of the tile sees this split
    const int n = min(kSpan, last + 1 - j0);
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int64_t base = seq * cache_stride + ((static_cast<int64_t>(layer) * kv_heads + kvh) * max_seq + j0) * HD;
    const int64_t row0 = static_cast<int64_t>(seq) * rows_per_seq + r0;  // global row of the tile's first row
    const uint32_t bar_kq = dev::smem_u32(&bars[0]), bar_v = dev::smem_u32(&bars[1]);
    if (tid == 0) {
        dev::mbar_init(bar_kq, 1);
        dev::mbar_init(bar_v, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (warp == 0) {
        const uint32_t kv_bytes = static_cast<uint32_t>(n * HD * sizeof(float));
        constexpr uint32_t q_row_bytes = G * HD * sizeof(float);
        if (lane == 0) {
            dev::mbar_expect_tx(bar_kq, kv_bytes + nr * q_row_bytes);
            dev::mbar_expect_tx(bar_v, kv_bytes);
            dev::bulk_load(dev::smem_u32(vs), vc + base, kv_bytes, bar_v);
        }
        __syncwarp();
        for (int j = lane; j < n; j += 32)
            dev::bulk_load(dev::smem_u32(ks + j * S::kPad), kc + base + static_cast<int64_t>(j) * HD,
                           HD * sizeof(float), bar_kq);
        for (int r = lane; r < nr; r += 32)
            dev::bulk_load(dev::smem_u32(qs + r * G * HD),
                           q + (row0 + r) * q_stride + static_cast<int64_t>(kvh) * G * HD, q_row_bytes, bar_kq);
    }
    bool ok = dev::mbar_wait_bounded(bar_kq, 0);
    if (__syncthreads_or(!ok)) {
        if (tid == 0) {
            atomicOr(err, 1);
            dev::mbar_wait_bounded(bar_kq, 0);
            dev::mbar_wait_bounded(bar_v, 0);
        }
        return;
    }
    const int tq = tid >> 4, tj = tid & 15;
    float sc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) sc[a][b] = 0.0f;
#pragma unroll 4
    for (int d = 0; d < HD; d += 4) {
        float4 qv[4], kv[4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
            qv[a] = tq + 16 * a < QV ? *reinterpret_cast<const float4*>(qs + (tq + 16 * a) * HD + d)
                                     : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int b = 0; b < 4; ++b) kv[b] = *reinterpret_cast<const float4*>(ks + (tj + 16 * b) * S::kPad + d);
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                sc[a][b] = fmaf(qv[a].x, kv[b].x, sc[a][b]);
                sc[a][b] = fmaf(qv[a].y, kv[b].y, sc[a][b]);
                sc[a][b] = fmaf(qv[a].z, kv[b].z, sc[a][b]);
                sc[a][b] = fmaf(qv[a].w, kv[b].w, sc[a][b]);
            }
    }
    __syncthreads();  // every thread is done with qs: its area becomes ps
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int qi = tq + 16 * a;
        const int r = qi / G;
        const int lim = p0 + r0 + r - j0;  // the row sees positions j0 .. j0 + lim
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int jj = tj + 16 * b;
            ps[qi * S::kPp + jj] = qi < QV && r < nr && jj < n && jj <= lim ? sc[a][b] * scale : -FLT_MAX;
        }
    }
    __syncthreads();
    // softmax statistics: warp w, query vectors 8w .. 8w + 7, lane -> positions lane, lane + 32
    for (int i = 0; i < 8; ++i) {
        const int qi = 8 * warp + i;
        const float s0 = ps[qi * S::kPp + lane], s1 = ps[qi * S::kPp + lane + 32];
        float mx = fmaxf(s0, s1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const bool any = mx > -FLT_MAX;
        const float e0 = any && s0 > -FLT_MAX ? expf(s0 - mx) : 0.0f;
        const float e1 = any && s1 > -FLT_MAX ? expf(s1 - mx) : 0.0f;
        ps[qi * S::kPp + lane] = e0;
        ps[qi * S::kPp + lane + 32] = e1;
        float sum = e0 + e1;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        if (lane == 0) {
            stat[qi][0] = mx;
            stat[qi][1] = sum;
        }
    }
    ok = dev::mbar_wait_bounded(bar_v, 0);
    if (__syncthreads_or(!ok)) {  // also publishes ps and stat
        if (tid == 0) {
            atomicOr(err, 1);
            dev::mbar_wait_bounded(bar_v, 0);
        }
        return;
    }
    // weighted values: thread (tq, td), query vectors tq + 16a, dims 4 td + 64 c
    constexpr int kC = HD / 64;  // float4 columns per thread: 1 (HD 64) or 2 (HD 128)
    const int td = tj;
    float4 o[4][kC];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int c = 0; c < kC; ++c) o[a][c] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int jj = 0; jj < n; ++jj) {
        float pv[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) pv[a] = ps[(tq + 16 * a) * S::kPp + jj];
#pragma unroll
        for (int c = 0; c < kC; ++c) {
            const float4 v4 = *reinterpret_cast<const float4*>(vs + jj * HD + 64 * c + 4 * td);
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                o[a][c].x = fmaf(pv[a], v4.x, o[a][c].x);
                o[a][c].y = fmaf(pv[a], v4.y, o[a][c].y);
                o[a][c].z = fmaf(pv[a], v4.z, o[a][c].z);
                o[a][c].w = fmaf(pv[a], v4.w, o[a][c].w);
            }
        }
    }
    const int64_t splits = (max_seq + kSpan - 1) / kSpan;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int qi = tq + 16 * a;
        const int r = qi / G, g = qi - r * G;
        if (qi >= QV || r >= nr || j0 > p0 + r0 + r) continue;  // no position of this split for the row
        float* out = scratch + (((row0 + r) * heads + kvh * G + g) * splits + split) * (HD + 2);
#pragma unroll
        for (int c = 0; c < kC; ++c) {  // rows of HD + 2 floats: 8-byte aligned only
            float* dst = out + 2 + 64 * c + 4 * td;
            dst[0] = o[a][c].x;
            dst[1] = o[a][c].y;
            dst[2] = o[a][c].z;
            dst[3] = o[a][c].w;
        }
        if (td == 0) {
            out[0] = stat[qi][0];
            out[1] = stat[qi][1];
        }
    }
}

__global__ void attention_merge_kernel(const float* __restrict__ scratch, float* __restrict__ ctx, int heads,
                                       int head_dim, int max_seq, const int32_t* __restrict__ pos, int rows_per_seq) {
    dev::pdl_wait();  // inputs may come from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
    const int h = blockIdx.x, t = blockIdx.y;
    const int splits = (*pos + t % rows_per_seq) / kSpan + 1;
    const int stride = head_dim + 2;
    const float* base =
        scratch + (static_cast<int64_t>(t) * heads + h) * ((max_seq + kSpan - 1) / kSpan) * stride;
    float m = -1e9f;
    for (int s = 0; s < splits; ++s) m = fmaxf(m, base[s * stride]);
    float l = 0.0f;
    for (int s = 0; s < splits; ++s) l += base[s * stride + 1] * expf(base[s * stride] - m);
    const float inv = 1.0f / l;
    for (int d = threadIdx.x; d < head_dim; d += blockDim.x) {
        float v = 0.0f;
        for (int s = 0; s < splits; ++s) v += base[s * stride + 2 + d] * expf(base[s * stride] - m);
        ctx[(static_cast<int64_t>(t) * heads + h) * head_dim + d] = v * inv;
    }
}

// gate = silu(gate) * up (Tensor.siluInPlace then mulInPlace)
__global__ void silu_mul_kernel(float* __restrict__ gate, const float* __restrict__ up, int64_t n) {
    dev::pdl_wait();  // inputs may come from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float x = gate[i];
        gate[i] = x / (1.0f + expf(-x)) * up[i];
    }
}

// out[t][j] = silu(gu[t][j]) * gu[t][hidden + j] for fused gate|up rows.
__global__ void silu_mul_rows_kernel(const float* __restrict__ gu, float* __restrict__ out, int rows, int hidden) {
    dev::pdl_wait();  // inputs may come from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
    const int64_t n = static_cast<int64_t>(rows) * hidden;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / hidden, j = i - t * hidden;
        const float x = gu[t * 2 * hidden + j];
        out[i] = x / (1.0f + expf(-x)) * gu[t * 2 * hidden + hidden + j];
    }
}

__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ y, int64_t n) {
    dev::pdl_wait();  // inputs may come from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        x[i] += y[i];
}

// Greedy pick of one row (argmaxOfLastToken, Transformer.kt:255-266): the
// largest logit above -1e9, the lowest index among equal ones, 0 if none.
// Stage 1: block (c, row) scans chunk c; stage 2: one block per row merges the
// chunks in order.
__device__ __forceinline__ void better(float& bv, int& bi, float ov, int oi) {
    if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
    }
}

__global__ void __launch_bounds__(kThreads) argmax_partial_kernel(const float* __restrict__ logits, int n, int chunk,
                                                                  float* __restrict__ pv, int* __restrict__ pi) {
    dev::pdl_wait();  // inputs may come from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
    __shared__ float bv[kThreads];
    __shared__ int bi[kThreads];
    const int row = blockIdx.y, c = blockIdx.x;
    const int v0 = c * chunk, v1 = min(v0 + chunk, n);
    float best = -1e9f;
    int idx = 0x7fffffff;
    for (int v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
        const float x = logits[static_cast<int64_t>(row) * n + v];
        if (x > best) {  // strictly greater: the first (lowest) index of a tie stays
            best = x;
            idx = v;
        }
    }
    bv[threadIdx.x] = best;
    bi[threadIdx.x] = idx;
    __syncthreads();
    for (int st = blockDim.x / 2; st > 0; st >>= 1) {
        if (threadIdx.x < st) better(bv[threadIdx.x], bi[threadIdx.x], bv[threadIdx.x + st], bi[threadIdx.x + st]);
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        pv[row * gridDim.x + c] = bv[0];
        pi[row * gridDim.x + c] = bi[0];
    }
}

__global__ void argmax_merge_kernel(const float* __restrict__ pv, const int* __restrict__ pi, int chunks,
                                    int32_t* __restrict__ out) {
    dev::pdl_wait();  // inputs may come from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
    if (threadIdx.x != 0) return;
    const int row = blockIdx.x;
    float best = -1e9f;
    int idx = 0x7fffffff;
    for (int c = 0; c < chunks; ++c) better(best, idx, pv[row * chunks + c], pi[row * chunks + c]);
    out[row] = idx == 0x7fffffff ? 0 : idx;
}

// dequantizeColumn(token) of a weight [K x N] (the tied embedding lookup):
// out[k] = value(k, *col) for k < K.
__global__ void dequantize_column_kernel(QView w, const int32_t* __restrict__ cols, float* __restrict__ outs,
                                         int32_t* __restrict__ status) {
    dev::pdl_wait();  // inputs may come from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents();
    const int c = cols[blockIdx.y];
    float* out = outs + static_cast<int64_t>(blockIdx.y) * w.rows;
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

__global__ void increment_kernel(int32_t* p, int32_t delta) {
    dev::pdl_wait();  // inputs may come from the previous kernel (programmatic dependent launch)
    dev::pdl_launch_dependents(); *p += delta; }

int grid_for(int64_t n) { return static_cast<int>(std::min<int64_t>((n + kThreads - 1) / kThreads, 148 * 8)); }

}  // namespace


// Launches with programmatic stream serialization: the kernel may start while
// the previous kernel on the stream finishes; every kernel here waits
// (griddepcontrol.wait) before touching memory the previous one wrote.
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = grid;
    lc.blockDim = block;
    lc.dynamicSmemBytes = smem;
    lc.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    return cudaLaunchKernelEx(&lc, kernel, static_cast<Params>(args)...);
}

cudaError_t launch_rmsnorm(const float* x, const float* w, float* out, int rows, int dim, float eps, cudaStream_t s) {
    launch_pdl(rmsnorm_kernel, dim3(rows), dim3(kThreads), 0, s, x, w, out, dim, eps);
    return cudaGetLastError();
}
cudaError_t launch_add_rmsnorm(float* x, const float* y, const float* w, float* out, int rows, int dim, float eps,
                               cudaStream_t s) {
    launch_pdl(add_rmsnorm_kernel, dim3(rows), dim3(kThreads), 0, s, x, y, w, out, dim, eps);
    return cudaGetLastError();
}
cudaError_t launch_rope_kv(float* qkv, int rows, int q_width, int kv_heads, int head_dim, const float* inv_freq,
                           float* kc, float* vc, int max_seq, int layer, const int32_t* pos, int rows_per_seq,
                           int64_t cache_stride, cudaStream_t s) {
    const int total = (q_width + kv_heads * head_dim) / 2 + kv_heads * head_dim;
    launch_pdl(rope_kv_kernel, dim3(dim3((total + kThreads - 1) / kThreads, rows)), dim3(kThreads), 0, s, 
        qkv, q_width, kv_heads, head_dim, inv_freq, kc, vc, max_seq, layer, pos, rows_per_seq, cache_stride);
    return cudaGetLastError();
}
// Split partials [rows][heads][splits][head_dim + 2], then one merge ticket
// (int32) per (row, head) for the fused decode kernel.
size_t attention_scratch_floats(int rows, int heads, int head_dim, int max_seq) {
    return static_cast<size_t>(rows) * heads * ((max_seq + kSpan - 1) / kSpan) * (head_dim + 2) +
           static_cast<size_t>(rows) * heads;
}

bool attention_fused_supported(int heads, int kv_heads, int head_dim, int max_seq) {
    return kv_heads > 0 && heads % kv_heads == 0 && heads / kv_heads <= 8 && (head_dim == 64 || head_dim == 128) &&
           (max_seq + kSpan - 1) / kSpan <= kMaxFusedSplits;
}

bool staged_attention_enabled();

// Dynamic shared memory of every staged fused-decode instantiation (once per device).
template <int HD>
cudaError_t prepare_staged_decode() {
    constexpr int kMaxDevices = 64;
    static std::atomic<bool> done[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < kMaxDevices && done[dev].load(std::memory_order_acquire)) return cudaSuccess;
#define KT_STAGED_ATTR(G_)                                                                                     \
    if (e == cudaSuccess)                                                                                      \
        e = cudaFuncSetAttribute(attention_decode_staged_kernel<G_, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 static_cast<int>(StagedAttention<HD>::template smem_bytes<G_>()));
    KT_STAGED_ATTR(1) KT_STAGED_ATTR(2) KT_STAGED_ATTR(3) KT_STAGED_ATTR(4)
    KT_STAGED_ATTR(5) KT_STAGED_ATTR(6) KT_STAGED_ATTR(7) KT_STAGED_ATTR(8)
#undef KT_STAGED_ATTR
    if (e == cudaSuccess && dev >= 0 && dev < kMaxDevices) done[dev].store(true, std::memory_order_release);
    return e;
}

cudaError_t launch_attention_decode_fused(const float* qkv, int rows, int q_width, int heads, int kv_heads,
                                          int head_dim, const float* inv_freq, float* kc, float* vc, float* ctx,
                                          float* scratch, int max_seq, int layer, float scale, const int32_t* pos,
                                          int64_t cache_stride, int32_t* err, cudaStream_t s) {
    if (!attention_fused_supported(heads, kv_heads, head_dim, max_seq)) return cudaErrorInvalidValue;
    const int splits = (max_seq + kSpan - 1) / kSpan;
    int32_t* tickets = reinterpret_cast<int32_t*>(
        scratch + static_cast<size_t>(rows) * heads * splits * (head_dim + 2));
    const dim3 grid(kv_heads, splits, rows);
    const int group = heads / kv_heads;
    // staged: the cache rows on 16-byte boundaries (bulk copies); measured faster
    // than the register-loading kernels at head_dim 128 and with several rows, and
    // a little slower at head_dim 64 on one row (where a step's tiles are small)
    const bool aligned = (reinterpret_cast<uintptr_t>(kc) & 15) == 0 && (reinterpret_cast<uintptr_t>(vc) & 15) == 0 &&
                         cache_stride % 4 == 0;
    if (staged_attention_enabled() && aligned && (head_dim == 128 || rows > 1)) {
#define KT_SFUSED_CASE(G_, HD_)                                                                                  \
    e = launch_pdl(attention_decode_staged_kernel<G_, HD_>, grid, dim3(kThreads),                               \
                   StagedAttention<HD_>::template smem_bytes<G_>(), s, qkv, q_width, inv_freq, kc, vc, scratch, \
                   tickets, ctx, heads, kv_heads, max_seq, layer, scale, pos, cache_stride, err)
#define KT_SFUSED_GROUPS(HD_)                    \
    switch (group) {                             \
        case 1: KT_SFUSED_CASE(1, HD_); break;   \
        case 2: KT_SFUSED_CASE(2, HD_); break;   \
        case 3: KT_SFUSED_CASE(3, HD_); break;   \
        case 4: KT_SFUSED_CASE(4, HD_); break;   \
        case 5: KT_SFUSED_CASE(5, HD_); break;   \
        case 6: KT_SFUSED_CASE(6, HD_); break;   \
        case 7: KT_SFUSED_CASE(7, HD_); break;   \
        default: KT_SFUSED_CASE(8, HD_); break;  \
    }
        cudaError_t e = head_dim == 64 ? prepare_staged_decode<64>() : prepare_staged_decode<128>();
        if (e != cudaSuccess) return e;
        if (head_dim == 64) {
            KT_SFUSED_GROUPS(64)
        } else {
            KT_SFUSED_GROUPS(128)
        }
#undef KT_SFUSED_GROUPS
#undef KT_SFUSED_CASE
        return e;
    }
#define KT_FUSED_CASE(G_, KP_)                                                                                  \
    launch_pdl(attention_decode_fused_kernel<G_, KP_>, grid, dim3(kThreads), 0, s, qkv, q_width, inv_freq, kc, vc, \
               scratch, tickets, ctx, heads, kv_heads, head_dim, max_seq, layer, scale, pos, cache_stride)
#define KT_FUSED_GROUPS(KP_)              \
    switch (group) {                      \
        case 1: KT_FUSED_CASE(1, KP_); break; \
        case 2: KT_FUSED_CASE(2, KP_); break; \
        case 3: KT_FUSED_CASE(3, KP_); break; \
        case 4: KT_FUSED_CASE(4, KP_); break; \
        case 5: KT_FUSED_CASE(5, KP_); break; \
        case 6: KT_FUSED_CASE(6, KP_); break; \
        case 7: KT_FUSED_CASE(7, KP_); break; \
        default: KT_FUSED_CASE(8, KP_); break; \
    }
    if (head_dim == 64) {
        KT_FUSED_GROUPS(64)
    } else {
#undef KT_FUSED_CASE
#define KT_FUSED_CASE(G_, KP_)                                                                                  \
    launch_pdl(attention_decode_fused_wide_kernel<G_, KP_>, grid, dim3(kThreads), 0, s, qkv, q_width, inv_freq, kc, \
               vc, scratch, tickets, ctx, heads, kv_heads, head_dim, max_seq, layer, scale, pos, cache_stride)
        KT_FUSED_GROUPS(4)
    }
#undef KT_FUSED_GROUPS
#undef KT_FUSED_CASE
    return cudaGetLastError();
}
cudaError_t launch_rope(float* v, int rows, int width, int head_dim, const float* inv_freq, const int32_t* pos,
                        cudaStream_t s) {
    launch_pdl(rope_kernel, dim3(grid_for(static_cast<int64_t>(rows) * width / 2)), dim3(kThreads), 0, s, v, rows, width, head_dim,
                                                                                       inv_freq, pos);
    return cudaGetLastError();
}
cudaError_t launch_kv_store(const float* k, const float* v, float* kc, float* vc, int rows, int kv_heads, int head_dim,
                            int max_seq, int layer, const int32_t* pos, cudaStream_t s) {
    launch_pdl(kv_store_kernel, dim3(grid_for(static_cast<int64_t>(rows) * kv_heads * head_dim)), dim3(kThreads), 0, s, 
        k, v, kc, vc, rows, kv_heads, head_dim, max_seq, layer, pos);
    return cudaGetLastError();
}
// Dynamic shared memory of every staged-attention instantiation (once per device).
template <int HD>
cudaError_t prepare_staged_attention() {
    constexpr int kMaxDevices = 64;
    static std::atomic<bool> done[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < kMaxDevices && done[dev].load(std::memory_order_acquire)) return cudaSuccess;
#define KT_STAGED_ATTR(G_)                                                                                    \
    if (e == cudaSuccess)                                                                                     \
        e = cudaFuncSetAttribute(attention_group_staged_kernel<G_, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                 static_cast<int>(StagedAttention<HD>::template smem_bytes<G_>()));
    KT_STAGED_ATTR(1) KT_STAGED_ATTR(2) KT_STAGED_ATTR(3) KT_STAGED_ATTR(4)
    KT_STAGED_ATTR(5) KT_STAGED_ATTR(6) KT_STAGED_ATTR(7) KT_STAGED_ATTR(8)
#undef KT_STAGED_ATTR
    if (e == cudaSuccess && dev >= 0 && dev < kMaxDevices) done[dev].store(true, std::memory_order_release);
    return e;
}

bool staged_attention_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("KT_ATTN_STAGED");
        return !(v && v[0] == '0');
    }();
    return on;
}

template <int HD>
cudaError_t launch_staged_attention(dim3 grid, int group, cudaStream_t s, const float* q, const float* kc,
                                    const float* vc, float* scores, int heads, int kv_heads, int max_seq, int layer,
                                    float scale, int q_stride, const int32_t* pos, int rows_per_seq,
                                    int64_t cache_stride, int32_t* err) {
    const cudaError_t e = prepare_staged_attention<HD>();
    if (e != cudaSuccess) return e;
#define KT_STAGED_CASE(G_)                                                                                        \
    return launch_pdl(attention_group_staged_kernel<G_, HD>, grid, dim3(kThreads),                                 \
                      StagedAttention<HD>::template smem_bytes<G_>(), s, q, kc, vc, scores, heads, kv_heads, max_seq, \
                      layer, scale, q_stride, pos, rows_per_seq, cache_stride, err)
    switch (group) {
        case 1: KT_STAGED_CASE(1);
        case 2: KT_STAGED_CASE(2);
        case 3: KT_STAGED_CASE(3);
        case 4: KT_STAGED_CASE(4);
        case 5: KT_STAGED_CASE(5);
        case 6: KT_STAGED_CASE(6);
        case 7: KT_STAGED_CASE(7);
        default: KT_STAGED_CASE(8);
    }
#undef KT_STAGED_CASE
}

// Causal attention for a prompt on tensor cores, flash style: one block per (kv
// head, tile of 64 / G query rows of one sequence) walks the 64-position spans
// up to the tile's last row with a running maximum and sum per query vector
// (online softmax), so no partials are written and no merge runs.  Both
// products run on mma.sync.m16n8k8 TF32 with fp32 accumulation: queries and
// probabilities rounded to 10-bit mantissas with cvt.rna, keys and values
// read as their fp32 bits (the tensor core ignores the low 13 mantissa bits:
// TF32 rounded toward zero, no conversion pass per tile); used where the prompt's matmuls already
// run on the bf16 tensor-core GEMM (9 or more rows), whose tolerance covers the
// rounding.  Warp w: query vectors 16 (w % 4) .. + 15 (vector r G + g: row r,
// head g of the group), their fragments held in registers for the whole block;
// for the scores positions 32 (w / 4) .. + 31 of the span, for the weighted
// values dims (w / 4) HD / 2 .. + HD / 2.  The two warps of a row block
// exchange their row maxima through shared memory each span and their sums at
// the end.  Key and value tiles come in by 2-D TMA copies (boxes of 32 floats x
// 64 positions, 128-byte swizzle: fragment reads hit distinct banks), double-
// buffered (span s + 2 is copied while s + 1 is used); value rows past the last
// position of the tile are zeroed (their probabilities are 0, but 0 * stale
// data could be NaN).  Heavy tiles (late rows, many spans) are scheduled first.
// Waits on the copies are bounded.
template <int G, int HD>
struct PrefillFlash {
    static constexpr int QT = 64 / G;       // query rows per block
    static constexpr int QV = QT * G;       // query vectors per block (<= 64)
    static constexpr int kBoxes = HD / 32;  // TMA boxes per tile (32 floats = 128 bytes wide)
    static constexpr int kStage = kSpan * HD;  // floats of one key or value tile
    static constexpr int kPp = kSpan + 4;   // floats between rows of probabilities
    static constexpr int kQPad = HD + 4;    // floats between staged query vectors (fragment loads: bank 4g + t)
    static constexpr int kQP = 64 * kQPad > 64 * kPp ? 64 * kQPad : 64 * kPp;  // staged queries, then probabilities
    __host__ __device__ static constexpr size_t smem_bytes() {
        return 1024 + sizeof(float) * (4 * static_cast<size_t>(kStage) + kQP + 2 * 2 * 64);
    }
};

// A key or value tile in shared memory: kBoxes TMA boxes of 64 rows x 32 floats
// with the 128-byte swizzle, so element (row, col) sits at float
//   (col / 32) * 64 * 32 + row * 32 + (((col % 32) / 4) ^ (row % 8)) * 4 + col % 4
// (16-byte chunk c of row r at chunk c ^ (r & 7)); the fragment loads below
// hoist the lane's part of that offset.

__device__ __forceinline__ uint32_t to_tf32(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ void mma_tf32(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int G, int HD>
__global__ void __launch_bounds__(kThreads) attention_prefill_flash_kernel(
    const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v, const float* __restrict__ q,
    float* __restrict__ ctx, int heads, int kv_heads, int max_seq, int layer, float scale, int q_stride,
    const int32_t* __restrict__ pos, int rows_per_seq, int64_t cache_rows_per_seq, int32_t* __restrict__ err) {
    using S = PrefillFlash<G, HD>;
    constexpr int QT = S::QT, QV = S::QV;
    static_assert(kThreads == 256 && QV <= 64 && kSpan == 64, "8 warps over 64 query vectors x 64 positions");
    extern __shared__ unsigned char smem_raw[];
    float* base = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    float* ks = base;                        // [2][kBoxes][64][32] swizzled
    float* vs = ks + 2 * S::kStage;          // [2][kBoxes][64][32] swizzled
    float* qs = vs + 2 * S::kStage;          // [64][kQPad] staged query vectors, then ps [64][kPp]
    float* ps = qs;
    float* red = qs + S::kQP;                // [2][2][64]: row maxima, then row sums, per half
    __shared__ __align__(8) uint64_t bars[3];  // query, span stage 0, span stage 1
    dev::pdl_wait();  // q and the cache rows come from the previous kernels
    dev::pdl_launch_dependents();
    const int kvh = blockIdx.x;
    const int tile = gridDim.y - 1 - blockIdx.y;  // heavy tiles first
    const int tiles_per_seq = (rows_per_seq + QT - 1) / QT;
    const int seq = tile / tiles_per_seq;
    const int r0 = (tile - seq * tiles_per_seq) * QT;  // first row of the tile inside its sequence
    const int nr = min(QT, rows_per_seq - r0);
    const int p0 = *pos;
    const int last = p0 + r0 + nr - 1;  // the position of the tile's last row
    const int n_spans = last / kSpan + 1;
    const int tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, t = lane & 3;
    // first cache row (of the 2-D [rows][HD] view) of this sequence, layer and kv head
    const int cache_row0 = static_cast<int>(seq * cache_rows_per_seq + (static_cast<int64_t>(layer) * kv_heads + kvh) * max_seq);
    const int64_t row0 = static_cast<int64_t>(seq) * rows_per_seq + r0;  // global row of the tile's first row
    const uint32_t bar_q = dev::smem_u32(&bars[0]);
    if (tid == 0) {
        for (int i = 0; i < 3; ++i) dev::mbar_init(dev::smem_u32(&bars[i]), 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // span sp's key and value tiles into stage sp & 1 (one thread)
    auto issue_span = [&](int sp) {
        const int st = sp & 1;
        const uint32_t bar = dev::smem_u32(&bars[1 + st]);
        dev::mbar_expect_tx(bar, 2u * S::kStage * sizeof(float));
#pragma unroll
        for (int b = 0; b < S::kBoxes; ++b) {
            dev::tma_load_2d(dev::smem_u32(ks + st * S::kStage + b * kSpan * 32), &tmap_k, 32 * b,
                             cache_row0 + sp * kSpan, bar);
            dev::tma_load_2d(dev::smem_u32(vs + st * S::kStage + b * kSpan * 32), &tmap_v, 32 * b,
                             cache_row0 + sp * kSpan, bar);
        }
    };
    constexpr uint32_t q_vec_bytes = HD * sizeof(float);
    if (warp == 0) {
        if (lane == 0) {
            dev::mbar_expect_tx(bar_q, nr * G * q_vec_bytes);
            issue_span(0);
            if (n_spans > 1) issue_span(1);
        }
        __syncwarp();
        for (int i = lane; i < nr * G; i += 32) {  // query vector i = row i / G, head i % G of the group
            const int r = i / G, gh = i - r * G;
            dev::bulk_load(dev::smem_u32(qs + i * S::kQPad),
                           q + (row0 + r) * q_stride + static_cast<int64_t>(kvh * G + gh) * HD, q_vec_bytes, bar_q);
        }
    }
    int issued = n_spans > 1 ? 2 : 1;  // spans whose copies were issued (thread 0's count)
    bool ok = dev::mbar_wait_bounded(bar_q, 0);
    if (__syncthreads_or(!ok)) {
        if (tid == 0) {
            atomicOr(err, 1);
            dev::mbar_wait_bounded(bar_q, 0);
            for (int sp = 0; sp < issued; ++sp) dev::mbar_wait_bounded(dev::smem_u32(&bars[1 + (sp & 1)]), 0);
        }
        return;
    }
    const int mt = warp & 3, half = warp >> 2;
    const int qa = 16 * mt + g;  // this lane's query vectors qa and qa + 8
    // this warp's query fragments for every k-step, tf32 (vectors past the tile's rows: zeros)
    uint32_t qf[HD / 8][4];
    {
        const bool v0 = qa < nr * G, v8 = qa + 8 < nr * G;
#pragma unroll
        for (int ks8 = 0; ks8 < HD / 8; ++ks8) {
            const int d = 8 * ks8 + t;
            qf[ks8][0] = v0 ? to_tf32(qs[qa * S::kQPad + d]) : 0u;
            qf[ks8][1] = v8 ? to_tf32(qs[(qa + 8) * S::kQPad + d]) : 0u;
            qf[ks8][2] = v0 ? to_tf32(qs[qa * S::kQPad + d + 4]) : 0u;
            qf[ks8][3] = v8 ? to_tf32(qs[(qa + 8) * S::kQPad + d + 4]) : 0u;
        }
    }
    constexpr int kNt = HD / 16;  // n-tiles of 8 dims per warp for the weighted values
    float o[kNt][4];
#pragma unroll
    for (int nt = 0; nt < kNt; ++nt) o[nt][0] = o[nt][1] = o[nt][2] = o[nt][3] = 0.0f;
    float m_run[2] = {-FLT_MAX, -FLT_MAX}, l_run[2] = {0.0f, 0.0f};
    int lim[2];  // the last position row qa + 8 h sees (-1: no such row)
    bool row_ok[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int qi = qa + 8 * h, r = qi / G;
        row_ok[h] = qi < QV && r < nr;
        lim[h] = row_ok[h] ? p0 + r0 + r : -1;
    }
    const uint32_t pair_bar = 1 + mt;  // named barrier of warps mt and mt + 4
    for (int sp = 0; sp < n_spans; ++sp) {
        const int st = sp & 1;
        const int j0 = sp * kSpan;
        const int n = min(kSpan, last + 1 - j0);
        ok = dev::mbar_wait_bounded(dev::smem_u32(&bars[1 + st]), (sp >> 1) & 1);
        if (__syncthreads_or(!ok)) {  // (the first one also ends every warp's reads of qs)
            if (tid == 0) {
                atomicOr(err, 1);
                for (int s2 = sp; s2 < issued; ++s2)
                    dev::mbar_wait_bounded(dev::smem_u32(&bars[1 + (s2 & 1)]), (s2 >> 1) & 1);
            }
            return;
        }
        float* kst = ks + st * S::kStage;
        float* vst = vs + st * S::kStage;
        if (n < kSpan) {  // value rows past n: zeros (the swizzle keeps rows whole: a box row is 32 floats of one row)
            for (int i = tid; i < S::kStage / 4; i += kThreads)
                if (((i >> 3) & (kSpan - 1)) >= n) reinterpret_cast<float4*>(vst)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
            __syncthreads();
        }
        // scores S = Q K^T: query vectors 16 mt .. + 15, positions 32 half .. + 31 of the span
        float acc[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.0f;
        {
            // key row 32 half + 8 nt + g (row & 7 = g), dims 8 ks8 + t and + 4: box ks8 / 4,
            // chunks 2 (ks8 % 4) and + 1, each XOR g
            const uint32_t* krow = reinterpret_cast<const uint32_t*>(kst) + (32 * half + g) * 32 + t;
#pragma unroll
            for (int ks8 = 0; ks8 < HD / 8; ++ks8) {
                const uint32_t* k0p = krow + (ks8 >> 2) * (kSpan * 32) + (((2 * (ks8 & 3)) ^ g) << 2);
                const uint32_t* k4p = krow + (ks8 >> 2) * (kSpan * 32) + (((2 * (ks8 & 3) + 1) ^ g) << 2);
#pragma unroll
                for (int nt = 0; nt < 4; ++nt)
                    mma_tf32(acc[nt], qf[ks8][0], qf[ks8][1], qf[ks8][2], qf[ks8][3], k0p[nt * 8 * 32],
                             k4p[nt * 8 * 32]);
            }
        }
        // masked, scaled scores and this half's row maxima
        float mx[2] = {-FLT_MAX, -FLT_MAX};
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const int jj = 32 * half + 8 * nt + 2 * t + c;
                    const bool v = jj < n && j0 + jj <= lim[h];
                    const float sv = v ? acc[nt][2 * h + c] * scale : -FLT_MAX;
                    acc[nt][2 * h + c] = sv;
                    mx[h] = fmaxf(mx[h], sv);
                }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
            mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
            if (t == 0) red[half * 64 + qa + 8 * h] = mx[h];
        }
        asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory");
        float alpha[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float other = red[(1 - half) * 64 + qa + 8 * h];
            const float m_new = fmaxf(m_run[h], fmaxf(mx[h], other));
            // the running values are rescaled to the new maximum (nothing seen yet: nothing to rescale)
            alpha[h] = m_run[h] > -FLT_MAX ? expf(m_run[h] - m_new) : 1.0f;
            float sum = 0.0f;
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const float sv = acc[nt][2 * h + c];
                    const float e = sv > -FLT_MAX ? expf(sv - m_new) : 0.0f;
                    sum += e;
                    const int jj = 32 * half + 8 * nt + 2 * t + c;
                    *reinterpret_cast<uint32_t*>(ps + (qa + 8 * h) * S::kPp + jj) = to_tf32(e);
                }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            l_run[h] = l_run[h] * alpha[h] + sum;
            m_run[h] = m_new;
        }
#pragma unroll
        for (int nt = 0; nt < kNt; ++nt) {
            o[nt][0] *= alpha[0];
            o[nt][1] *= alpha[0];
            o[nt][2] *= alpha[1];
            o[nt][3] *= alpha[1];
        }
        asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory");  // both halves of P written
        // weighted values O += P V: query vectors 16 mt .. + 15, dims HD / 2 half .. + HD / 2
        {
            const uint32_t* pa0 = reinterpret_cast<const uint32_t*>(ps + qa * S::kPp + t);
            const uint32_t* pa8 = pa0 + 8 * S::kPp;
            // value rows k0 + t and k0 + t + 4 (row & 7 = t, t + 4); n-tile nt takes box
            // half HD / 64 + nt / 4 and, of it, chunks c = nt % 4 and c + 4: column g is
            // element g % 4 of chunk c + 4 (g / 4), XOR the row's low bits -- over the 32
            // lanes 8 distinct chunks x 4 elements, no bank conflict (adjacent chunks c, c + 1
            // would meet the same four chunks after the XOR with rows 0-3)
            const uint32_t* vrow =
                reinterpret_cast<const uint32_t*>(vst) + half * (HD / 64) * (kSpan * 32) + t * 32 + (g & 3);
            int vo0[4], vo1[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                vo0[c] = ((c + 4 * (g >> 2)) ^ t) << 2;
                vo1[c] = (((c + 4 * (g >> 2)) ^ (t + 4)) << 2) + 4 * 32;
            }
            const int kend = (n + 7) & ~7;  // positions past n carry probability 0
            for (int k0 = 0; k0 < kend; k0 += 8) {
                const uint32_t a0 = pa0[k0], a1 = pa8[k0], a2 = pa0[k0 + 4], a3 = pa8[k0 + 4];
                const uint32_t* vk = vrow + k0 * 32;
#pragma unroll
                for (int nt = 0; nt < kNt; ++nt)
                    mma_tf32(o[nt], a0, a1, a2, a3, vk[(nt >> 2) * (kSpan * 32) + vo0[nt & 3]],
                             vk[(nt >> 2) * (kSpan * 32) + vo1[nt & 3]]);
            }
        }
        __syncthreads();  // every warp is done with this stage, ps and red
        if (tid == 0 && sp + 2 < n_spans) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue_span(sp + 2);
            ++issued;
        }
    }
    // every row's sum over both halves, then O / l into the context rows
#pragma unroll
    for (int h = 0; h < 2; ++h)
        if (t == 0) red[128 + half * 64 + qa + 8 * h] = l_run[h];
    asm volatile("bar.sync %0, 64;" ::"r"(pair_bar) : "memory");
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        if (!row_ok[h]) continue;
        const int qi = qa + 8 * h;
        const int r = qi / G, gh = qi - r * G;
        const float inv = 1.0f / (red[128 + qi] + red[128 + 64 + qi]);
        float* out = ctx + ((row0 + r) * heads + kvh * G + gh) * HD + (HD / 2) * half;
        // C columns 2t, 2t + 1 of n-tile nt: elements 2 (t % 2), + 1 of chunk nt % 4 + 4 (t / 2)
        // of box nt / 4 (the column order of the weighted values above)
#pragma unroll
        for (int nt = 0; nt < kNt; ++nt)
            *reinterpret_cast<float2*>(out + 32 * (nt >> 2) + 4 * ((nt & 3) + 4 * (t >> 1)) + 2 * (t & 1)) =
                make_float2(o[nt][2 * h] * inv, o[nt][2 * h + 1] * inv);
    }
}

bool prefill_attention_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("KT_ATTN_PREFILL");
        return !(v && v[0] == '0');
    }();
    return on;
}

// The TF32 tensor-core (flash) prefill kernel for blocks of 9 rows or more
// (KT_ATTN_PREFILL_MMA=0: the fp32 kernel and merge everywhere, for comparison).
bool prefill_mma_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("KT_ATTN_PREFILL_MMA");
        return !(v && v[0] == '0');
    }();
    return on;
}

template <int G, int HD>
cudaError_t launch_prefill_attention_g(int rows, int rows_per_seq, int splits, cudaStream_t s, const float* q,
                                       const float* kc, const float* vc, float* scores, int heads, int kv_heads,
                                       int max_seq, int layer, float scale, int q_stride, const int32_t* pos,
                                       int64_t cache_stride, int32_t* err) {
    using P = PrefillAttention<G, HD>;
    constexpr int kMaxDevices = 64;
    static std::atomic<bool> done[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (!(dev >= 0 && dev < kMaxDevices && done[dev].load(std::memory_order_acquire))) {
        e = cudaFuncSetAttribute(attention_prefill_kernel<G, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(P::smem_bytes()));
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < kMaxDevices) done[dev].store(true, std::memory_order_release);
    }
    const int tiles = (rows / rows_per_seq) * ((rows_per_seq + P::QT - 1) / P::QT);
    return launch_pdl(attention_prefill_kernel<G, HD>, dim3(kv_heads, splits, tiles), dim3(kThreads), P::smem_bytes(),
                      s, q, kc, vc, scores, heads, kv_heads, max_seq, layer, scale, q_stride, pos, rows_per_seq,
                      cache_stride, err);
}

template <int G, int HD>
cudaError_t launch_prefill_flash_g(int rows, int rows_per_seq, cudaStream_t s, const float* q, const float* kc,
                                   const float* vc, float* ctx, int heads, int kv_heads, int max_seq, int layer,
                                   float scale, int q_stride, const int32_t* pos, int64_t cache_stride, int32_t* err) {
    using F = PrefillFlash<G, HD>;
    constexpr int kMaxDevices = 64;
    static std::atomic<bool> done[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (!(dev >= 0 && dev < kMaxDevices && done[dev].load(std::memory_order_acquire))) {
        e = cudaFuncSetAttribute(attention_prefill_flash_kernel<G, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(F::smem_bytes()));
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < kMaxDevices) done[dev].store(true, std::memory_order_release);
    }
    // the caches of this call's sequences as 2-D [rows][HD] tensors, boxes of 32 floats x 64 positions
    const int64_t rows_per_seq_cache = cache_stride / HD;
    const int64_t cache_rows = static_cast<int64_t>(rows / rows_per_seq) * rows_per_seq_cache;
    if (cache_rows > INT32_MAX) return cudaErrorInvalidValue;
    alignas(64) CUtensorMap tk, tv;
    if (!encode_tmap_2d(&tk, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, kc, HD, static_cast<uint64_t>(cache_rows),
                        HD * sizeof(float), 32, kSpan, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_tmap_2d(&tv, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, vc, HD, static_cast<uint64_t>(cache_rows),
                        HD * sizeof(float), 32, kSpan, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    const int tiles = (rows / rows_per_seq) * ((rows_per_seq + F::QT - 1) / F::QT);
    return launch_pdl(attention_prefill_flash_kernel<G, HD>, dim3(kv_heads, tiles), dim3(kThreads), F::smem_bytes(), s,
                      tk, tv, q, ctx, heads, kv_heads, max_seq, layer, scale, q_stride, pos, rows_per_seq,
                      rows_per_seq_cache, err);
}

template <int HD>
cudaError_t launch_prefill_flash(int group, int rows, int rows_per_seq, cudaStream_t s, const float* q,
                                 const float* kc, const float* vc, float* ctx, int heads, int kv_heads, int max_seq,
                                 int layer, float scale, int q_stride, const int32_t* pos, int64_t cache_stride,
                                 int32_t* err) {
#define KT_FLASH_CASE(G_)                                                                                       \
    return launch_prefill_flash_g<G_, HD>(rows, rows_per_seq, s, q, kc, vc, ctx, heads, kv_heads, max_seq, layer, \
                                          scale, q_stride, pos, cache_stride, err)
    switch (group) {
        case 1: KT_FLASH_CASE(1);
        case 2: KT_FLASH_CASE(2);
        case 3: KT_FLASH_CASE(3);
        case 4: KT_FLASH_CASE(4);
        case 5: KT_FLASH_CASE(5);
        case 6: KT_FLASH_CASE(6);
        case 7: KT_FLASH_CASE(7);
        default: KT_FLASH_CASE(8);
    }
#undef KT_FLASH_CASE
}

template <int HD>
cudaError_t launch_prefill_attention(int group, int rows, int rows_per_seq, int splits, cudaStream_t s,
                                     const float* q, const float* kc, const float* vc, float* scores, int heads,
                                     int kv_heads, int max_seq, int layer, float scale, int q_stride,
                                     const int32_t* pos, int64_t cache_stride, int32_t* err) {
#define KT_PREFILL_CASE(G_)                                                                                      \
    return launch_prefill_attention_g<G_, HD>(rows, rows_per_seq, splits, s, q, kc, vc, scores, heads, kv_heads, \
                                              max_seq, layer, scale, q_stride, pos, cache_stride, err)
    switch (group) {
        case 1: KT_PREFILL_CASE(1);
        case 2: KT_PREFILL_CASE(2);
        case 3: KT_PREFILL_CASE(3);
        case 4: KT_PREFILL_CASE(4);
        case 5: KT_PREFILL_CASE(5);
        case 6: KT_PREFILL_CASE(6);
        case 7: KT_PREFILL_CASE(7);
        default: KT_PREFILL_CASE(8);
    }
#undef KT_PREFILL_CASE
}

cudaError_t launch_attention_decode(const float* q, const float* kc, const float* vc, float* ctx, float* scores,
                                    int rows, int q_stride, int heads, int kv_heads, int head_dim, int max_seq,
                                    int layer, float scale, const int32_t* pos, int rows_per_seq,
                                    int64_t cache_stride, int32_t* err, cudaStream_t s) {
    if (head_dim > kMaxHeadDim) return cudaErrorInvalidValue;
    const int splits = (max_seq + kSpan - 1) / kSpan;
    const int group = heads / kv_heads;
    const dim3 ggrid(kv_heads, splits, rows);
    // staged: head_dim 64 / 128, cache rows on 16-byte boundaries (bulk copies)
    const bool aligned = (reinterpret_cast<uintptr_t>(kc) & 15) == 0 && (reinterpret_cast<uintptr_t>(vc) & 15) == 0 &&
                         cache_stride % 4 == 0;
    // a prompt: tiles of query rows per block (the query rows copied in bulk too)
    if (rows_per_seq > 1 && prefill_attention_enabled() && aligned && group <= 8 && (head_dim == 64 || head_dim == 128) &&
        (reinterpret_cast<uintptr_t>(q) & 15) == 0 && q_stride % 4 == 0) {
        if (rows >= 9 && prefill_mma_enabled() && cache_stride % head_dim == 0) {
            // (the TMA maps view the caches as [rows][head_dim]: sequences a whole number of rows apart)
            // 9 rows or more: the block's matmuls run on the bf16 GEMM, whose tolerance covers the TF32 products
            return head_dim == 64 ? launch_prefill_flash<64>(group, rows, rows_per_seq, s, q, kc, vc, ctx, heads,
                                                             kv_heads, max_seq, layer, scale, q_stride, pos,
                                                             cache_stride, err)
                                  : launch_prefill_flash<128>(group, rows, rows_per_seq, s, q, kc, vc, ctx, heads,
                                                              kv_heads, max_seq, layer, scale, q_stride, pos,
                                                              cache_stride, err);
        }
        const cudaError_t e =
            head_dim == 64 ? launch_prefill_attention<64>(group, rows, rows_per_seq, splits, s, q, kc, vc, scores,
                                                          heads, kv_heads, max_seq, layer, scale, q_stride, pos,
                                                          cache_stride, err)
                           : launch_prefill_attention<128>(group, rows, rows_per_seq, splits, s, q, kc, vc, scores,
                                                           heads, kv_heads, max_seq, layer, scale, q_stride, pos,
                                                           cache_stride, err);
        if (e != cudaSuccess) return e;
        launch_pdl(attention_merge_kernel, dim3(dim3(heads, rows)), dim3(128), 0, s, scores, ctx, heads, head_dim,
                   max_seq, pos, rows_per_seq);
        return cudaGetLastError();
    }
    if (staged_attention_enabled() && aligned && group <= 8 && (head_dim == 64 || head_dim == 128)) {
        const cudaError_t e =
            head_dim == 64
                ? launch_staged_attention<64>(ggrid, group, s, q, kc, vc, scores, heads, kv_heads, max_seq, layer,
                                              scale, q_stride, pos, rows_per_seq, cache_stride, err)
                : launch_staged_attention<128>(ggrid, group, s, q, kc, vc, scores, heads, kv_heads, max_seq, layer,
                                               scale, q_stride, pos, rows_per_seq, cache_stride, err);
        if (e != cudaSuccess) return e;
        launch_pdl(attention_merge_kernel, dim3(dim3(heads, rows)), dim3(128), 0, s, scores, ctx, heads, head_dim,
                   max_seq, pos, rows_per_seq);
        return cudaGetLastError();
    }
#define KT_GROUP_CASE(G_, KP_)                                                                                     \
    launch_pdl(attention_group_kernel<G_, KP_>, dim3(ggrid), dim3(kThreads), 0, s, q, kc, vc, scores, heads, kv_heads, head_dim,       \
                                                               max_seq, layer, scale, q_stride, pos, rows_per_seq, \
                                                               cache_stride)
    bool grouped = true;
    if (group >= 2 && group <= 8 && head_dim <= 64) {
        switch (group) {
            case 2: KT_GROUP_CASE(2, 2); break;
            case 3: KT_GROUP_CASE(3, 2); break;
            case 4: KT_GROUP_CASE(4, 2); break;
            case 5: KT_GROUP_CASE(5, 2); break;
            case 6: KT_GROUP_CASE(6, 2); break;
            case 7: KT_GROUP_CASE(7, 2); break;
            default: KT_GROUP_CASE(8, 2); break;
        }
    } else if (group >= 2 && group <= 8 && head_dim <= 128) {
        switch (group) {
            case 2: KT_GROUP_CASE(2, 4); break;
            case 3: KT_GROUP_CASE(3, 4); break;
            case 4: KT_GROUP_CASE(4, 4); break;
            case 5: KT_GROUP_CASE(5, 4); break;
            case 6: KT_GROUP_CASE(6, 4); break;
            case 7: KT_GROUP_CASE(7, 4); break;
            default: KT_GROUP_CASE(8, 4); break;
        }
    } else {
        grouped = false;
    }
#undef KT_GROUP_CASE
    if (!grouped) {
        const dim3 grid(heads, splits, rows);
        launch_pdl(attention_partial_kernel, dim3(grid), dim3(kThreads), 0, s, q, kc, vc, scores, heads, kv_heads, head_dim, max_seq,
                                                           layer, scale, q_stride, pos, rows_per_seq, cache_stride);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    launch_pdl(attention_merge_kernel, dim3(dim3(heads, rows)), dim3(128), 0, s, scores, ctx, heads, head_dim, max_seq, pos,
                                                             rows_per_seq);
    return cudaGetLastError();
}
cudaError_t launch_silu_mul(float* gate, const float* up, int64_t n, cudaStream_t s) {
    launch_pdl(silu_mul_kernel, dim3(grid_for(n)), dim3(kThreads), 0, s, gate, up, n);
    return cudaGetLastError();
}
cudaError_t launch_silu_mul_rows(const float* gu, float* out, int rows, int hidden, cudaStream_t s) {
    launch_pdl(silu_mul_rows_kernel, dim3(grid_for(static_cast<int64_t>(rows) * hidden)), dim3(kThreads), 0, s, gu, out, rows, hidden);
    return cudaGetLastError();
}
cudaError_t launch_add(float* x, const float* y, int64_t n, cudaStream_t s) {
    launch_pdl(add_kernel, dim3(grid_for(n)), dim3(kThreads), 0, s, x, y, n);
    return cudaGetLastError();
}
size_t argmax_scratch_bytes(int rows) { return static_cast<size_t>(rows) * 128 * 8; }

cudaError_t launch_argmax(const float* logits, int rows, int n, int32_t* out, void* scratch, cudaStream_t s) {
    const int chunks = std::min(128, std::max(1, (n + 2047) / 2048));
    const int chunk = (n + chunks - 1) / chunks;
    float* pv = static_cast<float*>(scratch);
    int* pi = reinterpret_cast<int*>(pv + static_cast<size_t>(rows) * 128);
    launch_pdl(argmax_partial_kernel, dim3(dim3(chunks, rows)), dim3(kThreads), 0, s, logits, n, chunk, pv, pi);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    launch_pdl(argmax_merge_kernel, dim3(rows), dim3(32), 0, s, pv, pi, chunks, out);
    return cudaGetLastError();
}
cudaError_t launch_dequantize_column(const QView& w, const int32_t* col, int count, float* out, int32_t* status,
                                     cudaStream_t s) {
    launch_pdl(dequantize_column_kernel, dim3(dim3(grid_for(w.rows), count)), dim3(kThreads), 0, s, w, col, out, status);
    return cudaGetLastError();
}
cudaError_t launch_increment(int32_t* p, int32_t delta, cudaStream_t s) {
    launch_pdl(increment_kernel, dim3(1), dim3(1), 0, s, p, delta);
    return cudaGetLastError();
}

}  // namespace kt
