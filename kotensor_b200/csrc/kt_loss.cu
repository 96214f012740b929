// kt_loss.cu -- fusedCrossEntropyLoss with a quantized head
// (Engine/kotensor/src/main/kotlin/Loss.kt:114-220): per chunk of active rows,
// the logits come from the quantized matmul (with the head's bias), then one
// block per row takes the max (floor -1e9), the sum of exponentials and the
// row's loss; for the backward the logits are turned in place into
// scale * (softmax - onehot) (logitGradients, Loss.kt:264-280), summed per
// column into the bias gradient, and sent back through the head with the
// transposed quantized matmul (multiplyByQuantizedTransposed) into the rows of
// the hidden gradient.  Reductions run in fixed orders: deterministic results.
#include "kt_internal.h"

namespace kt {
namespace {

constexpr int kThreads = 256;

__global__ void gather_rows_kernel(const float* __restrict__ src, const int32_t* __restrict__ rows, int32_t count,
                                   int32_t dim, float* __restrict__ dst) {
    const int64_t n = static_cast<int64_t>(count) * dim;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / dim, d = i - r * dim;
        dst[i] = src[static_cast<int64_t>(rows[r]) * dim + d];
    }
}

template <bool MAX>
__device__ float block_reduce(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float u = __shfl_xor_sync(0xffffffffu, v, o);
        v = MAX ? fmaxf(v, u) : v + u;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = red[0];
    for (int w = 1; w < kThreads / 32; ++w) r = MAX ? fmaxf(r, red[w]) : r + red[w];
    return r;
}

// One block per row of the chunk: row max (at least -1e9, Loss.kt:150-156),
// sum of exp(logit - max), and the row's loss max + ln(sum) - logit[target].
__global__ void __launch_bounds__(kThreads) row_stats_kernel(const float* __restrict__ logits, int32_t vocab,
                                                             const int32_t* __restrict__ targets,
                                                             float* __restrict__ row_max, float* __restrict__ row_sum,
                                                             float* __restrict__ row_loss) {
    __shared__ float red[kThreads / 32];
    const int r = blockIdx.x;
    const float* l = logits + static_cast<int64_t>(r) * vocab;
    float mx = -1e9f;
    for (int v = threadIdx.x; v < vocab; v += kThreads) mx = fmaxf(mx, l[v]);
    mx = block_reduce<true>(mx, red);
    float s = 0.0f;
    for (int v = threadIdx.x; v < vocab; v += kThreads) s += expf(l[v] - mx);
    s = block_reduce<false>(s, red);
    if (threadIdx.x == 0) {
        row_max[r] = mx;
        row_sum[r] = s;
        row_loss[r] = mx + logf(s) - l[targets[r]];
    }
}

// logits <- scale * (exp(logit - max) / sum - [v == target]), in place.
__global__ void logit_grad_kernel(float* __restrict__ logits, int32_t count, int32_t vocab,
                                  const int32_t* __restrict__ targets, const float* __restrict__ row_max,
                                  const float* __restrict__ row_sum, float scale) {
    const int64_t n = static_cast<int64_t>(count) * vocab;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / vocab;
        const int v = static_cast<int>(i - r * vocab);
        const float prob = expf(logits[i] - row_max[r]) * (1.0f / row_sum[r]);
        logits[i] = scale * (prob - (v == targets[r] ? 1.0f : 0.0f));
    }
}

// bias_grad[v] += sum over the chunk's rows (in row order) of the logit gradients.
__global__ void bias_grad_kernel(const float* __restrict__ grads, int32_t count, int32_t vocab,
                                 float* __restrict__ bias_grad) {
    for (int v = blockIdx.x * blockDim.x + threadIdx.x; v < vocab; v += gridDim.x * blockDim.x) {
        float s = bias_grad[v];
        for (int r = 0; r < count; ++r) s += grads[static_cast<int64_t>(r) * vocab + v];
        bias_grad[v] = s;
    }
}

// dst[rows[r]] += src[r] (rows are distinct).
__global__ void scatter_add_rows_kernel(const float* __restrict__ src, const int32_t* __restrict__ rows,
                                        int32_t count, int32_t dim, float* __restrict__ dst) {
    const int64_t n = static_cast<int64_t>(count) * dim;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / dim, d = i - r * dim;
        dst[static_cast<int64_t>(rows[r]) * dim + d] += src[i];
    }
}

// loss = (sum of the row losses in row order) / active (Loss.kt:162, :189).
__global__ void mean_loss_kernel(const float* __restrict__ row_loss, int32_t active, float* __restrict__ out) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        float total = 0.0f;
        for (int r = 0; r < active; ++r) total += row_loss[r];
        *out = total / static_cast<float>(active);
    }
}

unsigned grid_for(int64_t n) { return static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 148 * 16)); }

}  // namespace

// Logit elements per chunk: bounds the chunk's logits buffer to 256 MiB.
constexpr int64_t kLossChunkElements = static_cast<int64_t>(1) << 26;

int32_t loss_chunk_rows(int32_t vocab, int32_t active) {
    return static_cast<int32_t>(std::max<int64_t>(1, std::min<int64_t>(kLossChunkElements / vocab, active)));
}

cudaError_t launch_gather_rows(const float* src, const int32_t* rows, int32_t count, int32_t dim, float* dst,
                               cudaStream_t s) {
    gather_rows_kernel<<<grid_for(static_cast<int64_t>(count) * dim), 256, 0, s>>>(src, rows, count, dim, dst);
    return cudaGetLastError();
}

cudaError_t launch_loss_rows(const float* logits, int32_t count, int32_t vocab, const int32_t* targets,
                             float* row_max, float* row_sum, float* row_loss, cudaStream_t s) {
    row_stats_kernel<<<count, kThreads, 0, s>>>(logits, vocab, targets, row_max, row_sum, row_loss);
    return cudaGetLastError();
}

cudaError_t launch_loss_grads(float* logits, int32_t count, int32_t vocab, const int32_t* targets,
                              const float* row_max, const float* row_sum, float scale, float* bias_grad,
                              cudaStream_t s) {
    logit_grad_kernel<<<grid_for(static_cast<int64_t>(count) * vocab), 256, 0, s>>>(logits, count, vocab, targets,
                                                                                    row_max, row_sum, scale);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess && bias_grad != nullptr) {
        bias_grad_kernel<<<grid_for(vocab), 256, 0, s>>>(logits, count, vocab, bias_grad);
        e = cudaGetLastError();
    }
    return e;
}

cudaError_t launch_scatter_add_rows(const float* src, const int32_t* rows, int32_t count, int32_t dim, float* dst,
                                    cudaStream_t s) {
    scatter_add_rows_kernel<<<grid_for(static_cast<int64_t>(count) * dim), 256, 0, s>>>(src, rows, count, dim, dst);
    return cudaGetLastError();
}

cudaError_t launch_mean_loss(const float* row_loss, int32_t active, float* out, cudaStream_t s) {
    mean_loss_kernel<<<1, 32, 0, s>>>(row_loss, active, out);
    return cudaGetLastError();
}

}  // namespace kt
