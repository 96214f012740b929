// kt_lora.cu -- the low-rank adapter of LoRALinear over a quantized base
// (Engine/kotensor/src/main/kotlin/LoRA.kt:7-57): the projection p = a . A that
// the matmul epilogue consumes (forwardInto, LoRA.kt:39-46), and the gradients
// of LoRALinear.forward (LoRA.kt:31-36) through the autograd of its matmuls.
//
// Shapes (row-major fp32 on the device): a [m x K], A [K x rank], B [rank x N],
// p [m x rank], dy [m x N].  With G = dy . B^T [m x rank]:
//   dx += scale * G . A^T      dA += scale * a^T . G      dB += scale * p^T . dy
// (dx's quantized part is MatMul.multiplyByQuantizedTransposed, kt_backward.cu).
//
// Every sum runs in a fixed order (per-thread sequential sums, fixed-shape
// block reductions, split partials added in split order by the last block of a
// row), so results are deterministic.  These are small products next to the
// weight stream of the base matmul: A and B together are (K + N) * rank floats.
#include "kt_internal.h"

namespace kt {
namespace {

constexpr int kThreads = 256;
constexpr int kSliceRows = 256;  // rows of A (or columns of B) per block

__device__ __forceinline__ int atomic_add_acq_rel(int32_t* p, int v) {
    int old;
    asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// The last of a row's `splits` blocks to arrive sums the row's partials in
// split order into out[t][0..rank) and re-arms the row's counter.
__device__ void finish_row(const float* partials, int32_t* tickets, float* out, int t, int splits, int rank) {
    __shared__ int s_last;
    __syncthreads();  // this block's partial stores precede thread 0's acq_rel atomic
    if (threadIdx.x == 0) s_last = atomic_add_acq_rel(tickets + t, 1) == splits - 1;
    __syncthreads();
    if (!s_last) return;
    const float* rowp = partials + static_cast<int64_t>(t) * splits * rank;
    for (int r = threadIdx.x; r < rank; r += blockDim.x) {
        float v = 0.0f;
        for (int s = 0; s < splits; ++s) v += __ldcg(rowp + static_cast<int64_t>(s) * rank + r);
        out[static_cast<int64_t>(t) * rank + r] = v;
    }
    if (threadIdx.x == 0) tickets[t] = 0;
}

// p[t][r] = sum_k a[t][k] * A[k][r].  Block (split, t) covers rows
// [split * kSliceRows, ...) of A; that slice of A is contiguous, and with
// T = rank * floor(256 / rank) threads stepping by T through it each thread
// keeps one fixed r.  Threads of equal r are then summed in thread order.
__global__ void __launch_bounds__(kThreads) project_a_kernel(const float* __restrict__ a, const float* __restrict__ A,
                                                             int32_t K, int32_t rank, float* __restrict__ partials,
                                                             int32_t* tickets, float* __restrict__ out) {
    __shared__ float red[kThreads];
    const int t = blockIdx.y, split = blockIdx.x, splits = gridDim.x;
    const int T = rank * (kThreads / rank);
    const int k0 = split * kSliceRows, k1 = min(K, k0 + kSliceRows);
    const float* arow = a + static_cast<int64_t>(t) * K;
    float acc = 0.0f;
    if (threadIdx.x < T) {
        const int64_t f0 = static_cast<int64_t>(k0) * rank, f1 = static_cast<int64_t>(k1) * rank;
        for (int64_t f = f0 + threadIdx.x; f < f1; f += T) acc = fmaf(__ldg(arow + f / rank), __ldg(A + f), acc);
    }
    red[threadIdx.x] = acc;
    __syncthreads();
    float* dst = splits == 1 ? out + static_cast<int64_t>(t) * rank
                             : partials + (static_cast<int64_t>(t) * splits + split) * rank;
    for (int r = threadIdx.x; r < rank; r += kThreads) {
        float v = 0.0f;
        for (int j = r; j < T; j += rank) v += red[j];
        dst[r] = v;
    }
    if (splits > 1) finish_row(partials, tickets, out, t, splits, rank);
}

// g[t][r] = sum_j dy[t][j] * B[r][j].  Block (split, t) covers columns
// [split * kSliceRows * 4, ...); one fixed-shape block reduction per r.
constexpr int kSliceCols = kSliceRows * 4;
__global__ void __launch_bounds__(kThreads) project_bt_kernel(const float* __restrict__ dy,
                                                              const float* __restrict__ B, int32_t N, int32_t rank,
                                                              float* __restrict__ partials, int32_t* tickets,
                                                              float* __restrict__ out) {
    __shared__ float red[kThreads / 32];
    const int t = blockIdx.y, split = blockIdx.x, splits = gridDim.x;
    const int j0 = split * kSliceCols, j1 = min(N, j0 + kSliceCols);
    const float* drow = dy + static_cast<int64_t>(t) * N;
    float* dst = splits == 1 ? out + static_cast<int64_t>(t) * rank
                             : partials + (static_cast<int64_t>(t) * splits + split) * rank;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int r = 0; r < rank; ++r) {
        const float* brow = B + static_cast<int64_t>(r) * N;
        float acc = 0.0f;
        for (int j = j0 + threadIdx.x; j < j1; j += kThreads) acc = fmaf(__ldg(drow + j), __ldg(brow + j), acc);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (lane == 0) red[warp] = acc;
        __syncthreads();
        if (threadIdx.x == 0) {
            float v = 0.0f;
            for (int w = 0; w < kThreads / 32; ++w) v += red[w];
            dst[r] = v;
        }
        __syncthreads();
    }
    if (splits > 1) finish_row(partials, tickets, out, t, splits, rank);
}

// dx[t][k] (+)= scale * sum_r g[t][r] * A[k][r]
__global__ void dx_kernel(const float* __restrict__ g, const float* __restrict__ A, int32_t m, int32_t K,
                          int32_t rank, float scale, float* __restrict__ dx) {
    const int64_t n = static_cast<int64_t>(m) * K;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / K, k = i - t * K;
        const float* gr = g + t * rank;
        const float* ar = A + k * rank;
        float s = 0.0f;
        for (int r = 0; r < rank; ++r) s = fmaf(__ldg(gr + r), __ldg(ar + r), s);
        dx[i] = fmaf(scale, s, dx[i]);
    }
}

// dA[k][r] += scale * sum_t a[t][k] * g[t][r]
__global__ void grad_a_kernel(const float* __restrict__ a, const float* __restrict__ g, int32_t m, int32_t K,
                              int32_t rank, float scale, float* __restrict__ dA) {
    const int64_t n = static_cast<int64_t>(K) * rank;
    for (int64_t f = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; f < n;
         f += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t k = f / rank;
        const int r = static_cast<int>(f - k * rank);
        float s = 0.0f;
        for (int t = 0; t < m; ++t)
            s = fmaf(__ldg(a + static_cast<int64_t>(t) * K + k), __ldg(g + static_cast<int64_t>(t) * rank + r), s);
        dA[f] = fmaf(scale, s, dA[f]);
    }
}

// dB[r][j] += scale * sum_t p[t][r] * dy[t][j]
__global__ void grad_b_kernel(const float* __restrict__ p, const float* __restrict__ dy, int32_t m, int32_t N,
                              int32_t rank, float scale, float* __restrict__ dB) {
    const int64_t n = static_cast<int64_t>(rank) * N;
    for (int64_t f = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; f < n;
         f += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = f / N, j = f - r * N;
        float s = 0.0f;
        for (int t = 0; t < m; ++t)
            s = fmaf(__ldg(p + static_cast<int64_t>(t) * rank + r), __ldg(dy + static_cast<int64_t>(t) * N + j), s);
        dB[f] = fmaf(scale, s, dB[f]);
    }
}

unsigned grid_for(int64_t n) { return static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 148 * 16)); }

int splits_for(int64_t extent, int64_t per, int32_t m) {
    const int64_t s = (extent + per - 1) / per;
    // one arrival counter per row: more rows than counters run unsplit
    return m > kTicketCapEach ? 1 : static_cast<int>(std::max<int64_t>(1, s));
}

}  // namespace

size_t lora_workspace_bytes(int32_t m, int32_t K, int32_t N, int32_t rank) {
    const int64_t sa = splits_for(K, kSliceRows, m), sb = splits_for(N, kSliceCols, m);
    const int64_t parts = static_cast<int64_t>(m) * std::max(sa, sb) * rank;
    // partials, then g [m x rank] for the backward
    return kWorkspaceReservedBytes + static_cast<size_t>(parts + static_cast<int64_t>(m) * rank) * sizeof(float);
}

cudaError_t launch_lora_project(const float* a, int32_t m, int32_t K, const float* A, int32_t rank, float* p,
                                void* workspace, cudaStream_t s) {
    auto* ws = static_cast<unsigned char*>(workspace);
    const int splits = splits_for(K, kSliceRows, m);
    project_a_kernel<<<dim3(splits, m), kThreads, 0, s>>>(a, A, K, rank,
                                                          reinterpret_cast<float*>(ws + kWorkspaceReservedBytes),
                                                          reinterpret_cast<int32_t*>(ws + kLoraTicketOffset), p);
    return cudaGetLastError();
}

cudaError_t launch_lora_backward(const float* a, const float* dy, const float* p, const float* A, const float* B,
                                 int32_t m, int32_t K, int32_t N, int32_t rank, float scale, float* dx, float* dA,
                                 float* dB, void* workspace, cudaStream_t s) {
    auto* ws = static_cast<unsigned char*>(workspace);
    const int sa = splits_for(K, kSliceRows, m), sb = splits_for(N, kSliceCols, m);
    auto* partials = reinterpret_cast<float*>(ws + kWorkspaceReservedBytes);
    float* g = partials + static_cast<int64_t>(m) * std::max(sa, sb) * rank;
    auto* tickets = reinterpret_cast<int32_t*>(ws + kLoraTicketOffset);
    cudaError_t e = cudaSuccess;
    if (dx != nullptr || dA != nullptr) {
        project_bt_kernel<<<dim3(sb, m), kThreads, 0, s>>>(dy, B, N, rank, partials, tickets, g);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess && dx != nullptr) {
        dx_kernel<<<grid_for(static_cast<int64_t>(m) * K), 256, 0, s>>>(g, A, m, K, rank, scale, dx);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess && dA != nullptr) {
        grad_a_kernel<<<grid_for(static_cast<int64_t>(K) * rank), 256, 0, s>>>(a, g, m, K, rank, scale, dA);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess && dB != nullptr) {
        grad_b_kernel<<<grid_for(static_cast<int64_t>(rank) * N), 256, 0, s>>>(p, dy, m, N, rank, scale, dB);
        e = cudaGetLastError();
    }
    (void)sa;
    return e;
}

}  // namespace kt
