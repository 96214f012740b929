// kt_backward.cu -- MatMul.multiplyByQuantizedTransposed
// (Engine/kotensor/src/main/kotlin/MatMul.kt:954-981):
//   dx[m x K] = (accumulate ? dx : 0) + dy[m x N] . dequant(W)^T
// The reference dequantizes one K-row of W (QuantizedTensor.dequantizeRow,
// QuantizedTensor.kt:188-213) and takes its dot product with every dy row.
// Here one warp owns one K-row: the lanes stride over the packed bytes of the
// row (coalesced), dequantize each weight as scale * (q - zero) in registers,
// accumulate up to 8 dy rows at once, and reduce across the warp with an
// xor-shuffle butterfly (fixed order, deterministic).
#include "kt_internal.h"

namespace kt {
namespace {

constexpr int kRowsPerPass = 8;

struct BackParams {
    QView w;
    const float* dy;
    float* dx;
    int32_t m0, mc;  // dy / dx rows handled by this launch
    int32_t accumulate;
};

__global__ void __launch_bounds__(256) matmul_t_kernel(BackParams p) {
    const int lane = threadIdx.x & 31;
    const int l = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);  // K-row of W
    if (l >= p.w.rows) return;
    const int N = p.w.columns, R = p.w.bytes_per_row;
    const int64_t go = static_cast<int64_t>(l / p.w.group_size) * N;
    const uint8_t* q = p.w.q + static_cast<int64_t>(l) * R;
    const float* s = p.w.scales + go;
    float acc[kRowsPerPass];
#pragma unroll
    for (int i = 0; i < kRowsPerPass; ++i) acc[i] = 0.0f;
    const float* dy = p.dy + static_cast<int64_t>(p.m0) * N;
    if (p.w.bits == 8) {
        for (int c = lane; c < N; c += 32) {
            const float wv = __fmul_rn(s[c], static_cast<float>(static_cast<int8_t>(q[c])));
#pragma unroll
            for (int i = 0; i < kRowsPerPass; ++i)
                if (i < p.mc) acc[i] = fmaf(dy[static_cast<int64_t>(i) * N + c], wv, acc[i]);
        }
    } else {
        const uint8_t* z = p.w.zeros + go;
        const int half = R;
        for (int b = lane; b < R; b += 32) {
            const uint8_t byte = q[b];
            const float w_lo = __fmul_rn(s[b], static_cast<float>((byte & 0xF) - static_cast<int>(z[b])));
            const int c_hi = half + b;
            const bool has_hi = c_hi < N;
            const float w_hi =
                has_hi ? __fmul_rn(s[c_hi], static_cast<float>((byte >> 4) - static_cast<int>(z[c_hi]))) : 0.0f;
#pragma unroll
            for (int i = 0; i < kRowsPerPass; ++i) {
                if (i < p.mc) {
                    const float* d = dy + static_cast<int64_t>(i) * N;
                    acc[i] = fmaf(d[b], w_lo, acc[i]);
                    if (has_hi) acc[i] = fmaf(d[c_hi], w_hi, acc[i]);
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < kRowsPerPass; ++i)
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], off);
    if (lane == 0) {
        for (int i = 0; i < p.mc; ++i) {
            float* out = p.dx + static_cast<int64_t>(p.m0 + i) * p.w.rows + l;
            *out = p.accumulate ? *out + acc[i] : acc[i];
        }
    }
}

// ---- tiled kernel (bytes_per_row % 16 == 0): a CTA owns one group of rows
// and one chunk of kChunk packed bytes (INT4: the chunk's low- and
// high-nibble columns).  Per group the factoring of the reference's forward
// combine (MatMul.kt:804-828) applies transposed:
//   dx[l] = sum_c dys[c] q[l,c] - sum_c dys[c] zero[c],   dys[c] = dy[c] * scale[g,c]
// dys is staged once per CTA in shared memory ([j][lane] order, so each lane's
// 16 bytes read conflict-free), held in registers across the group's rows, and
// each chunk's per-row partial sums go to a workspace; a second kernel adds the
// chunks in fixed order.
constexpr int kChunk = 512;      // packed bytes per CTA
constexpr int kTWarps = 8;

template <int BITS, int MT>
__global__ void __launch_bounds__(kTWarps * 32) matmul_t_tiled_kernel(QView w, const float* __restrict__ dy,
                                                                      int32_t m0, float* __restrict__ partial) {
    __shared__ float dys_lo[MT][16][32];
    __shared__ float dys_hi[MT][16][32];
    __shared__ float zc_part[MT][kTWarps];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gi = blockIdx.x, chunk = blockIdx.y;
    const int N = w.columns, R = w.bytes_per_row, K = w.rows;
    const int b0 = chunk * kChunk;
    const int64_t go = static_cast<int64_t>(gi) * N;
    // stage dys (0 beyond the row's bytes / columns) and the zero-point correction
    float zc[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) zc[t] = 0.0f;
    for (int idx = tid; idx < kChunk; idx += kTWarps * 32) {
        const int b = b0 + idx;
        const int ln = idx >> 4, j = idx & 15;  // byte idx belongs to lane ln, position j
#pragma unroll
        for (int t = 0; t < MT; ++t) {
            const float* dyt = dy + static_cast<int64_t>(m0 + t) * N;
            float lo = 0.0f, hi = 0.0f;
            if (b < R) {
                lo = dyt[b] * w.scales[go + b];
                if constexpr (BITS == 4) {
                    zc[t] = fmaf(lo, static_cast<float>(w.zeros[go + b]), zc[t]);
                    if (R + b < N) {
                        hi = dyt[R + b] * w.scales[go + R + b];
                        zc[t] = fmaf(hi, static_cast<float>(w.zeros[go + R + b]), zc[t]);
                    }
                }
            }
            dys_lo[t][j][ln] = lo;
            if constexpr (BITS == 4) dys_hi[t][j][ln] = hi;
        }
    }
#pragma unroll
    for (int t = 0; t < MT; ++t) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) zc[t] += __shfl_xor_sync(0xffffffffu, zc[t], off);
        if (lane == 0) zc_part[t][warp] = zc[t];
    }
    __syncthreads();
    float zsum[MT];
#pragma unroll
    for (int t = 0; t < MT; ++t) {
        float v = 0.0f;
#pragma unroll
        for (int q = 0; q < kTWarps; ++q) v += zc_part[t][q];
        zsum[t] = v;
    }
    // this lane's 16 bytes of the chunk, its dys in registers
    float dl[MT][16], dh[MT][16];
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            dl[t][j] = dys_lo[t][j][lane];
            dh[t][j] = BITS == 4 ? dys_hi[t][j][lane] : 0.0f;
        }
    const int bl = b0 + 16 * lane;
    const bool lane_in = bl < R;  // R % 16 == 0: a lane's 16 bytes are all in or all out
    const int r0 = gi * w.group_size, r1 = min(r0 + w.group_size, K);
    for (int l = r0 + warp; l < r1; l += kTWarps) {
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (lane_in) v = __ldg(reinterpret_cast<const uint4*>(w.q + static_cast<int64_t>(l) * R + bl));
        const uint32_t word[4] = {v.x, v.y, v.z, v.w};
        float acc[MT];
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[t] = 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const uint32_t byte = (word[j >> 2] >> (8 * (j & 3))) & 0xFFu;
            if constexpr (BITS == 4) {
                // 2^23 + q as a float minus 2^23 is exactly q
                const float ql = __uint_as_float(0x4B000000u | (byte & 15u)) - 8388608.0f;
                const float qh = __uint_as_float(0x4B000000u | (byte >> 4)) - 8388608.0f;
#pragma unroll
                for (int t = 0; t < MT; ++t) acc[t] = fmaf(qh, dh[t][j], fmaf(ql, dl[t][j], acc[t]));
            } else {
                const float q = __uint_as_float(byte ^ 0x4B000080u) - 8388736.0f;  // signed byte
#pragma unroll
                for (int t = 0; t < MT; ++t) acc[t] = fmaf(q, dl[t][j], acc[t]);
            }
        }
#pragma unroll
        for (int t = 0; t < MT; ++t) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], off);
        }
        if (lane == 0) {
#pragma unroll
            for (int t = 0; t < MT; ++t)
                partial[(static_cast<int64_t>(chunk) * MT + t) * K + l] = acc[t] - zsum[t];
        }
    }
}

// dx[m0 + t][l] = (accumulate ? dx : 0) + sum over chunks (in order) of partial
__global__ void matmul_t_reduce_kernel(const float* __restrict__ partial, int32_t chunks, int32_t mt, int32_t K,
                                       float* __restrict__ dx, int32_t m0, int32_t accumulate) {
    const int64_t total = static_cast<int64_t>(mt) * K;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float v = 0.0f;
        for (int c = 0; c < chunks; ++c) v += partial[static_cast<int64_t>(c) * total + i];
        const int64_t t = i / K, l = i - t * K;
        float* out = dx + (m0 + t) * static_cast<int64_t>(K) + l;
        *out = accumulate ? *out + v : v;
    }
}

template <int BITS, int MT>
cudaError_t launch_tiled(const QView& w, const float* dy, float* dx, int32_t m0, int32_t accumulate,
                         float* partial, cudaStream_t s) {
    const int chunks = (w.bytes_per_row + kChunk - 1) / kChunk;
    matmul_t_tiled_kernel<BITS, MT><<<dim3(w.groups, chunks), kTWarps * 32, 0, s>>>(w, dy, m0, partial);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const int64_t total = static_cast<int64_t>(MT) * w.rows;
    const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 8));
    matmul_t_reduce_kernel<<<blocks, 256, 0, s>>>(partial, chunks, MT, w.rows, dx, m0, accumulate);
    return cudaGetLastError();
}

template <int BITS>
cudaError_t launch_tiled_m(const QView& w, const float* dy, float* dx, int32_t m0, int32_t mt, int32_t accumulate,
                           float* partial, cudaStream_t s) {
    switch (mt) {
        case 1: return launch_tiled<BITS, 1>(w, dy, dx, m0, accumulate, partial, s);
        case 2: return launch_tiled<BITS, 2>(w, dy, dx, m0, accumulate, partial, s);
        case 3: return launch_tiled<BITS, 3>(w, dy, dx, m0, accumulate, partial, s);
        default: return launch_tiled<BITS, 4>(w, dy, dx, m0, accumulate, partial, s);
    }
}

constexpr int kTiledMaxM = 4;

bool tiled_supported(const QView& w) { return w.bytes_per_row % 16 == 0; }

}  // namespace

size_t matmul_t_workspace_bytes(const QView& w, int32_t m) {
    (void)m;
    if (!tiled_supported(w)) return 0;
    const size_t chunks = (w.bytes_per_row + kChunk - 1) / kChunk;
    return kWorkspaceReservedBytes + chunks * kTiledMaxM * static_cast<size_t>(w.rows) * sizeof(float);
}

cudaError_t launch_matmul_t(const QView& w, const float* dy, float* dx, int32_t m, int32_t accumulate,
                            cudaStream_t s, void* workspace, size_t workspace_bytes) {
    if (tiled_supported(w)) {
        if (workspace == nullptr || workspace_bytes < matmul_t_workspace_bytes(w, m)) return cudaErrorInvalidValue;
        float* partial = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + kWorkspaceReservedBytes);
        for (int m0 = 0; m0 < m; m0 += kTiledMaxM) {
            const int mt = std::min(kTiledMaxM, m - m0);
            const cudaError_t e = w.bits == 4 ? launch_tiled_m<4>(w, dy, dx, m0, mt, accumulate, partial, s)
                                              : launch_tiled_m<8>(w, dy, dx, m0, mt, accumulate, partial, s);
            if (e != cudaSuccess) return e;
        }
        return cudaSuccess;
    }
    const int warps = 8;
    const int blocks = (w.rows + warps - 1) / warps;
    for (int m0 = 0; m0 < m; m0 += kRowsPerPass) {
        BackParams p{w, dy, dx, m0, m - m0 < kRowsPerPass ? m - m0 : kRowsPerPass, accumulate};
        matmul_t_kernel<<<blocks, warps * 32, 0, s>>>(p);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace kt
