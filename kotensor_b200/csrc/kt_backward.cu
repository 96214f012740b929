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

}  // namespace

cudaError_t launch_matmul_t(const QView& w, const float* dy, float* dx, int32_t m, int32_t accumulate,
                            cudaStream_t s) {
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
