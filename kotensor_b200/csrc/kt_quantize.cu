// kt_quantize.cu -- device quantize/pack and dequantize kernels.
//
// quantize_kernel restates QuantizedTensor.quantize (Engine/kotensor/src/main/
// kotlin/QuantizedTensor.kt:261-324) bit for bit:
//   INT8 (quantizeSymmetric, :280-294): maxAbs over the group with a strict '>',
//     scale = maxAbs > 0 ? maxAbs / 127f : 1f, q = clamp(round(w * (1f / scale)), -127, 127)
//   INT4 (quantizeAsymmetric, :296-324): min/max with strict compares, clamped so
//     min <= 0 <= max, scale = range > 0 ? range / 15f : 1f,
//     zero = clamp(round(-min / scale), 0, 15), q = clamp(round(w * inverse) + zero, 0, 15),
//     split-half nibble packing (column c < half -> low nibble of byte c,
//     column c >= half -> high nibble of byte c - half).
// Every rounding step uses an explicit _rn intrinsic so no FMA contraction or
// approximate division can change a bit; the file is built without fast-math
// and with denormals preserved, as on the JVM.  round() is Java's Math.round
// (ties toward +infinity, saturating) and NaN is reported through the status
// word instead of trapping.
//
// Layout in HBM: one thread owns one packed byte column of one group (INT8: one
// weight column; INT4: the column pair c, c + half that shares the byte), so the
// reads of a row of the group and the byte writes are coalesced across the warp
// and no two threads ever write the same byte.
#include <climits>

#include "kt_internal.h"

namespace kt {
namespace {

// Java Math.round(float) after Kotlin's NaN check.  Returns false on NaN.
__device__ __forceinline__ bool java_round(float x, int32_t* out) {
    if (isnan(x)) return false;
    if (x >= 2147483648.0f) { *out = INT_MAX; return true; }
    if (x <= -2147483648.0f) { *out = INT_MIN; return true; }
    const float f = floorf(x);
    // x - f is exact for every float, so this is floor(x + 1/2) without the
    // rounding error of the addition (the 0.49999997f case).
    const float r = (__fsub_rn(x, f) >= 0.5f) ? __fadd_rn(f, 1.0f) : f;
    *out = static_cast<int32_t>(r);
    return true;
}

__device__ __forceinline__ int32_t clampi(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : (v > hi ? hi : v); }

// Kotlin Int '+' wraps modulo 2^32.
__device__ __forceinline__ int32_t wrap_add(int32_t a, int32_t b) {
    return static_cast<int32_t>(static_cast<uint32_t>(a) + static_cast<uint32_t>(b));
}

__global__ void __launch_bounds__(256) quantize_int8_kernel(const float* __restrict__ data, int32_t rows,
                                                            int32_t columns, int32_t group_size,
                                                            uint8_t* __restrict__ qdata, float* __restrict__ scales,
                                                            int32_t* __restrict__ status) {
    const int32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= columns) return;
    const int32_t groups = (rows + group_size - 1) / group_size;
    for (int32_t group = blockIdx.y; group < groups; group += gridDim.y) {
    const int32_t r0 = group * group_size;
    const int32_t r1 = min(r0 + group_size, rows);
    float max_abs = 0.0f;
    for (int32_t r = r0; r < r1; ++r) {
        const float v = fabsf(data[static_cast<int64_t>(r) * columns + c]);
        if (v > max_abs) max_abs = v;
    }
    const float scale = (max_abs > 0.0f) ? __fdiv_rn(max_abs, 127.0f) : 1.0f;
    scales[static_cast<int64_t>(group) * columns + c] = scale;
    const float inverse = __fdiv_rn(1.0f, scale);
    bool nan_seen = false;
    for (int32_t r = r0; r < r1; ++r) {
        const int64_t idx = static_cast<int64_t>(r) * columns + c;
        int32_t q = 0;
        if (!java_round(__fmul_rn(data[idx], inverse), &q)) nan_seen = true;
        qdata[idx] = static_cast<uint8_t>(static_cast<int8_t>(clampi(q, -127, 127)));
    }
    if (nan_seen) atomicOr(status, 1);
    }
    __threadfence();  // weight bytes visible GPU-wide before exit: matmuls read weights before their PDL wait
}

// Scale and zero point of one INT4 column over the group rows (:297-308).
__device__ __forceinline__ bool int4_params(const float* __restrict__ data, int32_t columns, int32_t r0, int32_t r1,
                                            int32_t c, float* scale_out, int32_t* zero_out) {
    float mn = 3.40282347e+38f, mx = -3.40282347e+38f;
    for (int32_t r = r0; r < r1; ++r) {
        const float v = data[static_cast<int64_t>(r) * columns + c];
        if (v < mn) mn = v;
        if (v > mx) mx = v;
    }
    if (mn > 0.0f) mn = 0.0f;
    if (mx < 0.0f) mx = 0.0f;
    const float range = __fsub_rn(mx, mn);
    const float scale = (range > 0.0f) ? __fdiv_rn(range, 15.0f) : 1.0f;
    int32_t zero = 0;
    const bool ok = java_round(__fdiv_rn(-mn, scale), &zero);
    *scale_out = scale;
    *zero_out = clampi(zero, 0, 15);
    return ok;
}

__global__ void __launch_bounds__(256) quantize_int4_kernel(const float* __restrict__ data, int32_t rows,
                                                            int32_t columns, int32_t half, int32_t group_size,
                                                            uint8_t* __restrict__ qdata, float* __restrict__ scales,
                                                            uint8_t* __restrict__ zeros,
                                                            int32_t* __restrict__ status) {
    const int32_t b = blockIdx.x * blockDim.x + threadIdx.x;  // packed byte column
    if (b >= half) return;
    const int32_t groups = (rows + group_size - 1) / group_size;
    for (int32_t group = blockIdx.y; group < groups; group += gridDim.y) {
    const int32_t r0 = group * group_size;
    const int32_t r1 = min(r0 + group_size, rows);
    const int32_t c_lo = b, c_hi = b + half;
    const bool has_hi = c_hi < columns;  // odd N: the last byte's high nibble is padding and stays 0
    bool ok = true;
    float s_lo = 1.0f, s_hi = 1.0f;
    int32_t z_lo = 0, z_hi = 0;
    ok &= int4_params(data, columns, r0, r1, c_lo, &s_lo, &z_lo);
    if (has_hi) ok &= int4_params(data, columns, r0, r1, c_hi, &s_hi, &z_hi);
    const int64_t go = static_cast<int64_t>(group) * columns;
    scales[go + c_lo] = s_lo;
    zeros[go + c_lo] = static_cast<uint8_t>(z_lo);
    if (has_hi) {
        scales[go + c_hi] = s_hi;
        zeros[go + c_hi] = static_cast<uint8_t>(z_hi);
    }
    const float inv_lo = __fdiv_rn(1.0f, s_lo);
    const float inv_hi = __fdiv_rn(1.0f, s_hi);
    for (int32_t r = r0; r < r1; ++r) {
        const int64_t row = static_cast<int64_t>(r) * columns;
        int32_t q_lo = 0, q_hi = 0;
        ok &= java_round(__fmul_rn(data[row + c_lo], inv_lo), &q_lo);
        q_lo = clampi(wrap_add(q_lo, z_lo), 0, 15);
        if (has_hi) {
            ok &= java_round(__fmul_rn(data[row + c_hi], inv_hi), &q_hi);
            q_hi = clampi(wrap_add(q_hi, z_hi), 0, 15);
        }
        qdata[static_cast<int64_t>(r) * half + b] = static_cast<uint8_t>(q_lo | (q_hi << 4));
    }
    if (!ok) atomicOr(status, 1);
    }
    __threadfence();  // weight bytes visible GPU-wide before exit: matmuls read weights before their PDL wait
}

// QuantizedTensor.dequantizeRow (:188-213): w = scale * q (INT8) or scale * (raw - zero) (INT4).
__device__ __forceinline__ float dequant_at(const QView& w, int32_t row, int32_t c) {
    const int64_t gi = static_cast<int64_t>(row / w.group_size) * w.columns + c;
    const uint8_t* q = w.q + static_cast<int64_t>(row) * w.bytes_per_row;
    if (w.bits == 8) return __fmul_rn(w.scales[gi], static_cast<float>(static_cast<int8_t>(q[c])));
    const int32_t half = w.bytes_per_row;
    const int32_t byte = q[c < half ? c : c - half];
    const int32_t raw = c < half ? (byte & 0xF) : ((byte >> 4) & 0xF);
    return __fmul_rn(w.scales[gi], static_cast<float>(raw - static_cast<int32_t>(w.zeros[gi])));
}

__global__ void __launch_bounds__(256) dequantize_kernel(QView w, float* __restrict__ out) {
    const int32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= w.columns) return;
    for (int32_t row = blockIdx.y; row < w.rows; row += gridDim.y)
        out[static_cast<int64_t>(row) * w.columns + c] = dequant_at(w, row, c);
}

__global__ void __launch_bounds__(256) dequantize_rows_kernel(QView w, const int32_t* __restrict__ rows,
                                                              int32_t count, float* __restrict__ out,
                                                              int32_t* __restrict__ status) {
    const int32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= w.columns) return;
    for (int32_t i = blockIdx.y; i < count; i += gridDim.y) {
        const int32_t row = rows[i];
        if (row < 0 || row >= w.rows) {
            if (c == 0 && status != nullptr) atomicOr(status, 1);
            continue;
        }
        out[static_cast<int64_t>(i) * w.columns + c] = dequant_at(w, row, c);
    }
}

}  // namespace

cudaError_t launch_quantize(const float* data, int32_t rows, int32_t columns, int32_t bits, int32_t group_size,
                            uint8_t* qdata, float* scales, uint8_t* zeros, int32_t* d_status, cudaStream_t s) {
    const int32_t groups = (rows + group_size - 1) / group_size;
    if (bits == 8) {
        dim3 grid((columns + 255) / 256, groups < 65535 ? groups : 65535);
        quantize_int8_kernel<<<grid, 256, 0, s>>>(data, rows, columns, group_size, qdata, scales, d_status);
    } else {
        const int32_t half = (columns + columns % 2) / 2;
        dim3 grid((half + 255) / 256, groups < 65535 ? groups : 65535);
        quantize_int4_kernel<<<grid, 256, 0, s>>>(data, rows, columns, half, group_size, qdata, scales, zeros,
                                                  d_status);
    }
    return cudaGetLastError();
}

cudaError_t launch_dequantize(const QView& w, float* out, cudaStream_t s) {
    dim3 grid((w.columns + 255) / 256, w.rows < 65535 ? w.rows : 65535);
    dequantize_kernel<<<grid, 256, 0, s>>>(w, out);
    return cudaGetLastError();
}

cudaError_t launch_dequantize_rows(const QView& w, const int32_t* rows, int32_t count, float* out,
                                   int32_t* d_status, cudaStream_t s) {
    if (count == 0) return cudaSuccess;
    dim3 grid((w.columns + 255) / 256, count < 65535 ? count : 65535);
    dequantize_rows_kernel<<<grid, 256, 0, s>>>(w, rows, count, out, d_status);
    return cudaGetLastError();
}

}  // namespace kt
