// kt_shard.cu -- tensor-parallel shards of a device-resident quantized weight.
//
// Quantization is per (group of rows, column), so a block of columns, or a
// block of whole row groups, of a quantized weight is exactly the quantization
// of the same block of the fp32 weight: a shard needs no requantization, only
// the reference layout rebuilt for its shape.  Row shards start on group
// boundaries and are contiguous slices of qdata / scales / zeros.  Column
// shards of an INT8 weight are strided copies; INT4 column shards are
// repacked, because the reference's split-half packing (QuantizedTensor.kt:
// 172-180: column c < half in the low nibble of byte c, column c >= half in the
// high nibble of byte c - half) depends on the shard's own column count.
#include "kt_internal.h"

namespace kt {
namespace {

// The matmul kernels read weights before griddepcontrol.wait (no kernel of a
// matmul chain writes them); a kernel that does write weight bytes makes its
// stores visible GPU-wide before its threads exit, so that a matmul launched
// right after it under programmatic dependent launch reads the new bytes.
__device__ __forceinline__ void weight_writes_visible() { __threadfence(); }

// One thread per output byte of one row of an INT4 column shard.
__global__ void repack_int4_columns_kernel(const uint8_t* __restrict__ src, int32_t src_half, int32_t c0,
                                           int32_t n_dst, int32_t dst_half, int32_t rows, uint8_t* __restrict__ dst) {
    const int64_t total = static_cast<int64_t>(rows) * dst_half;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / dst_half;
        const int32_t b = static_cast<int32_t>(i - r * dst_half);
        const uint8_t* row = src + r * src_half;
        auto nibble = [&](int32_t c) -> uint32_t {  // column c of the source weight
            const uint32_t byte = row[c < src_half ? c : c - src_half];
            return c < src_half ? (byte & 15u) : (byte >> 4);
        };
        const uint32_t lo = nibble(c0 + b);
        const uint32_t hi = dst_half + b < n_dst ? nibble(c0 + dst_half + b) : 0u;  // odd width: pad nibble 0
        dst[r * dst_half + b] = static_cast<uint8_t>(lo | (hi << 4));
    }
    weight_writes_visible();
}

// One thread per output byte of one row of an INT4 weight made of up to
// kMaxConcat column blocks (sources in order).
constexpr int kMaxConcat = 4;
struct ConcatSources {
    const uint8_t* q[kMaxConcat];
    int32_t half[kMaxConcat];    // bytes per row of each source
    int32_t begin[kMaxConcat + 1];  // first destination column of each source; begin[count] = N
    int32_t count;
};

__global__ void concat_int4_columns_kernel(ConcatSources src, int32_t n_dst, int32_t dst_half, int32_t rows,
                                           uint8_t* __restrict__ dst) {
    const int64_t total = static_cast<int64_t>(rows) * dst_half;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / dst_half;
        const int32_t b = static_cast<int32_t>(i - r * dst_half);
        auto nibble = [&](int32_t j) -> uint32_t {  // destination column j
            int p = 0;
            while (p + 1 < src.count && j >= src.begin[p + 1]) ++p;
            const int32_t c = j - src.begin[p], h = src.half[p];
            const uint32_t byte = src.q[p][r * h + (c < h ? c : c - h)];
            return c < h ? (byte & 15u) : (byte >> 4);
        };
        const uint32_t lo = nibble(b);
        const uint32_t hi = dst_half + b < n_dst ? nibble(dst_half + b) : 0u;
        dst[r * dst_half + b] = static_cast<uint8_t>(lo | (hi << 4));
    }
    weight_writes_visible();
}

}  // namespace

cudaError_t launch_concat_int4_columns(const kt_qweight* const* srcs, int32_t count, const kt_qweight* dst,
                                       cudaStream_t s) {
    if (count < 1 || count > kMaxConcat) return cudaErrorInvalidValue;
    ConcatSources cs{};
    cs.count = count;
    int32_t c = 0;
    for (int i = 0; i < count; ++i) {
        cs.q[i] = srcs[i]->qdata;
        cs.half[i] = srcs[i]->bytes_per_row;
        cs.begin[i] = c;
        c += srcs[i]->columns;
    }
    cs.begin[count] = c;
    const int64_t total = static_cast<int64_t>(dst->rows) * dst->bytes_per_row;
    const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 32));
    concat_int4_columns_kernel<<<blocks, 256, 0, s>>>(cs, dst->columns, dst->bytes_per_row, dst->rows, dst->qdata);
    return cudaGetLastError();
}

bool shard_bounds(int32_t axis, int32_t extent, int32_t group_size, int32_t parts, int32_t index, int32_t* begin,
                  int32_t* end) {
    if (parts <= 0 || index < 0 || index >= parts || extent <= 0) return false;
    if (axis == 0) {
        if (group_size <= 0) return false;
        const int64_t groups = (static_cast<int64_t>(extent) + group_size - 1) / group_size;
        const int64_t g0 = index * groups / parts, g1 = (index + 1) * groups / parts;
        *begin = static_cast<int32_t>(std::min<int64_t>(g0 * group_size, extent));
        *end = static_cast<int32_t>(std::min<int64_t>(g1 * group_size, extent));
    } else if (axis == 1) {
        *begin = static_cast<int32_t>(static_cast<int64_t>(index) * extent / parts);
        *end = static_cast<int32_t>(static_cast<int64_t>(index + 1) * extent / parts);
    } else {
        return false;
    }
    return *end > *begin;
}

cudaError_t launch_repack_int4_columns(const kt_qweight* src, int32_t c0, const kt_qweight* dst, cudaStream_t s) {
    const int64_t total = static_cast<int64_t>(dst->rows) * dst->bytes_per_row;
    const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 32));
    repack_int4_columns_kernel<<<blocks, 256, 0, s>>>(src->qdata, src->bytes_per_row, c0, dst->columns,
                                                      dst->bytes_per_row, dst->rows, dst->qdata);
    return cudaGetLastError();
}

}  // namespace kt
