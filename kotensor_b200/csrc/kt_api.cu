// kt_api.cu -- the C ABI (include/kt_cuda.h) over the CUDA runtime: contexts,
// device-resident quantized weights, argument checks with the reference's error
// convention, and dispatch to the kernels.
//
// Argument checks follow the reference's require(...) calls
// (Engine/kotensor/src/main/kotlin/QuantizedTensor.kt:14-17 and :63-70,
// MatMul.kt:470-473, MatMul.kt:963-965): a failed check returns
// KT_ERR_INVALID_ARGUMENT with the reference's message in kt_last_error(),
// m == 0 is a no-op.  No product path falls back to the CPU: every compute call
// launches a CUDA kernel or fails.
#include <cstdio>
#include <algorithm>
#include <cstring>
#include <new>
#include <string>

#include "kt_internal.h"

#define KT_VERSION 1

namespace kt {
namespace {
thread_local std::string g_last_error;

kt_status fail(kt_status st, const std::string& msg) {
    g_last_error = msg;
    return st;
}

kt_status cuda_fail(cudaError_t e, const char* what) {
    return fail(e == cudaErrorMemoryAllocation ? KT_ERR_OUT_OF_MEMORY : KT_ERR_CUDA,
                std::string(what) + ": " + cudaGetErrorString(e));
}

#define KT_CUDA_TRY(expr, what)                       \
    do {                                              \
        cudaError_t e__ = (expr);                     \
        if (e__ != cudaSuccess) return cuda_fail(e__, what); \
    } while (0)

int32_t groups_of(int32_t rows, int32_t g) { return (rows + g - 1) / g; }
int32_t bytes_per_row_of(int32_t bits, int32_t columns) { return bits == 4 ? (columns + columns % 2) / 2 : columns; }

kt_status check_quant(int32_t bits, int32_t group_size) {
    if (bits != 4 && bits != 8) return fail(KT_ERR_INVALID_ARGUMENT, "bits must be 4 or 8, got " + std::to_string(bits));
    if (group_size <= 0) return fail(KT_ERR_INVALID_ARGUMENT, "groupSize must be positive");
    return KT_OK;
}

kt_status check_shape(int32_t rows, int32_t columns) {
    if (rows <= 0 || columns <= 0)
        return fail(KT_ERR_INVALID_ARGUMENT, "QuantizedTensor needs a 2-D shape, got [" + std::to_string(rows) + ", " +
                                                 std::to_string(columns) + "]");
    // Byte offsets are 64-bit everywhere; element counts of one row / one scale
    // row must stay addressable with 32-bit column indices.
    return KT_OK;
}

// A NULL stream is CUDA's default stream, as everywhere in the CUDA runtime;
// the context's own stream is reachable through kt_ctx_stream().
cudaStream_t pick(kt_ctx* ctx, void* stream) {
    (void)ctx;
    return static_cast<cudaStream_t>(stream);
}

// Allocates an empty device weight with the reference's size bookkeeping.
kt_status alloc_weight(kt_ctx* ctx, int32_t bits, int32_t group_size, int32_t rows, int32_t columns,
                       kt_qweight** out) {
    auto* w = new (std::nothrow) kt_qweight();
    if (!w) return fail(KT_ERR_OUT_OF_MEMORY, "host allocation failed");
    w->ctx = ctx;
    w->bits = bits;
    w->group_size = group_size;
    w->rows = rows;
    w->columns = columns;
    w->groups = groups_of(rows, group_size);
    w->bytes_per_row = bytes_per_row_of(bits, columns);
    w->stored_columns = bits == 4 ? columns + columns % 2 : columns;
    const size_t qbytes = static_cast<size_t>(rows) * w->bytes_per_row;
    const size_t gcols = static_cast<size_t>(w->groups) * columns;
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e == cudaSuccess) e = cudaMalloc(&w->qdata, qbytes);
    if (e == cudaSuccess) e = cudaMalloc(&w->scales, gcols * sizeof(float));
    if (e == cudaSuccess && bits == 4) e = cudaMalloc(&w->zeros, gcols);
    if (e != cudaSuccess) {
        cudaFree(w->qdata);
        cudaFree(w->scales);
        cudaFree(w->zeros);
        delete w;
        return cuda_fail(e, "cudaMalloc(quantized weight)");
    }
    make_tensor_maps(w);  // absent maps only disable the TMA streaming kernel
    *out = w;
    return KT_OK;
}

void free_weight(kt_qweight* w) {
    if (!w) return;
    cudaSetDevice(w->ctx->device);
    cudaFree(w->qdata);
    cudaFree(w->scales);
    cudaFree(w->zeros);
    delete w;
}

}  // namespace

cudaError_t stream_workspace(kt_ctx* ctx, cudaStream_t s, size_t bytes, void** out) {
    std::lock_guard<std::mutex> lock(ctx->ws_mutex);
    kt_ctx::Workspace* hit = nullptr;
    for (auto& ws : ctx->workspaces)
        if (ws.stream == s) hit = &ws;
    if (hit != nullptr && hit->bytes >= bytes) {
        *out = hit->ptr;
        return cudaSuccess;
    }
    // Grow to at least 1 MiB at a time.  cudaMalloc is not a stream operation;
    // while `s` is being captured into a CUDA graph it is allowed in relaxed
    // capture mode, and the zeroing below then becomes a node of that graph.
    const size_t cap = std::max(bytes, static_cast<size_t>(1) << 20);
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    cudaThreadExchangeStreamCaptureMode(&mode);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, cap);
    cudaThreadExchangeStreamCaptureMode(&mode);
    if (e != cudaSuccess) return e;
    e = cudaMemsetAsync(p, 0, cap, s);
    if (e != cudaSuccess) {
        cudaFree(p);
        return e;
    }
    if (hit != nullptr) {
        ctx->retired.push_back(hit->ptr);  // queued launches may still use it
        hit->ptr = p;
        hit->bytes = cap;
    } else {
        ctx->workspaces.push_back({s, p, cap});
    }
    *out = p;
    return cudaSuccess;
}

namespace {

kt_status grow(float** buf, size_t* cap, size_t need) {
    if (*cap >= need) return KT_OK;
    cudaFree(*buf);
    *buf = nullptr;
    *cap = 0;
    cudaError_t e = cudaMalloc(buf, need * sizeof(float));
    if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc(staging)");
    *cap = need;
    return KT_OK;
}

kt_status run_matmul(kt_ctx* ctx, const kt_qweight* w, const float* a, float* c, int32_t m, int32_t accumulate,
                     float alpha, const float* bias, cudaStream_t s, const LoraEpilogue* lora = nullptr) {
    const QView v = view(w);
    MatmulArgs args{a, c, bias, m, accumulate, alpha, ctx->d_error};
    if (lora) args.lora = *lora;
    cudaError_t e;
    if (gemv_imma_supported(v, m, a)) {
        const size_t need = gemv_imma_workspace_bytes(v, ctx->sm_count);
        void* ws = nullptr;
        if (need > 0) {
            e = stream_workspace(ctx, s, need, &ws);
            if (e != cudaSuccess) return cuda_fail(e, "qmatmul workspace");
        }
        e = launch_gemv_imma(v, args, ctx->sm_count, s, ws, need);
    } else if (gemv_mma_supported(v, m, a)) {
        const size_t need = gemv_mma_workspace_bytes(v, m, ctx->sm_count);
        void* ws = nullptr;
        if (need > 0) {
            e = stream_workspace(ctx, s, need, &ws);
            if (e != cudaSuccess) return cuda_fail(e, "qmatmul workspace");
        }
        e = launch_gemv_mma(v, args, ctx->sm_count, s, ws, need);
    } else if (gemv_fast_supported(v, m, a)) {
        e = launch_gemv(v, args, ctx->sm_count, s);
    } else if (gemm_tc_supported(v, m, a)) {
        void* ws = nullptr;
        const size_t need = gemm_tc_workspace_bytes(v, m, ctx->sm_count);
        e = stream_workspace(ctx, s, need, &ws);
        if (e != cudaSuccess) return cuda_fail(e, "qmatmul workspace");
        e = launch_gemm_tc(v, args, ctx->sm_count, s, ws, need);
    } else {
        e = launch_matmul_generic(v, args, s);
    }
    if (e != cudaSuccess) return cuda_fail(e, "qmatmul launch");
    return KT_OK;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on libcuda).
EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = []() -> EncodeTiledFn {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return nullptr;
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }

// qdata as a 2-D u8 tensor {bytes_per_row (inner), rows}, boxes of
// kStageRows rows x 128 / 256 bytes, out-of-range boxes zero-filled.  TMA
// needs 16-byte aligned rows, so weights with bytes_per_row % 16 != 0 get none.
bool make_tensor_maps(kt_qweight* w) {
    w->has_tmaps = false;
    if (w->bytes_per_row % 16 != 0) return false;
    EncodeTiledFn encode = encode_tiled();
    if (!encode) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(w->bytes_per_row), static_cast<cuuint64_t>(w->rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(w->bytes_per_row)};
    const cuuint32_t estr[2] = {1, 1};
    const cuuint32_t box128[2] = {128, kStageRows};
    const cuuint32_t box256[2] = {256, kStageRows};
    if (encode(&w->tmap_w128, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w->qdata, dims, strides, box128, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    if (encode(&w->tmap_w256, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w->qdata, dims, strides, box256, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    w->has_tmaps = true;
    if (w->bytes_per_row >= 128) {
        const cuuint32_t box_mma[2] = {128, 32};
        w->has_tmap_mma =
            encode(&w->tmap_mma, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w->qdata, dims, strides, box_mma, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        const cuuint32_t box_raw[2] = {128, 64};
        w->has_tmap_raw64 =
            encode(&w->tmap_raw64, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w->qdata, dims, strides, box_raw, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    return true;
}

bool encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType type, uint32_t elem_bytes, const void* base,
                    uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapSwizzle swizzle) {
    (void)elem_bytes;
    EncodeTiledFn encode = encode_tiled();
    if (!encode) return false;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return encode(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

kt_status run_qmatmul(kt_ctx* ctx, const kt_qweight* w, const float* a, float* c, int32_t m, int32_t accumulate,
                      float alpha, const float* bias, cudaStream_t s, const LoraEpilogue* lora) {
    return run_matmul(ctx, w, a, c, m, accumulate, alpha, bias, s, lora);
}

}  // namespace kt

using namespace kt;

extern "C" {

int32_t kt_version(void) { return KT_VERSION; }

const char* kt_last_error(void) { return g_last_error.c_str(); }

kt_status kt_check_quantization(int32_t bits, int32_t group_size) { return check_quant(bits, group_size); }

kt_status kt_init(int32_t device, kt_ctx** out) {
    if (!out) return fail(KT_ERR_INVALID_ARGUMENT, "out is NULL");
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= count)
        return fail(KT_ERR_INVALID_ARGUMENT, "device " + std::to_string(device) + " out of range (" +
                                                 std::to_string(count) + " devices)");
    auto* ctx = new (std::nothrow) kt_ctx();
    if (!ctx) return fail(KT_ERR_OUT_OF_MEMORY, "host allocation failed");
    ctx->device = device;
    e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
    if (e == cudaSuccess)
        e = cudaDeviceGetAttribute(&ctx->max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&ctx->d_status, 2 * sizeof(int32_t));
    if (e == cudaSuccess) e = cudaMemset(ctx->d_status, 0, 2 * sizeof(int32_t));
    if (e == cudaSuccess) ctx->d_error = ctx->d_status + 1;
    if (e != cudaSuccess) {
        if (ctx->stream) cudaStreamDestroy(ctx->stream);
        cudaFree(ctx->d_status);
        delete ctx;
        return cuda_fail(e, "kt_init");
    }
    *out = ctx;
    return KT_OK;
}

kt_status kt_destroy(kt_ctx* ctx) {
    if (!ctx) return KT_OK;
    cudaSetDevice(ctx->device);
    cudaDeviceSynchronize();  // workspaces may be in use on any stream
    for (auto& ws : ctx->workspaces) cudaFree(ws.ptr);
    for (void* p : ctx->retired) cudaFree(p);
    cudaFree(ctx->h2d_a);
    cudaFree(ctx->d2h_c);
    cudaFree(ctx->bias_buf);
    cudaFree(ctx->d_status);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return KT_OK;
}

kt_status kt_ctx_stream(kt_ctx* ctx, void** stream_out) {
    if (!ctx || !stream_out) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    *stream_out = ctx->stream;
    return KT_OK;
}

kt_status kt_alloc(kt_ctx* ctx, size_t bytes, void** out) {
    if (!ctx || !out) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    KT_CUDA_TRY(cudaSetDevice(ctx->device), "cudaSetDevice");
    KT_CUDA_TRY(cudaMalloc(out, bytes), "cudaMalloc");
    return KT_OK;
}

kt_status kt_free(kt_ctx* ctx, void* ptr) {
    if (!ctx) return fail(KT_ERR_INVALID_ARGUMENT, "NULL context");
    KT_CUDA_TRY(cudaSetDevice(ctx->device), "cudaSetDevice");
    KT_CUDA_TRY(cudaFree(ptr), "cudaFree");
    return KT_OK;
}

kt_status kt_memcpy_h2d(kt_ctx* ctx, void* dst, const void* src, size_t bytes, void* stream) {
    if (!ctx) return fail(KT_ERR_INVALID_ARGUMENT, "NULL context");
    KT_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, pick(ctx, stream)), "cudaMemcpyAsync(H2D)");
    return KT_OK;
}

kt_status kt_memcpy_d2h(kt_ctx* ctx, void* dst, const void* src, size_t bytes, void* stream) {
    if (!ctx) return fail(KT_ERR_INVALID_ARGUMENT, "NULL context");
    KT_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, pick(ctx, stream)), "cudaMemcpyAsync(D2H)");
    return KT_OK;
}

kt_status kt_stream_sync(kt_ctx* ctx, void* stream) {
    if (!ctx) return fail(KT_ERR_INVALID_ARGUMENT, "NULL context");
    KT_CUDA_TRY(cudaStreamSynchronize(pick(ctx, stream)), "cudaStreamSynchronize");
    return KT_OK;
}

kt_status kt_qweight_upload(kt_ctx* ctx, int32_t bits, int32_t group_size, int32_t rows, int32_t columns,
                            const void* qdata, const float* scales, const uint8_t* zeros, kt_qweight** out) {
    if (!ctx || !out || !qdata || !scales) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    kt_status st = check_quant(bits, group_size);
    if (st != KT_OK) return st;
    if ((st = check_shape(rows, columns)) != KT_OK) return st;
    if (bits == 4 && !zeros) return fail(KT_ERR_INVALID_ARGUMENT, "4-bit tensors need zero points");
    if (bits == 8 && zeros) return fail(KT_ERR_INVALID_ARGUMENT, "8-bit tensors have no zero points");
    kt_qweight* w = nullptr;
    if ((st = alloc_weight(ctx, bits, group_size, rows, columns, &w)) != KT_OK) return st;
    const size_t qbytes = static_cast<size_t>(rows) * w->bytes_per_row;
    const size_t gcols = static_cast<size_t>(w->groups) * columns;
    cudaError_t e = cudaMemcpy(w->qdata, qdata, qbytes, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(w->scales, scales, gcols * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess && bits == 4) e = cudaMemcpy(w->zeros, zeros, gcols, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        free_weight(w);
        return cuda_fail(e, "kt_qweight_upload");
    }
    *out = w;
    return KT_OK;
}

kt_status kt_qweight_from_device(kt_ctx* ctx, int32_t bits, int32_t group_size, int32_t rows, int32_t columns,
                                 const void* qdata, const float* scales, const uint8_t* zeros, void* stream,
                                 kt_qweight** out) {
    if (!ctx || !out || !qdata || !scales) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    kt_status st = check_quant(bits, group_size);
    if (st != KT_OK) return st;
    if ((st = check_shape(rows, columns)) != KT_OK) return st;
    if (bits == 4 && !zeros) return fail(KT_ERR_INVALID_ARGUMENT, "4-bit tensors need zero points");
    kt_qweight* w = nullptr;
    if ((st = alloc_weight(ctx, bits, group_size, rows, columns, &w)) != KT_OK) return st;
    cudaStream_t s = pick(ctx, stream);
    const size_t qbytes = static_cast<size_t>(rows) * w->bytes_per_row;
    const size_t gcols = static_cast<size_t>(w->groups) * columns;
    cudaError_t e = cudaMemcpyAsync(w->qdata, qdata, qbytes, cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(w->scales, scales, gcols * sizeof(float), cudaMemcpyDeviceToDevice, s);
    if (e == cudaSuccess && bits == 4) e = cudaMemcpyAsync(w->zeros, zeros, gcols, cudaMemcpyDeviceToDevice, s);
    if (e != cudaSuccess) {
        free_weight(w);
        return cuda_fail(e, "kt_qweight_from_device");
    }
    *out = w;
    return KT_OK;
}

kt_status kt_quantize(kt_ctx* ctx, int32_t bits, int32_t group_size, int32_t rows, int32_t columns,
                      const float* data, void* stream, kt_qweight** out) {
    if (!ctx || !out || !data) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    kt_status st = check_quant(bits, group_size);
    if (st != KT_OK) return st;
    if ((st = check_shape(rows, columns)) != KT_OK) return st;
    kt_qweight* w = nullptr;
    if ((st = alloc_weight(ctx, bits, group_size, rows, columns, &w)) != KT_OK) return st;
    cudaStream_t s = pick(ctx, stream);
    int32_t status = 0;
    cudaError_t e = cudaMemsetAsync(ctx->d_status, 0, sizeof(int32_t), s);
    if (e == cudaSuccess)
        e = launch_quantize(data, rows, columns, bits, group_size, w->qdata, w->scales, w->zeros, ctx->d_status, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&status, ctx->d_status, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) {
        free_weight(w);
        return cuda_fail(e, "kt_quantize");
    }
    if (status != 0) {
        free_weight(w);
        return fail(KT_ERR_NAN, "Cannot round NaN value.");
    }
    *out = w;
    return KT_OK;
}

kt_status kt_qweight_info_get(const kt_qweight* w, kt_qweight_info* out) {
    if (!w || !out) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    out->bits = w->bits;
    out->group_size = w->group_size;
    out->rows = w->rows;
    out->columns = w->columns;
    out->groups = w->groups;
    out->bytes_per_row = w->bytes_per_row;
    out->stored_columns = w->stored_columns;
    out->size_in_bytes = static_cast<int64_t>(w->rows) * w->bytes_per_row +
                         static_cast<int64_t>(w->groups) * w->columns * 4 +
                         (w->bits == 4 ? static_cast<int64_t>(w->groups) * w->columns : 0);
    out->qdata = w->qdata;
    out->scales = w->scales;
    out->zeros = w->zeros;
    return KT_OK;
}

kt_status kt_qweight_download(const kt_qweight* w, void* qdata, float* scales, uint8_t* zeros) {
    if (!w || !qdata || !scales) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (w->bits == 4 && !zeros) return fail(KT_ERR_INVALID_ARGUMENT, "4-bit tensors need a zeros buffer");
    KT_CUDA_TRY(cudaSetDevice(w->ctx->device), "cudaSetDevice");
    // The weight may have been written on any stream (kt_quantize, kt_qweight_from_device).
    KT_CUDA_TRY(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    const size_t qbytes = static_cast<size_t>(w->rows) * w->bytes_per_row;
    const size_t gcols = static_cast<size_t>(w->groups) * w->columns;
    KT_CUDA_TRY(cudaMemcpy(qdata, w->qdata, qbytes, cudaMemcpyDeviceToHost), "download qdata");
    KT_CUDA_TRY(cudaMemcpy(scales, w->scales, gcols * sizeof(float), cudaMemcpyDeviceToHost), "download scales");
    if (w->bits == 4) KT_CUDA_TRY(cudaMemcpy(zeros, w->zeros, gcols, cudaMemcpyDeviceToHost), "download zeros");
    return KT_OK;
}

kt_status kt_qweight_free(kt_qweight* w) {
    free_weight(w);
    return KT_OK;
}

kt_status kt_qweight_concat_columns(kt_ctx* ctx, const kt_qweight* const* ws, int32_t count, void* stream,
                                    kt_qweight** out) {
    if (!ctx || !ws || !out || count < 1 || count > 4) return fail(KT_ERR_INVALID_ARGUMENT, "1 to 4 weights");
    *out = nullptr;
    int64_t n = 0;
    for (int i = 0; i < count; ++i) {
        if (!ws[i]) return fail(KT_ERR_INVALID_ARGUMENT, "NULL weight");
        if (ws[i]->bits != ws[0]->bits || ws[i]->group_size != ws[0]->group_size || ws[i]->rows != ws[0]->rows)
            return fail(KT_ERR_INVALID_ARGUMENT, "weights differ in bits, group size or rows");
        n += ws[i]->columns;
    }
    if (n > INT32_MAX) return fail(KT_ERR_INVALID_ARGUMENT, "too many columns");
    kt_qweight* d = nullptr;
    kt_status st = alloc_weight(ctx, ws[0]->bits, ws[0]->group_size, ws[0]->rows, static_cast<int32_t>(n), &d);
    if (st != KT_OK) return st;
    cudaStream_t s = pick(ctx, stream);
    cudaError_t err = cudaSuccess;
    if (d->bits == 4) err = launch_concat_int4_columns(ws, count, d, s);
    size_t c0 = 0;
    for (int i = 0; i < count && err == cudaSuccess; ++i) {
        const kt_qweight* w = ws[i];
        const size_t nc = static_cast<size_t>(w->columns);
        if (d->bits == 8)
            err = cudaMemcpy2DAsync(d->qdata + c0, d->bytes_per_row, w->qdata, w->bytes_per_row, nc, w->rows,
                                    cudaMemcpyDeviceToDevice, s);
        if (err == cudaSuccess)
            err = cudaMemcpy2DAsync(d->scales + c0, d->columns * sizeof(float), w->scales, nc * sizeof(float),
                                    nc * sizeof(float), w->groups, cudaMemcpyDeviceToDevice, s);
        if (err == cudaSuccess && d->bits == 4)
            err = cudaMemcpy2DAsync(d->zeros + c0, d->columns, w->zeros, nc, nc, w->groups, cudaMemcpyDeviceToDevice, s);
        c0 += nc;
    }
    if (err != cudaSuccess) {
        free_weight(d);
        return cuda_fail(err, "kt_qweight_concat_columns");
    }
    *out = d;
    return KT_OK;
}

kt_status kt_shard_bounds(int32_t axis, int32_t extent, int32_t group_size, int32_t parts, int32_t index,
                          int32_t* begin, int32_t* end) {
    if (!begin || !end) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (!shard_bounds(axis, extent, group_size, parts, index, begin, end))
        return fail(KT_ERR_INVALID_ARGUMENT, "no shard " + std::to_string(index) + " of " + std::to_string(parts) +
                                                 " along axis " + std::to_string(axis) + " of extent " +
                                                 std::to_string(extent));
    return KT_OK;
}

kt_status kt_qweight_slice(kt_ctx* ctx, const kt_qweight* w, int32_t axis, int32_t b, int32_t e, void* stream,
                           kt_qweight** out) {
    if (!ctx || !w || !out) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    if (axis != 0 && axis != 1) return fail(KT_ERR_INVALID_ARGUMENT, "axis must be 0 (rows) or 1 (columns)");
    const int32_t extent = axis == 0 ? w->rows : w->columns;
    if (b < 0 || e > extent || e <= b)
        return fail(KT_ERR_INVALID_ARGUMENT, "slice [" + std::to_string(b) + ", " + std::to_string(e) +
                                                 ") outside [0, " + std::to_string(extent) + ")");
    if (axis == 0 && (b % w->group_size != 0 || (e % w->group_size != 0 && e != w->rows)))
        return fail(KT_ERR_INVALID_ARGUMENT, "a row slice must start and end on group boundaries");
    kt_qweight* d = nullptr;
    kt_status st = alloc_weight(ctx, w->bits, w->group_size, axis == 0 ? e - b : w->rows,
                                axis == 0 ? w->columns : e - b, &d);
    if (st != KT_OK) return st;
    cudaStream_t s = pick(ctx, stream);
    cudaError_t err = cudaSuccess;
    if (axis == 0) {
        // whole groups: contiguous slices of every array
        const int32_t g0 = b / w->group_size;
        const size_t gcols = static_cast<size_t>(d->groups) * w->columns;
        err = cudaMemcpyAsync(d->qdata, w->qdata + static_cast<size_t>(b) * w->bytes_per_row,
                              static_cast<size_t>(d->rows) * d->bytes_per_row, cudaMemcpyDeviceToDevice, s);
        if (err == cudaSuccess)
            err = cudaMemcpyAsync(d->scales, w->scales + static_cast<size_t>(g0) * w->columns, gcols * sizeof(float),
                                  cudaMemcpyDeviceToDevice, s);
        if (err == cudaSuccess && w->bits == 4)
            err = cudaMemcpyAsync(d->zeros, w->zeros + static_cast<size_t>(g0) * w->columns, gcols,
                                  cudaMemcpyDeviceToDevice, s);
    } else {
        const size_t n = static_cast<size_t>(e - b);
        if (w->bits == 8)
            err = cudaMemcpy2DAsync(d->qdata, n, w->qdata + b, w->bytes_per_row, n, w->rows, cudaMemcpyDeviceToDevice, s);
        else
            err = launch_repack_int4_columns(w, b, d, s);
        if (err == cudaSuccess)
            err = cudaMemcpy2DAsync(d->scales, n * sizeof(float), w->scales + b, w->columns * sizeof(float),
                                    n * sizeof(float), w->groups, cudaMemcpyDeviceToDevice, s);
        if (err == cudaSuccess && w->bits == 4)
            err = cudaMemcpy2DAsync(d->zeros, n, w->zeros + b, w->columns, n, w->groups, cudaMemcpyDeviceToDevice, s);
    }
    if (err != cudaSuccess) {
        free_weight(d);
        return cuda_fail(err, "kt_qweight_slice");
    }
    *out = d;
    return KT_OK;
}

kt_status kt_qweight_shard(kt_ctx* ctx, const kt_qweight* w, int32_t axis, int32_t parts, int32_t index,
                           void* stream, kt_qweight** out) {
    if (!ctx || !w || !out) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    int32_t b = 0, e = 0;
    const int32_t extent = axis == 0 ? w->rows : w->columns;
    kt_status st = kt_shard_bounds(axis, extent, w->group_size, parts, index, &b, &e);
    if (st != KT_OK) return st;
    return kt_qweight_slice(ctx, w, axis, b, e, stream, out);
}

kt_status kt_qweight_load(kt_ctx* ctx, kt_stfile* f, const char* name, int32_t bits, int32_t group_size,
                          int32_t rows, int32_t columns, void* stream, kt_qweight** out) {
    if (!ctx || !f || !name || !out) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    kt_status st = check_quant(bits, group_size);
    if (st != KT_OK) return st;
    if ((st = check_shape(rows, columns)) != KT_OK) return st;
    // QuantizedTensor.mapFrom's checks (QuantizedTensor.kt:109-116), with its messages
    const std::string base(name);
    const int64_t groups = groups_of(rows, group_size);
    const int64_t qbytes = static_cast<int64_t>(rows) * bytes_per_row_of(bits, columns);
    const int64_t gcols = groups * columns;
    kt_st_entry_info qi{}, si{}, zi{};
    if ((st = kt_st_entry(f, (base + ".qweight").c_str(), &qi)) != KT_OK) return st;
    if (qi.bytes != qbytes)
        return fail(KT_ERR_INVALID_ARGUMENT, base + ".qweight has " + std::to_string(qi.bytes) + " bytes, expected " +
                                                 std::to_string(qbytes));
    if ((st = kt_st_entry(f, (base + ".scales").c_str(), &si)) != KT_OK) return st;
    if (std::strcmp(si.dtype, "F32") != 0 || si.bytes != gcols * 4)
        return fail(KT_ERR_INVALID_ARGUMENT, base + ".scales is " + si.dtype + " with " + std::to_string(si.bytes) +
                                                 " bytes, expected F32 with " + std::to_string(gcols * 4));
    if (bits == 4) {
        if ((st = kt_st_entry(f, (base + ".zeros").c_str(), &zi)) != KT_OK) return st;
        if (zi.bytes != gcols)
            return fail(KT_ERR_INVALID_ARGUMENT, base + ".zeros has " + std::to_string(zi.bytes) + " bytes, expected " +
                                                     std::to_string(gcols));
    }
    kt_qweight* w = nullptr;
    if ((st = alloc_weight(ctx, bits, group_size, rows, columns, &w)) != KT_OK) return st;
    st = kt_st_read_raw_device(ctx, f, (base + ".qweight").c_str(), w->qdata, qbytes, stream);
    if (st == KT_OK) st = kt_st_read_raw_device(ctx, f, (base + ".scales").c_str(), w->scales, gcols * 4, stream);
    if (st == KT_OK && bits == 4) st = kt_st_read_raw_device(ctx, f, (base + ".zeros").c_str(), w->zeros, gcols, stream);
    if (st != KT_OK) {
        // copies already queued read the staging buffers into this weight: let them finish first
        cudaStreamSynchronize(pick(ctx, stream));
        free_weight(w);
        return st;
    }
    *out = w;
    return KT_OK;
}

kt_status kt_dequantize(kt_ctx* ctx, const kt_qweight* w, float* out, void* stream) {
    if (!ctx || !w || !out) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    KT_CUDA_TRY(launch_dequantize(view(w), out, pick(ctx, stream)), "dequantize launch");
    return KT_OK;
}

kt_status kt_dequantize_rows(kt_ctx* ctx, const kt_qweight* w, const int32_t* rows, int32_t count, float* out,
                             int32_t* status, void* stream) {
    if (!ctx || !w) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (count < 0) return fail(KT_ERR_INVALID_ARGUMENT, "negative row count " + std::to_string(count));
    if (count == 0) return KT_OK;
    if (!rows || !out) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    KT_CUDA_TRY(launch_dequantize_rows(view(w), rows, count, out, status, pick(ctx, stream)), "dequantize_rows launch");
    return KT_OK;
}

kt_status kt_qmatmul(kt_ctx* ctx, const kt_qweight* w, const float* a, float* c, int32_t m, int32_t accumulate,
                     float alpha, const float* bias, void* stream) {
    if (!ctx || !w) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (m < 0) return fail(KT_ERR_INVALID_ARGUMENT, "Negative row count " + std::to_string(m));
    if (m == 0) return KT_OK;
    if (!a || !c) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    return run_matmul(ctx, w, a, c, m, accumulate, alpha, bias, pick(ctx, stream));
}

kt_status kt_qmatmul_path(const kt_qweight* w, int32_t m, int32_t* path_out) {
    if (!w || !path_out) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (m < 0) return fail(KT_ERR_INVALID_ARGUMENT, "Negative row count " + std::to_string(m));
    const QView v = view(w);
    const bool mma_rows = gemv_mma_supported(v, m, nullptr);
    *path_out = gemv_imma_supported(v, m, nullptr) || mma_rows ? KT_PATH_GEMV_MMA
                : gemv_fast_supported(v, m, nullptr) ? KT_PATH_GEMV
                : gemm_tc_supported(v, m, nullptr)   ? KT_PATH_TENSOR_CORE
                                                     : KT_PATH_GENERIC;
    return KT_OK;
}

kt_status kt_set_gemv_tuning(int32_t lane_bytes, int32_t cluster_k) {
    set_gemv_tuning(lane_bytes, cluster_k);
    return KT_OK;
}

kt_status kt_qmatmul_t_path(const kt_qweight* w, int32_t m, int32_t* path_out) {
    if (!w || !path_out) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (m < 0) return fail(KT_ERR_INVALID_ARGUMENT, "Negative row count " + std::to_string(m));
    *path_out = gemm_t_supported(view(w), m, nullptr) ? KT_PATH_TENSOR_CORE : KT_PATH_GENERIC;
    return KT_OK;
}

kt_status kt_set_gemv_mma_tuning(int32_t k_splits) {
    set_mma_tuning(k_splits);
    set_imma_tuning(k_splits);
    return KT_OK;
}

kt_status kt_ctx_take_error(kt_ctx* ctx, int32_t* error_out) {
    if (!ctx || !error_out) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    KT_CUDA_TRY(cudaSetDevice(ctx->device), "cudaSetDevice");
    KT_CUDA_TRY(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    KT_CUDA_TRY(cudaMemcpy(error_out, ctx->d_error, sizeof(int32_t), cudaMemcpyDeviceToHost), "read error word");
    KT_CUDA_TRY(cudaMemset(ctx->d_error, 0, sizeof(int32_t)), "clear error word");
    return KT_OK;
}

kt_status kt_qmatmul_host(kt_ctx* ctx, const kt_qweight* w, const float* a, float* c, int32_t m, int32_t accumulate,
                          float alpha, const float* bias) {
    if (!ctx || !w) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (m < 0) return fail(KT_ERR_INVALID_ARGUMENT, "Negative row count " + std::to_string(m));
    if (m == 0) return KT_OK;
    if (!a || !c) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    std::lock_guard<std::mutex> lock(ctx->host_mutex);
    KT_CUDA_TRY(cudaSetDevice(ctx->device), "cudaSetDevice");
    const size_t an = static_cast<size_t>(m) * w->rows, cn = static_cast<size_t>(m) * w->columns;
    kt_status st;
    if ((st = grow(&ctx->h2d_a, &ctx->a_cap, an)) != KT_OK) return st;
    if ((st = grow(&ctx->d2h_c, &ctx->c_cap, cn)) != KT_OK) return st;
    if (bias && (st = grow(&ctx->bias_buf, &ctx->bias_cap, w->columns)) != KT_OK) return st;
    cudaStream_t s = ctx->stream;
    // c in page-locked host memory (cudaHostAlloc / cudaHostRegister, mapped into
    // the device's address space): the kernel writes it directly over the bus
    // (posted writes, no device-to-host copy); otherwise through device staging.
    // a is always staged: every column tile of the product reads it.
    cudaPointerAttributes pa{};
    float* c_dev = ctx->d2h_c;
    if (cudaPointerGetAttributes(&pa, c) == cudaSuccess && pa.type == cudaMemoryTypeHost && pa.devicePointer != nullptr)
        c_dev = static_cast<float*>(pa.devicePointer);
    cudaGetLastError();  // a pageable pointer is not an error here
    KT_CUDA_TRY(cudaMemcpyAsync(ctx->h2d_a, a, an * sizeof(float), cudaMemcpyHostToDevice, s), "H2D a");
    if (accumulate && c_dev == ctx->d2h_c)
        KT_CUDA_TRY(cudaMemcpyAsync(ctx->d2h_c, c, cn * sizeof(float), cudaMemcpyHostToDevice, s), "H2D c");
    if (bias)
        KT_CUDA_TRY(cudaMemcpyAsync(ctx->bias_buf, bias, w->columns * sizeof(float), cudaMemcpyHostToDevice, s),
                    "H2D bias");
    if ((st = run_matmul(ctx, w, ctx->h2d_a, c_dev, m, accumulate, alpha, bias ? ctx->bias_buf : nullptr, s)) != KT_OK)
        return st;
    if (c_dev == ctx->d2h_c)
        KT_CUDA_TRY(cudaMemcpyAsync(c, ctx->d2h_c, cn * sizeof(float), cudaMemcpyDeviceToHost, s), "D2H c");
    KT_CUDA_TRY(cudaStreamSynchronize(s), "cudaStreamSynchronize");
    return KT_OK;
}

kt_status kt_qmatmul_t(kt_ctx* ctx, const kt_qweight* w, const float* dy, float* dx, int32_t m, int32_t accumulate,
                       void* stream) {
    if (!ctx || !w) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (m < 0) return fail(KT_ERR_INVALID_ARGUMENT, "Negative row count " + std::to_string(m));
    if (m == 0) return KT_OK;
    if (!dy || !dx) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    const QView v = view(w);
    const cudaStream_t s = pick(ctx, stream);
    if (gemm_t_supported(v, m, dy)) {  // m >= 16: bf16 tensor cores (tolerance 2e-2)
        const size_t need = gemm_t_workspace_bytes(v, m, ctx->sm_count);
        void* ws = nullptr;
        KT_CUDA_TRY(stream_workspace(ctx, s, need, &ws), "qmatmul_t workspace");
        KT_CUDA_TRY(launch_gemm_t(v, dy, dx, m, accumulate, ctx->d_error, ctx->sm_count, s, ws, need),
                    "qmatmul_t launch");
        return KT_OK;
    }
    const size_t need = matmul_t_workspace_bytes(v, m);
    void* ws = nullptr;
    if (need > 0) KT_CUDA_TRY(stream_workspace(ctx, s, need, &ws), "qmatmul_t workspace");
    KT_CUDA_TRY(launch_matmul_t(v, dy, dx, m, accumulate, s, ws, need), "qmatmul_t launch");
    return KT_OK;
}

// ---- LoRALinear over a quantized base (kt_lora.cu)

namespace {
kt_status check_lora(int32_t m, int32_t k, int32_t rank, const float* lora_a) {
    if (m < 0) return fail(KT_ERR_INVALID_ARGUMENT, "Negative row count " + std::to_string(m));
    if (k <= 0) return fail(KT_ERR_INVALID_ARGUMENT, "in-features must be positive");
    if (rank < 1 || rank > kLoraMaxRank)
        return fail(KT_ERR_INVALID_ARGUMENT, "LoRA rank must be in 1.." + std::to_string(kLoraMaxRank) + ", got " +
                                                 std::to_string(rank));
    if (!lora_a) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    return KT_OK;
}
}  // namespace

kt_status kt_lora_project(kt_ctx* ctx, const float* a, int32_t m, int32_t k, const float* lora_a, int32_t rank,
                          float* projected, void* stream) {
    if (!ctx) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    kt_status st = check_lora(m, k, rank, lora_a);
    if (st != KT_OK || m == 0) return st;
    if (!a || !projected) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    const cudaStream_t s = pick(ctx, stream);
    void* ws = nullptr;
    KT_CUDA_TRY(stream_workspace(ctx, s, lora_workspace_bytes(m, k, 1, rank), &ws), "lora workspace");
    KT_CUDA_TRY(launch_lora_project(a, m, k, lora_a, rank, projected, ws, s), "lora project launch");
    return KT_OK;
}

kt_status kt_lora_qmatmul(kt_ctx* ctx, const kt_qweight* w, const float* a, float* c, int32_t m, int32_t accumulate,
                          float alpha, const float* bias, const float* lora_a, const float* lora_b, int32_t rank,
                          float scaling, float* projected, void* stream) {
    if (!ctx || !w) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    kt_status st = check_lora(m, w->rows, rank, lora_a);
    if (st != KT_OK || m == 0) return st;
    if (!a || !c || !lora_b || !projected) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if ((st = kt_lora_project(ctx, a, m, w->rows, lora_a, rank, projected, stream)) != KT_OK) return st;
    LoraEpilogue lora;
    lora.p = projected;
    lora.b = lora_b;
    lora.rank = rank;
    lora.scale = scaling;
    return run_matmul(ctx, w, a, c, m, accumulate, alpha, bias, pick(ctx, stream), &lora);
}

kt_status kt_lora_backward(kt_ctx* ctx, const kt_qweight* w, const float* a, const float* dy, const float* projected,
                           const float* lora_a, const float* lora_b, int32_t rank, float scaling, int32_t m, float* dx,
                           int32_t accumulate_dx, float* grad_a, float* grad_b, void* stream) {
    if (!ctx || !w) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    kt_status st = check_lora(m, w->rows, rank, lora_a);
    if (st != KT_OK || m == 0) return st;
    if (!dy || !lora_b || (grad_a && !a) || (grad_b && !projected))
        return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    const cudaStream_t s = pick(ctx, stream);
    if (dx && (st = kt_qmatmul_t(ctx, w, dy, dx, m, accumulate_dx, stream)) != KT_OK) return st;
    if (!dx && !grad_a && !grad_b) return KT_OK;
    void* ws = nullptr;
    KT_CUDA_TRY(stream_workspace(ctx, s, lora_workspace_bytes(m, w->rows, w->columns, rank), &ws), "lora workspace");
    KT_CUDA_TRY(launch_lora_backward(a, dy, projected, lora_a, lora_b, m, w->rows, w->columns, rank, scaling, dx,
                                     grad_a, grad_b, ws, s),
                "lora backward launch");
    return KT_OK;
}

kt_status kt_gather_rows(kt_ctx* ctx, const float* src, const int32_t* rows, int32_t count, int32_t width, float* dst,
                         void* stream) {
    if (!ctx || count < 0 || width <= 0) return fail(KT_ERR_INVALID_ARGUMENT, "bad gather_rows arguments");
    if (count == 0) return KT_OK;
    if (!src || !rows || !dst) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    KT_CUDA_TRY(launch_gather_rows(src, rows, count, width, dst, pick(ctx, stream)), "gather_rows launch");
    return KT_OK;
}

// ---- fusedCrossEntropyLoss with a quantized head (kt_loss.cu)

kt_status kt_fused_cross_entropy(kt_ctx* ctx, const kt_qweight* head, const float* bias, const float* hidden,
                                 int32_t rows, const int32_t* targets, int32_t ignore_index, float* loss,
                                 float* hidden_grad, float* bias_grad, void* stream) {
    if (!ctx || !head || !hidden || !targets || !loss) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (rows <= 0) return fail(KT_ERR_INVALID_ARGUMENT, "targets cannot be empty");
    const int32_t vocab = head->columns, dim = head->rows;
    std::vector<int32_t> active_rows, active_targets;
    for (int32_t i = 0; i < rows; ++i) {
        if (targets[i] == ignore_index) continue;
        if (targets[i] < 0 || targets[i] >= vocab)
            return fail(KT_ERR_INVALID_ARGUMENT,
                        "target " + std::to_string(targets[i]) + " out of bounds " + std::to_string(vocab));
        active_rows.push_back(i);
        active_targets.push_back(targets[i]);
    }
    const cudaStream_t s = pick(ctx, stream);
    KT_CUDA_TRY(cudaSetDevice(ctx->device), "cudaSetDevice");
    const int32_t active = static_cast<int32_t>(active_rows.size());
    if (active == 0) {  // emptyLoss(): 0, no gradients
        KT_CUDA_TRY(cudaMemsetAsync(loss, 0, sizeof(float), s), "loss");
        return KT_OK;
    }
    const int32_t chunk = loss_chunk_rows(vocab, active);
    const bool grads = hidden_grad != nullptr || bias_grad != nullptr;
    int32_t* d_rows = nullptr;
    int32_t* d_targets = nullptr;
    float *stats = nullptr, *inputs = nullptr, *logits = nullptr, *chunk_grad = nullptr;
    auto release = [&] {
        cudaFreeAsync(d_rows, s);
        cudaFreeAsync(d_targets, s);
        cudaFreeAsync(stats, s);
        cudaFreeAsync(inputs, s);
        cudaFreeAsync(logits, s);
        if (chunk_grad) cudaFreeAsync(chunk_grad, s);
    };
    cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&d_rows), active * sizeof(int32_t), s);
    if (e == cudaSuccess) e = cudaMallocAsync(reinterpret_cast<void**>(&d_targets), active * sizeof(int32_t), s);
    if (e == cudaSuccess) e = cudaMallocAsync(reinterpret_cast<void**>(&stats), 3 * static_cast<size_t>(active) * 4, s);
    if (e == cudaSuccess)
        e = cudaMallocAsync(reinterpret_cast<void**>(&inputs), static_cast<size_t>(chunk) * dim * sizeof(float), s);
    if (e == cudaSuccess)
        e = cudaMallocAsync(reinterpret_cast<void**>(&logits), static_cast<size_t>(chunk) * vocab * sizeof(float), s);
    if (e == cudaSuccess && hidden_grad)
        e = cudaMallocAsync(reinterpret_cast<void**>(&chunk_grad), static_cast<size_t>(chunk) * dim * sizeof(float), s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(d_rows, active_rows.data(), active * sizeof(int32_t), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(d_targets, active_targets.data(), active * sizeof(int32_t), cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // the host vectors go out of scope with this call
    if (e != cudaSuccess) {
        release();
        return cuda_fail(e, "fused cross entropy setup");
    }
    float* row_max = stats;
    float* row_sum = stats + active;
    float* row_loss = stats + 2 * static_cast<size_t>(active);
    const float scale = 1.0f / static_cast<float>(active);
    kt_status st = KT_OK;
    for (int32_t start = 0; start < active && st == KT_OK; start += chunk) {
        const int32_t count = std::min(chunk, active - start);
        e = launch_gather_rows(hidden, d_rows + start, count, dim, inputs, s);
        if (e != cudaSuccess) break;
        if ((st = run_matmul(ctx, head, inputs, logits, count, 0, 1.0f, bias, s)) != KT_OK) break;
        e = launch_loss_rows(logits, count, vocab, d_targets + start, row_max + start, row_sum + start,
                             row_loss + start, s);
        if (e != cudaSuccess) break;
        if (!grads) continue;
        e = launch_loss_grads(logits, count, vocab, d_targets + start, row_max + start, row_sum + start, scale,
                              bias_grad, s);
        if (e != cudaSuccess) break;
        if (!hidden_grad) continue;
        if ((st = kt_qmatmul_t(ctx, head, logits, chunk_grad, count, 0, s)) != KT_OK) break;
        e = launch_scatter_add_rows(chunk_grad, d_rows + start, count, dim, hidden_grad, s);
        if (e != cudaSuccess) break;
    }
    if (st == KT_OK && e == cudaSuccess) e = launch_mean_loss(row_loss, active, loss, s);
    release();
    if (st != KT_OK) return st;
    if (e != cudaSuccess) return cuda_fail(e, "fused cross entropy");
    return KT_OK;
}

// ---- decode step (kt_decode.cu)

kt_status kt_rmsnorm(kt_ctx* ctx, const float* x, const float* weight, float* out, int32_t rows, int32_t dim, float eps,
                     void* stream) {
    if (!ctx || !x || !weight || !out || rows <= 0 || dim <= 0) return fail(KT_ERR_INVALID_ARGUMENT, "bad rmsnorm arguments");
    KT_CUDA_TRY(launch_rmsnorm(x, weight, out, rows, dim, eps, pick(ctx, stream)), "rmsnorm launch");
    return KT_OK;
}

kt_status kt_add_rmsnorm(kt_ctx* ctx, float* x, const float* y, const float* weight, float* out, int32_t rows,
                         int32_t dim, float eps, void* stream) {
    if (!ctx || !x || !y || !weight || !out || rows <= 0 || dim <= 0)
        return fail(KT_ERR_INVALID_ARGUMENT, "bad add_rmsnorm arguments");
    KT_CUDA_TRY(launch_add_rmsnorm(x, y, weight, out, rows, dim, eps, pick(ctx, stream)), "add_rmsnorm launch");
    return KT_OK;
}

kt_status kt_rope_kv_seqs(kt_ctx* ctx, float* qkv, int32_t rows, int32_t q_width, int32_t kv_heads,
                          int32_t head_dim, const float* inv_freq, float* k_cache, float* v_cache, int32_t max_seq,
                          int32_t layer, const int32_t* position_dev, int32_t rows_per_seq, int64_t cache_stride,
                          void* stream) {
    if (!ctx || !qkv || !inv_freq || !k_cache || !v_cache || !position_dev || rows <= 0 || rows > 65535 ||
        head_dim <= 0 || head_dim % 2 != 0 || q_width % head_dim != 0 || kv_heads <= 0 || max_seq <= 0 || layer < 0 ||
        rows_per_seq <= 0 || rows % rows_per_seq != 0 || cache_stride < 0 ||
        (rows / rows_per_seq > 1 && cache_stride == 0))
        return fail(KT_ERR_INVALID_ARGUMENT, "bad rope_kv arguments");
    KT_CUDA_TRY(launch_rope_kv(qkv, rows, q_width, kv_heads, head_dim, inv_freq, k_cache, v_cache, max_seq, layer,
                               position_dev, rows_per_seq, cache_stride, pick(ctx, stream)),
                "rope_kv launch");
    return KT_OK;
}

kt_status kt_rope_kv(kt_ctx* ctx, float* qkv, int32_t rows, int32_t q_width, int32_t kv_heads, int32_t head_dim,
                     const float* inv_freq, float* k_cache, float* v_cache, int32_t max_seq, int32_t layer,
                     const int32_t* position_dev, void* stream) {
    return kt_rope_kv_seqs(ctx, qkv, rows, q_width, kv_heads, head_dim, inv_freq, k_cache, v_cache, max_seq, layer,
                           position_dev, rows > 0 ? rows : 1, 0, stream);
}

size_t kt_attention_scratch_floats(int32_t rows, int32_t heads, int32_t head_dim, int32_t max_seq) {
    if (rows <= 0 || heads <= 0 || head_dim <= 0 || max_seq <= 0) return 0;
    return attention_scratch_floats(rows, heads, head_dim, max_seq);
}

kt_status kt_silu_mul_rows(kt_ctx* ctx, const float* gu, float* out, int32_t rows, int32_t hidden, void* stream) {
    if (!ctx || !gu || !out || rows <= 0 || hidden <= 0) return fail(KT_ERR_INVALID_ARGUMENT, "bad silu_mul_rows arguments");
    KT_CUDA_TRY(launch_silu_mul_rows(gu, out, rows, hidden, pick(ctx, stream)), "silu_mul_rows launch");
    return KT_OK;
}

kt_status kt_rope(kt_ctx* ctx, float* v, int32_t rows, int32_t width, int32_t head_dim, const float* inv_freq,
                  const int32_t* position_dev, void* stream) {
    if (!ctx || !v || !inv_freq || !position_dev || rows <= 0 || head_dim <= 0 || head_dim % 2 != 0 ||
        width % head_dim != 0)
        return fail(KT_ERR_INVALID_ARGUMENT, "bad rope arguments");
    KT_CUDA_TRY(launch_rope(v, rows, width, head_dim, inv_freq, position_dev, pick(ctx, stream)), "rope launch");
    return KT_OK;
}

kt_status kt_kv_store(kt_ctx* ctx, const float* k, const float* v, float* k_cache, float* v_cache, int32_t rows,
                      int32_t kv_heads, int32_t head_dim, int32_t max_seq, int32_t layer, const int32_t* position_dev,
                      void* stream) {
    if (!ctx || !k || !v || !k_cache || !v_cache || !position_dev || rows <= 0 || kv_heads <= 0 || head_dim <= 0 ||
        max_seq <= 0 || layer < 0)
        return fail(KT_ERR_INVALID_ARGUMENT, "bad kv_store arguments");
    KT_CUDA_TRY(launch_kv_store(k, v, k_cache, v_cache, rows, kv_heads, head_dim, max_seq, layer, position_dev,
                                pick(ctx, stream)),
                "kv_store launch");
    return KT_OK;
}

kt_status kt_attention_seqs(kt_ctx* ctx, const float* q, const float* k_cache, const float* v_cache, float* context,
                            float* scores, int32_t rows, int32_t q_stride, int32_t heads, int32_t kv_heads,
                            int32_t head_dim, int32_t max_seq, int32_t layer, float scale,
                            const int32_t* position_dev, int32_t rows_per_seq, int64_t cache_stride, void* stream) {
    if (!ctx || !q || !k_cache || !v_cache || !context || !scores || !position_dev || rows <= 0 || rows > 65535 ||
        q_stride < heads * head_dim ||
        heads <= 0 || kv_heads <= 0 || heads % kv_heads != 0 || head_dim <= 0 || head_dim > 254 || max_seq <= 0 ||
        layer < 0 || rows_per_seq <= 0 || rows % rows_per_seq != 0 || cache_stride < 0 ||
        (rows / rows_per_seq > 1 && cache_stride == 0))
        return fail(KT_ERR_INVALID_ARGUMENT, "bad attention arguments");
    KT_CUDA_TRY(launch_attention_decode(q, k_cache, v_cache, context, scores, rows, q_stride, heads, kv_heads,
                                        head_dim, max_seq, layer, scale, position_dev, rows_per_seq, cache_stride,
                                        ctx->d_error, pick(ctx, stream)),
                "attention launch");
    return KT_OK;
}

kt_status kt_qmatmul_swiglu(kt_ctx* ctx, const kt_qweight* w, const float* a, float* gu, float* act, int32_t m,
                            float alpha, const float* bias, void* stream) {
    if (!ctx || !w) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (m < 0) return fail(KT_ERR_INVALID_ARGUMENT, "Negative row count " + std::to_string(m));
    if (m == 0) return KT_OK;
    if (!a || !act) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (w->columns % 2 != 0)
        return fail(KT_ERR_INVALID_ARGUMENT, "SwiGLU needs a gate | up weight with an even number of columns");
    const cudaStream_t s = pick(ctx, stream);
    const QView v = view(w);
    if (swiglu_fused_supported(v, m, a)) {
        MatmulArgs args{a, act, bias, m, 0, alpha, ctx->d_error};
        args.swiglu = 1;
        const size_t need = gemv_imma_workspace_bytes(v, ctx->sm_count);
        void* ws = nullptr;
        if (need > 0) KT_CUDA_TRY(stream_workspace(ctx, s, need, &ws), "qmatmul workspace");
        KT_CUDA_TRY(launch_gemv_imma(v, args, ctx->sm_count, s, ws, need), "qmatmul_swiglu launch");
        return KT_OK;
    }
    if (gemm_tc_supported(v, m, a) && gemm_swiglu_fused(v, m, ctx->sm_count)) {
        // m >= 9: silu(gate) * up in the GEMM's split-K reduction
        MatmulArgs args{a, act, bias, m, 0, alpha, ctx->d_error};
        args.swiglu = 1;
        void* ws = nullptr;
        KT_CUDA_TRY(stream_workspace(ctx, s, gemm_tc_workspace_bytes(v, m, ctx->sm_count), &ws), "qmatmul workspace");
        KT_CUDA_TRY(launch_gemm_tc(v, args, ctx->sm_count, s, ws, gemm_tc_workspace_bytes(v, m, ctx->sm_count)),
                    "qmatmul_swiglu launch");
        return KT_OK;
    }
    if (!gu) return fail(KT_ERR_INVALID_ARGUMENT, "this shape needs the gate | up scratch gu");
    const kt_status st = run_matmul(ctx, w, a, gu, m, 0, alpha, bias, s);
    if (st != KT_OK) return st;
    KT_CUDA_TRY(launch_silu_mul_rows(gu, act, m, w->columns / 2, s), "silu_mul launch");
    return KT_OK;
}

namespace {
// RMSNorm + matmul (+ SwiGLU): the m = 1 INT4 GEMV normalises its input row
// while staging it; elsewhere kt_rmsnorm into xn, then the matmul.
kt_status rmsnorm_matmul(kt_ctx* ctx, const kt_qweight* w, const float* x, const float* norm_w, float eps,
                         float* xn, float* gu, float* c, int32_t m, int32_t accumulate, const float* bias,
                         bool swiglu, void* stream) {
    if (!ctx || !w) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (m < 0) return fail(KT_ERR_INVALID_ARGUMENT, "Negative row count " + std::to_string(m));
    if (m == 0) return KT_OK;
    if (!x || !norm_w || !c) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (swiglu && w->columns % 2 != 0)
        return fail(KT_ERR_INVALID_ARGUMENT, "SwiGLU needs a gate | up weight with an even number of columns");
    const cudaStream_t s = pick(ctx, stream);
    const QView v = view(w);
    const bool norm_in = norm_fused_supported(v, m, x) && reinterpret_cast<uintptr_t>(norm_w) % 16 == 0;
    const bool swiglu_in = swiglu && swiglu_fused_supported(v, m, x);
    if (norm_in && swiglu && !swiglu_in && !gu)
        return fail(KT_ERR_INVALID_ARGUMENT, "this shape needs the gate | up scratch gu");
    // 2..8 rows on the INT4 tensor-core GEMV: the norm in its prologue as well
    // (float4 loads of each x row), silu(gate) * up by a separate kernel
    const bool norm_mma = !norm_in && m >= 2 && gemv_mma_supported(v, m, x) &&
                          reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(norm_w) % 16 == 0;
    if (norm_mma) {
        if (swiglu && !gu) return fail(KT_ERR_INVALID_ARGUMENT, "this shape needs the gate | up scratch gu");
        MatmulArgs args{x, swiglu ? gu : c, bias, m, swiglu ? 0 : accumulate, 1.0f, ctx->d_error};
        args.norm_weight = norm_w;
        args.norm_eps = eps;
        const size_t need = gemv_mma_workspace_bytes(v, m, ctx->sm_count);
        void* ws = nullptr;
        if (need > 0) KT_CUDA_TRY(stream_workspace(ctx, s, need, &ws), "qmatmul workspace");
        KT_CUDA_TRY(launch_gemv_mma(v, args, ctx->sm_count, s, ws, need), "rmsnorm_qmatmul launch");
        if (swiglu) KT_CUDA_TRY(launch_silu_mul_rows(gu, c, m, w->columns / 2, s), "silu_mul launch");
        return KT_OK;
    }
    // m >= 9 on the tcgen05 GEMM: the norm in its bf16 pre-pass, silu(gate) * up
    // in its split-K reduction where that applies, else a separate kernel
    const bool norm_gemm = !norm_in && !norm_mma && gemm_tc_supported(v, m, x) &&
                           reinterpret_cast<uintptr_t>(norm_w) % 16 == 0;
    if (norm_gemm) {
        const bool sw_in = swiglu && gemm_swiglu_fused(v, m, ctx->sm_count);
        if (swiglu && !sw_in && !gu) return fail(KT_ERR_INVALID_ARGUMENT, "this shape needs the gate | up scratch gu");
        MatmulArgs args{x, swiglu && !sw_in ? gu : c, bias, m, swiglu ? 0 : accumulate, 1.0f, ctx->d_error};
        args.norm_weight = norm_w;
        args.norm_eps = eps;
        args.swiglu = sw_in ? 1 : 0;
        const size_t need = gemm_tc_workspace_bytes(v, m, ctx->sm_count);
        void* ws = nullptr;
        KT_CUDA_TRY(stream_workspace(ctx, s, need, &ws), "qmatmul workspace");
        KT_CUDA_TRY(launch_gemm_tc(v, args, ctx->sm_count, s, ws, need), "rmsnorm_qmatmul launch");
        if (swiglu && !sw_in) KT_CUDA_TRY(launch_silu_mul_rows(gu, c, m, w->columns / 2, s), "silu_mul launch");
        return KT_OK;
    }
    if (norm_in) {
        // the norm in the GEMV's prologue; silu(gate) * up in its epilogue, or
        // (weights whose gate and up columns do not share a tile) a separate kernel
        MatmulArgs args{x, swiglu && !swiglu_in ? gu : c, bias, m, swiglu ? 0 : accumulate, 1.0f, ctx->d_error};
        args.norm_weight = norm_w;
        args.norm_eps = eps;
        args.swiglu = swiglu_in ? 1 : 0;
        const size_t need = gemv_imma_workspace_bytes(v, ctx->sm_count);
        void* ws = nullptr;
        if (need > 0) KT_CUDA_TRY(stream_workspace(ctx, s, need, &ws), "qmatmul workspace");
        KT_CUDA_TRY(launch_gemv_imma(v, args, ctx->sm_count, s, ws, need), "rmsnorm_qmatmul launch");
        if (swiglu && !swiglu_in)
            KT_CUDA_TRY(launch_silu_mul_rows(gu, c, m, w->columns / 2, s), "silu_mul launch");
        return KT_OK;
    }
    if (!xn || (swiglu && !gu)) return fail(KT_ERR_INVALID_ARGUMENT, "this shape needs the scratch rows xn / gu");
    KT_CUDA_TRY(launch_rmsnorm(x, norm_w, xn, m, w->rows, eps, s), "rmsnorm launch");
    if (!swiglu) return run_matmul(ctx, w, xn, c, m, accumulate, 1.0f, bias, s);
    return kt_qmatmul_swiglu(ctx, w, xn, gu, c, m, 1.0f, bias, stream);
}
}  // namespace

kt_status kt_rmsnorm_qmatmul(kt_ctx* ctx, const kt_qweight* w, const float* x, const float* norm_w, float eps,
                             float* xn, float* c, int32_t m, int32_t accumulate, const float* bias, void* stream) {
    return rmsnorm_matmul(ctx, w, x, norm_w, eps, xn, nullptr, c, m, accumulate, bias, false, stream);
}

kt_status kt_rmsnorm_qmatmul_swiglu(kt_ctx* ctx, const kt_qweight* w, const float* x, const float* norm_w, float eps,
                                    float* xn, float* gu, float* act, int32_t m, const float* bias, void* stream) {
    return rmsnorm_matmul(ctx, w, x, norm_w, eps, xn, gu, act, m, 0, bias, true, stream);
}

kt_status kt_attention_rope_decode(kt_ctx* ctx, const float* qkv, int32_t rows, int32_t q_width, int32_t heads,
                                   int32_t kv_heads, int32_t head_dim, const float* inv_freq, float* k_cache,
                                   float* v_cache, float* context, float* scratch, int32_t max_seq, int32_t layer,
                                   float scale, const int32_t* position_dev, int64_t cache_stride, void* stream) {
    if (!ctx || !qkv || !inv_freq || !k_cache || !v_cache || !context || !scratch || !position_dev || rows <= 0 ||
        rows > 65535 || heads <= 0 || kv_heads <= 0 || head_dim <= 0 || q_width != heads * head_dim ||
        max_seq <= 0 || layer < 0 || cache_stride < 0 || (rows > 1 && cache_stride == 0))
        return fail(KT_ERR_INVALID_ARGUMENT, "bad fused attention arguments");
    if (!attention_fused_supported(heads, kv_heads, head_dim, max_seq))
        return fail(KT_ERR_UNSUPPORTED,
                    "fused decode attention needs heads / kv_heads <= 8, head_dim 64 or 128 and max_seq <= 16384");
    KT_CUDA_TRY(launch_attention_decode_fused(qkv, rows, q_width, heads, kv_heads, head_dim, inv_freq, k_cache,
                                              v_cache, context, scratch, max_seq, layer, scale, position_dev,
                                              cache_stride, ctx->d_error, pick(ctx, stream)),
                "fused attention launch");
    return KT_OK;
}

kt_status kt_attention_decode(kt_ctx* ctx, const float* q, const float* k_cache, const float* v_cache, float* context,
                              float* scores, int32_t rows, int32_t q_stride, int32_t heads, int32_t kv_heads,
                              int32_t head_dim, int32_t max_seq, int32_t layer, float scale,
                              const int32_t* position_dev, void* stream) {
    return kt_attention_seqs(ctx, q, k_cache, v_cache, context, scores, rows, q_stride, heads, kv_heads, head_dim,
                             max_seq, layer, scale, position_dev, rows > 0 ? rows : 1, 0, stream);
}

kt_status kt_silu_mul(kt_ctx* ctx, float* gate, const float* up, int64_t n, void* stream) {
    if (!ctx || !gate || !up || n < 0) return fail(KT_ERR_INVALID_ARGUMENT, "bad silu_mul arguments");
    if (n == 0) return KT_OK;
    KT_CUDA_TRY(launch_silu_mul(gate, up, n, pick(ctx, stream)), "silu_mul launch");
    return KT_OK;
}

kt_status kt_add(kt_ctx* ctx, float* x, const float* y, int64_t n, void* stream) {
    if (!ctx || !x || !y || n < 0) return fail(KT_ERR_INVALID_ARGUMENT, "bad add arguments");
    if (n == 0) return KT_OK;
    KT_CUDA_TRY(launch_add(x, y, n, pick(ctx, stream)), "add launch");
    return KT_OK;
}

kt_status kt_argmax(kt_ctx* ctx, const float* logits, int32_t rows, int32_t n, int32_t* out_dev, void* stream) {
    if (!ctx || !logits || !out_dev || rows <= 0 || n <= 0) return fail(KT_ERR_INVALID_ARGUMENT, "bad argmax arguments");
    const cudaStream_t s = pick(ctx, stream);
    void* ws = nullptr;
    KT_CUDA_TRY(stream_workspace(ctx, s, kWorkspaceReservedBytes + argmax_scratch_bytes(rows), &ws), "argmax workspace");
    KT_CUDA_TRY(launch_argmax(logits, rows, n, out_dev, static_cast<unsigned char*>(ws) + kWorkspaceReservedBytes, s),
                "argmax launch");
    return KT_OK;
}

kt_status kt_dequantize_column(kt_ctx* ctx, const kt_qweight* w, const int32_t* columns_dev, int32_t count,
                               float* out_dev, int32_t* status_dev, void* stream) {
    if (!ctx || !w || !columns_dev || !out_dev || count <= 0 || count > 65535)
        return fail(KT_ERR_INVALID_ARGUMENT, "bad dequantize_column arguments");
    KT_CUDA_TRY(launch_dequantize_column(view(w), columns_dev, count, out_dev, status_dev, pick(ctx, stream)),
                "dequantize_column launch");
    return KT_OK;
}

kt_status kt_increment(kt_ctx* ctx, int32_t* value_dev, int32_t delta, void* stream) {
    if (!ctx || !value_dev) return fail(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    KT_CUDA_TRY(launch_increment(value_dev, delta, pick(ctx, stream)), "increment launch");
    return KT_OK;
}

}  // extern "C"
