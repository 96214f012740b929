// kt_noalloc.cu -- kt_qmatmul_noalloc: the quantized matmul of kt_qmatmul for
// callers that must not allocate device memory.
//
// Several of kt_qmatmul's kernels need device scratch memory: the INT4
// tensor-core GEMVs split K across CTAs (per-tile arrival counters and partial
// tiles), and the tcgen05 GEMM keeps a bf16 copy of the activations and, when
// it splits K, fp32 partial tiles.  kt_qmatmul takes that scratch from a
// per-stream buffer that it allocates on first use and grows on demand.  Some
// callers cannot let a library allocate at call time: a decode loop with a
// fixed memory budget that must not trigger cudaMalloc (which can synchronize
// the device and fail under memory pressure mid-step), or a host runtime that
// accounts for every device byte itself.  This entry point runs exactly the
// kernels kt_qmatmul would choose, with the scratch in the library image
// instead: a file-scope __device__ array of kStaticWorkspaceBytes (16 MiB),
// zero-initialized when the module loads.  Its address is looked up once per
// device.
//
// Rules for callers:
//  * The first call on a device looks up the array's address
//    (cudaGetSymbolAddress); make that first call before capturing a stream.
//  * The arrival counters at the front of the array start at zero (static
//    initialization) and every launch leaves them at zero: every CTA of a grid
//    runs to its end, also after one of its bounded waits timed out (that
//    launch's output and partial tiles are then invalid and the context's error
//    word is set; the next launch overwrites the partials before reading them).
//  * There is one array per device: calls that overlap in time on that device
//    (different streams, threads or processes sharing the context) race on it.
//    Order them on one stream.
//  * A shape whose scratch exceeds kStaticWorkspaceBytes is rejected with
//    KT_ERR_INVALID_ARGUMENT (kt_qmatmul handles it).  Shapes the tensor-core
//    kernels do not take run the fp32 kernels, which need no scratch, as in
//    kt_qmatmul.
#include <mutex>
#include <string>

#include "kt_internal.h"

namespace {

constexpr size_t kStaticWorkspaceBytes = static_cast<size_t>(16) << 20;  // 16 MiB
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_static_workspace[kStaticWorkspaceBytes];

std::mutex g_addr_mutex;
void* g_addr[kMaxDevices] = {};

kt_status fail_noalloc(kt_status st, const std::string& msg) {
    kt::set_error(msg);
    return st;
}

kt_status too_big(size_t need) {
    return fail_noalloc(KT_ERR_INVALID_ARGUMENT, "this shape needs " + std::to_string(need) +
                                                     " bytes of scratch; the static workspace holds " +
                                                     std::to_string(kStaticWorkspaceBytes) + " (use kt_qmatmul)");
}

}  // namespace

extern "C" kt_status kt_qmatmul_noalloc(kt_ctx* ctx, const kt_qweight* w, const float* a, float* c, int32_t m,
                                        int32_t accumulate, float alpha, const float* bias, void* stream) {
    using namespace kt;
    if (!ctx || !w) return fail_noalloc(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (m < 0) return fail_noalloc(KT_ERR_INVALID_ARGUMENT, "Negative row count " + std::to_string(m));
    if (m == 0) return KT_OK;
    if (!a || !c) return fail_noalloc(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (ctx->device < 0 || ctx->device >= kMaxDevices)
        return fail_noalloc(KT_ERR_UNSUPPORTED, "device index beyond the static workspace table");
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return fail_noalloc(KT_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
    void* ws = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_addr_mutex);
        if (g_addr[ctx->device] == nullptr) {
            void* p = nullptr;
            e = cudaGetSymbolAddress(&p, g_static_workspace);
            if (e != cudaSuccess)
                return fail_noalloc(KT_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
            g_addr[ctx->device] = p;
        }
        ws = g_addr[ctx->device];
    }
    const QView v = view(w);
    const MatmulArgs args{a, c, bias, m, accumulate, alpha, ctx->d_error};
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    // The same routing as kt_qmatmul (run_matmul in kt_api.cu), scratch from the static array.
    if (gemv_imma_supported(v, m, a)) {
        const size_t need = gemv_imma_workspace_bytes(v, ctx->sm_count);
        if (need > kStaticWorkspaceBytes) return too_big(need);
        e = launch_gemv_imma(v, args, ctx->sm_count, s, need > 0 ? ws : nullptr, kStaticWorkspaceBytes);
    } else if (gemv_mma_supported(v, m, a)) {
        const size_t need = gemv_mma_workspace_bytes(v, m, ctx->sm_count);
        if (need > kStaticWorkspaceBytes) return too_big(need);
        e = launch_gemv_mma(v, args, ctx->sm_count, s, need > 0 ? ws : nullptr, kStaticWorkspaceBytes);
    } else if (gemv_fast_supported(v, m, a)) {
        e = launch_gemv(v, args, ctx->sm_count, s);
    } else if (gemm_tc_supported(v, m, a)) {
        const size_t need = gemm_tc_workspace_bytes(v, m, ctx->sm_count);
        if (need > kStaticWorkspaceBytes) return too_big(need);
        e = launch_gemm_tc(v, args, ctx->sm_count, s, ws, kStaticWorkspaceBytes);
    } else {
        e = launch_matmul_generic(v, args, s);
    }
    if (e != cudaSuccess)
        return fail_noalloc(KT_ERR_CUDA, std::string("qmatmul_noalloc launch: ") + cudaGetErrorString(e));
    return KT_OK;
}
