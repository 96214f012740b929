// kt_internal.h -- shared host-side declarations of the B200 quantized-matmul
// library: the weight and context objects behind the C ABI (include/kt_cuda.h)
// and the launchers each kernel translation unit exports.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/kt_cuda.h"

struct kt_ctx {
    int device = 0;
    int sm_count = 0;
    int max_smem_optin = 0;
    cudaStream_t stream = nullptr;  // the context's own non-blocking stream
    int32_t* d_status = nullptr;    // device status word for kernels that detect NaN / bad input
    int32_t* d_error = nullptr;     // sticky device error word: bounded waits that timed out
    std::mutex host_mutex;          // serialises the host-buffer entry points
    // staging for kt_qmatmul_host (grown on demand, owned by the context)
    float* h2d_a = nullptr;
    float* d2h_c = nullptr;
    float* bias_buf = nullptr;
    size_t a_cap = 0, c_cap = 0, bias_cap = 0;
    // Kernel workspaces, one per stream that launched on this context (launches
    // on one stream are ordered, so they may share one); grown by replacement,
    // the replaced ones kept until kt_destroy because queued work may use them.
    struct Workspace {
        cudaStream_t stream;
        void* ptr;
        size_t bytes;
    };
    std::mutex ws_mutex;
    std::vector<Workspace> workspaces;
    std::vector<void*> retired;
};

struct kt_qweight {
    kt_ctx* ctx = nullptr;
    int32_t bits = 0, group_size = 0, rows = 0, columns = 0;
    int32_t groups = 0, bytes_per_row = 0, stored_columns = 0;
    uint8_t* qdata = nullptr;  // device
    float* scales = nullptr;   // device
    uint8_t* zeros = nullptr;  // device, INT4 only
    // TMA descriptors of qdata as a 2-D u8 tensor [rows x bytes_per_row] with
    // boxes of 8 rows x 128 / 256 bytes (built when bytes_per_row % 16 == 0).
    alignas(64) CUtensorMap tmap_w128;
    alignas(64) CUtensorMap tmap_w256;
    bool has_tmaps = false;
    // Box of 32 rows x 128 bytes with the 128-byte swizzle (INT4 tensor-core
    // GEMV; built when bytes_per_row % 16 == 0 and bytes_per_row >= 128).
    alignas(64) CUtensorMap tmap_mma;
    bool has_tmap_mma = false;
    // Box of 64 rows x 128 bytes, no swizzle (INT4 tensor-core GEMM; same condition).
    alignas(64) CUtensorMap tmap_raw64;
    bool has_tmap_raw64 = false;
    // row-parallel exchange-fused GEMV agreed by every rank for this shard on
    // communicator tp_comm (kt_qmatmul_row_parallel): 0 not asked yet, 1 fused, 2 NCCL
    int32_t tp_fused = 0;
    const void* tp_comm = nullptr;
};

namespace kt {

// Thread-local last-error message (kt_last_error()).
void set_error(const std::string& msg);

// Shape of one quantized matrix as the kernels see it.
struct QView {
    const uint8_t* q;
    const float* scales;
    const uint8_t* zeros;
    int32_t bits, group_size, rows, columns, groups, bytes_per_row;
    const CUtensorMap* tmap_w128;  // NULL when the weight has no TMA descriptors
    const CUtensorMap* tmap_w256;
    const CUtensorMap* tmap_mma;
    const CUtensorMap* tmap_raw64;
};

inline QView view(const kt_qweight* w) {
    return QView{w->qdata, w->scales, w->zeros, w->bits, w->group_size, w->rows, w->columns, w->groups,
                 w->bytes_per_row, w->has_tmaps ? &w->tmap_w128 : nullptr,
                 w->has_tmaps ? &w->tmap_w256 : nullptr, w->has_tmap_mma ? &w->tmap_mma : nullptr,
                 w->has_tmap_raw64 ? &w->tmap_raw64 : nullptr};
}

// The low-rank term of LoRALinear.forwardInto (LoRA.kt:39-46) applied in a
// matmul's epilogue: c[t][j] += scale * sum_r p[t][r] * b[r][j], with
// p = a . A ([m x rank], computed before the matmul) and b = B ([rank x N]).
struct LoraEpilogue {
    const float* p = nullptr;  // NULL: no LoRA term
    const float* b = nullptr;
    int32_t rank = 0;
    float scale = 0.0f;
};
#ifdef __CUDACC__
__device__ __forceinline__ float lora_term(const LoraEpilogue& l, int t, int col, int n) {
    const float* pr = l.p + static_cast<int64_t>(t) * l.rank;
    const float* bc = l.b + col;
    float s = 0.0f;
    for (int r = 0; r < l.rank; ++r) s = fmaf(__ldg(pr + r), __ldg(bc + static_cast<int64_t>(r) * n), s);
    return l.scale * s;
}
#endif

// The dispatch behind kt_qmatmul (kt_api.cu): argument-checked by the caller.
kt_status run_qmatmul(kt_ctx* ctx, const kt_qweight* w, const float* a, float* c, int32_t m, int32_t accumulate,
                      float alpha, const float* bias, cudaStream_t s, const LoraEpilogue* lora = nullptr);

// Zero-initialised device workspace of at least `bytes` for launches on stream
// `s` (kt_api.cu).  Its first kWorkspaceReservedBytes hold the split-K arrival
// counters of the INT4 GEMV and of the INT4 GEMM at fixed offsets (zero
// between launches, whatever shapes ran before); kernels use the rest freely.
cudaError_t stream_workspace(kt_ctx* ctx, cudaStream_t s, size_t bytes, void** out);
constexpr size_t kWorkspaceReservedBytes = static_cast<size_t>(96) << 10;
constexpr size_t kGemvTicketOffset = 0;
constexpr size_t kGemmTicketOffset = static_cast<size_t>(32) << 10;
constexpr size_t kLoraTicketOffset = static_cast<size_t>(64) << 10;
constexpr int kTicketCapEach = 8192;  // counters per kernel family


// A 2-D tiled TMA descriptor (kt_api.cu): `inner` x `outer` elements of
// `elem_bytes`, rows `row_bytes` apart, box `box_inner` x `box_outer`.
bool encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType type, uint32_t elem_bytes, const void* base,
                    uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                    CUtensorMapSwizzle swizzle);

// Rows per TMA box / pipeline stage of the streaming kernel.
constexpr int kStageRows = 8;
// Builds kt_qweight::tmap_w128 / tmap_w256 (kt_api.cu).
bool make_tensor_maps(kt_qweight* w);

// ---- kt_lora.cu  (LoRALinear over a quantized base; rank 1..kLoraMaxRank)
constexpr int kLoraMaxRank = 256;
size_t lora_workspace_bytes(int32_t m, int32_t K, int32_t N, int32_t rank);
cudaError_t launch_lora_project(const float* a, int32_t m, int32_t K, const float* A, int32_t rank, float* p,
                                void* workspace, cudaStream_t s);
cudaError_t launch_lora_backward(const float* a, const float* dy, const float* p, const float* A, const float* B,
                                 int32_t m, int32_t K, int32_t N, int32_t rank, float scale, float* dx, float* dA,
                                 float* dB, void* workspace, cudaStream_t s);

// ---- kt_loss.cu  (fusedCrossEntropyLoss with a quantized head)
int32_t loss_chunk_rows(int32_t vocab, int32_t active);
cudaError_t launch_gather_rows(const float* src, const int32_t* rows, int32_t count, int32_t dim, float* dst,
                               cudaStream_t s);
cudaError_t launch_loss_rows(const float* logits, int32_t count, int32_t vocab, const int32_t* targets,
                             float* row_max, float* row_sum, float* row_loss, cudaStream_t s);
cudaError_t launch_loss_grads(float* logits, int32_t count, int32_t vocab, const int32_t* targets,
                              const float* row_max, const float* row_sum, float scale, float* bias_grad,
                              cudaStream_t s);
cudaError_t launch_scatter_add_rows(const float* src, const int32_t* rows, int32_t count, int32_t dim, float* dst,
                                    cudaStream_t s);
cudaError_t launch_mean_loss(const float* row_loss, int32_t active, float* out, cudaStream_t s);

// ---- kt_quantize.cu
cudaError_t launch_quantize(const float* data, int32_t rows, int32_t columns, int32_t bits, int32_t group_size,
                            uint8_t* qdata, float* scales, uint8_t* zeros, int32_t* d_status, cudaStream_t s);
cudaError_t launch_dequantize(const QView& w, float* out, cudaStream_t s);
cudaError_t launch_dequantize_rows(const QView& w, const int32_t* rows, int32_t count, float* out,
                                   int32_t* d_status, cudaStream_t s);

// ---- kt_gemv.cu  (fp32-accumulate CUDA-core kernels; small m)
// Row-parallel exchange fused into the m = 1 GEMV (set up by kt_tp.cu): the
// thread finishing output column j stores {call number, alpha * its partial}
// as one 64-bit word into every rank's receive area over peer memory, then
// polls (bounded) the word of every rank for column j until it carries this
// call's number and writes c = sum over ranks in rank order + (accumulate ? c
// : 0) + bias.  A word is stored and read whole, so its number vouches for
// its value: no fences, no separate flags.  nranks == 0: no exchange.
struct TpExchange {
    unsigned long long* const* recv = nullptr;  // device array [P]: rank q's receive area ([2][P][n_cap] words), mapped here
    uint32_t* state = nullptr;                  // this rank's own {calls completed, CTAs exited in this call}
    int32_t nranks = 0, rank = 0, n_cap = 0;
    uint64_t wait_ns = 0;                       // limit of the wait for the other ranks' words
};

struct MatmulArgs {
    const float* a;
    float* c;
    const float* bias;
    int32_t m;
    int32_t accumulate;
    float alpha;
    int32_t* err;  // context error word (bounded-wait timeouts)
    LoraEpilogue lora;
    TpExchange tp;
    // SwiGLU epilogue (fused gate|up weight, N = 2H, split-half packed so gate
    // column j and up column H + j are the two nibbles of byte j): c receives
    // [m x H] silu(gate) * up instead of [m x N] (accumulate must be 0).
    int32_t swiglu = 0;
    // RMSNorm of the input row before the product (RMSNorm.forwardInto,
    // RMSNorm.kt:71-90): a is read as a * (1 / sqrt(mean(a^2) + eps)) * norm_weight
    // (norm_weight NULL: off; the INT4 GEMVs: m = 1 integer, m = 2..8 fp16
    // products; the tcgen05 GEMM: in its bf16 pre-pass).
    const float* norm_weight = nullptr;
    float norm_eps = 0.0f;
};
// Largest m the fp32-accumulate streaming kernel takes.
constexpr int kGemvMaxM = 8;
bool gemv_fast_supported(const QView& w, int32_t m, const float* a);
void set_gemv_tuning(int lane_bytes, int cluster_k);
cudaError_t launch_gemv(const QView& w, const MatmulArgs& args, int sm_count, cudaStream_t s);
cudaError_t launch_matmul_generic(const QView& w, const MatmulArgs& args, cudaStream_t s);

// ---- kt_gemv_mma.cu  (INT4, m <= kGemvMmaMaxM: tensor-core products, fp32 group combine;
// m = 5..8 as two groups of 4 tokens in one launch)
constexpr int kGemvMmaMaxM = 8;
bool gemv_mma_supported(const QView& w, int32_t m, const float* a);
void set_mma_tuning(int k_splits);
// Device workspace one launch needs (0: none): split-K partial tiles and
// per-tile arrival counters.  The counters must be zero before the first
// launch; every launch leaves them zero.  Launches that share a workspace
// must be ordered (one stream).
size_t gemv_mma_workspace_bytes(const QView& w, int32_t m, int sm_count);
cudaError_t launch_gemv_mma(const QView& w, const MatmulArgs& args, int sm_count, cudaStream_t s, void* workspace,
                            size_t workspace_bytes);

// ---- kt_gemv_imma.cu  (INT4, m = 1: integer tensor-core products, fp32 group combine)
bool gemv_imma_supported(const QView& w, int32_t m, const float* a);
// The kernels that take MatmulArgs::swiglu for this weight and m.
bool swiglu_fused_supported(const QView& w, int32_t m, const float* a);
// The kernels that take MatmulArgs::norm_weight for this weight and m.
bool norm_fused_supported(const QView& w, int32_t m, const float* a);
void set_imma_tuning(int k_splits);
size_t gemv_imma_workspace_bytes(const QView& w, int sm_count, bool no_cluster = false);
// The shard can run the exchange-fused GEMV: the m = 1 kernel applies, and its
// whole grid is resident at once (a CTA waiting on other ranks must not keep
// another CTA of its grid from running).
bool gemv_imma_tp_supported(const QView& w, int sm_count);
cudaError_t launch_gemv_imma(const QView& w, const MatmulArgs& a, int sm_count, cudaStream_t s, void* workspace,
                             size_t workspace_bytes);


// ---- kt_gemm_tc.cu  (INT4, m >= 9: bf16 tcgen05 MMAs, TMEM accumulators)
bool gemm_tc_supported(const QView& w, int32_t m, const float* a);
// The transposed product (kt_qmatmul_t) on tcgen05: m >= 16, INT4 with N % 128 == 0 or INT8 with N % 64 == 0,
// group size 32, 64 or a multiple of 128 (kt_gemm_tc.cu).
bool gemm_t_supported(const QView& w, int32_t m, const float* dy);
size_t gemm_t_workspace_bytes(const QView& w, int32_t m, int sm_count);
cudaError_t launch_gemm_t(const QView& w, const float* dy, float* dx, int32_t m, int32_t accumulate, int32_t* err,
                          int sm_count, cudaStream_t s, void* workspace, size_t workspace_bytes);
size_t gemm_tc_workspace_bytes(const QView& w, int32_t m, int sm_count);
// The GEMM forms silu(gate) * up in its split-K reduction for this INT4 gate | up
// weight at this m (MatmulArgs::swiglu); elsewhere the caller runs kt_silu_mul_rows.
bool gemm_swiglu_fused(const QView& w, int32_t m, int sm_count);
cudaError_t launch_gemm_tc(const QView& w, const MatmulArgs& args, int sm_count, cudaStream_t s, void* workspace,
                           size_t workspace_bytes);

// ---- kt_shard.cu  (tensor-parallel shards)
// [begin, end) of shard `index` of `parts` along rows (axis 0: whole groups of
// group_size rows) or columns (axis 1); false for bad arguments or an empty shard.
bool shard_bounds(int32_t axis, int32_t extent, int32_t group_size, int32_t parts, int32_t index, int32_t* begin,
                  int32_t* end);
// dst (INT4, allocated, dst->columns wide) <- columns [c0, c0 + dst->columns) of src, repacked.
cudaError_t launch_repack_int4_columns(const kt_qweight* src, int32_t c0, const kt_qweight* dst, cudaStream_t s);
// dst (INT4, allocated, sum of the sources' columns wide) <- the sources' columns side by side.
cudaError_t launch_concat_int4_columns(const kt_qweight* const* srcs, int32_t count, const kt_qweight* dst,
                                       cudaStream_t s);

// ---- kt_decode.cu  (the decode step around the matmul)
cudaError_t launch_rmsnorm(const float* x, const float* w, float* out, int rows, int dim, float eps, cudaStream_t s);
cudaError_t launch_add_rmsnorm(float* x, const float* y, const float* w, float* out, int rows, int dim, float eps,
                               cudaStream_t s);
// Row r of rope_kv / attention: sequence r / rows_per_seq (its KV cache
// cache_stride floats after the previous sequence's), position *pos + r % rows_per_seq.
cudaError_t launch_rope_kv(float* qkv, int rows, int q_width, int kv_heads, int head_dim, const float* inv_freq,
                           float* kc, float* vc, int max_seq, int layer, const int32_t* pos, int rows_per_seq,
                           int64_t cache_stride, cudaStream_t s);
size_t attention_scratch_floats(int rows, int heads, int head_dim, int max_seq);
// One decode token per sequence (row r = sequence r at position *pos): RoPE of
// the query and key heads, key / value into the cache, attention and the merge
// of its splits in one launch; scratch as attention_scratch_floats, its
// tickets zero before the first launch (each launch leaves them zero).
bool attention_fused_supported(int heads, int kv_heads, int head_dim, int max_seq);
cudaError_t launch_attention_decode_fused(const float* qkv, int rows, int q_width, int heads, int kv_heads,
                                          int head_dim, const float* inv_freq, float* kc, float* vc, float* ctx,
                                          float* scratch, int max_seq, int layer, float scale, const int32_t* pos,
                                          int64_t cache_stride, int32_t* err, cudaStream_t s);
cudaError_t launch_silu_mul_rows(const float* gu, float* out, int rows, int hidden, cudaStream_t s);
cudaError_t launch_rope(float* v, int rows, int width, int head_dim, const float* inv_freq, const int32_t* pos,
                        cudaStream_t s);
cudaError_t launch_kv_store(const float* k, const float* v, float* kc, float* vc, int rows, int kv_heads, int head_dim,
                            int max_seq, int layer, const int32_t* pos, cudaStream_t s);
cudaError_t launch_attention_decode(const float* q, const float* kc, const float* vc, float* ctx, float* scores,
                                    int rows, int q_stride, int heads, int kv_heads, int head_dim, int max_seq,
                                    int layer, float scale, const int32_t* pos, int rows_per_seq,
                                    int64_t cache_stride, int32_t* err, cudaStream_t s);
cudaError_t launch_silu_mul(float* gate, const float* up, int64_t n, cudaStream_t s);
cudaError_t launch_add(float* x, const float* y, int64_t n, cudaStream_t s);
size_t argmax_scratch_bytes(int rows);
cudaError_t launch_argmax(const float* logits, int rows, int n, int32_t* out, void* scratch, cudaStream_t s);
cudaError_t launch_dequantize_column(const QView& w, const int32_t* col, int count, float* out, int32_t* status,
                                     cudaStream_t s);
cudaError_t launch_increment(int32_t* p, int32_t delta, cudaStream_t s);

// ---- kt_backward.cu
// Workspace of one call (0: none); the per-chunk partial sums follow the reserved front.
size_t matmul_t_workspace_bytes(const QView& w, int32_t m);
cudaError_t launch_matmul_t(const QView& w, const float* dy, float* dx, int32_t m, int32_t accumulate,
                            cudaStream_t s, void* workspace, size_t workspace_bytes);

}  // namespace kt
