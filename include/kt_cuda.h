/*
 * kt_cuda.h -- C ABI of the B200 (sm_100a) implementation of Kotensor's
 * group-wise weight-only INT8/INT4 quantized matmul.
 *
 * Every entry point is extern "C", takes plain pointers and sizes, returns a
 * kt_status and never lets a C++ exception cross the boundary.  The message of
 * the last failure on the calling thread is kt_last_error().
 *
 * Reference interfaces (paths inside the Kotensor project, Engine/kotensor/):
 *   Quantization(bits, groupSize)                      src/main/kotlin/QuantizedTensor.kt:10-25
 *   QuantizedTensor(qdata, scales, zeros, shape, ...)  src/main/kotlin/QuantizedTensor.kt:36-70
 *   QuantizedTensor.quantize(data, rows, columns, q)   src/main/kotlin/QuantizedTensor.kt:261-278
 *   QuantizedTensor.dequantize / dequantizeRow         src/main/kotlin/QuantizedTensor.kt:188-249
 *   MatMul.multiplyQuantized(a, W, c, m, acc, alpha)   src/main/kotlin/MatMul.kt:460-486
 *   MatMul.multiplyByQuantizedTransposed(dy,W,dx,m,acc) src/main/kotlin/MatMul.kt:954-981
 *   QuantizedLinear.forwardInto (+ bias)               src/main/kotlin/QuantizedLinear.kt:18-25
 *   Tensor.matmulDequantInto(W, out, acc, scale)       src/main/kotlin/Tensor.kt:180-188
 *
 * Layout (identical to the reference's heap and safetensors layout,
 * QuantizedTensor.kt:45-49, Transformer.kt:423-428):
 *   rows = K = in-features, columns = N = out-features, groups G = ceil(K / groupSize)
 *   qdata  INT8: int8 [K x N] row-major.
 *          INT4: uint8 [K x ceil(N/2)] split-half packed: column c < half sits in
 *          the low nibble of byte c, column c >= half in the high nibble of byte
 *          c - half (half = ceil(N/2)).
 *   scales float32 [G x N];  zeros (INT4 only) uint8 [G x N], values 0..15.
 *   a / c fp32 row-major [m x K] / [m x N].
 *
 * Streams: a `stream` argument is a cudaStream_t; NULL is CUDA's default
 * stream (kt_ctx_stream() returns the context's own non-blocking stream).
 * Calls are stream-ordered and asynchronous unless documented otherwise.  Results are deterministic: the same inputs give the same bits on
 * every run (fixed reduction order, no floating-point atomics).
 */
#ifndef KT_CUDA_H
#define KT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t kt_status;
enum {
    KT_OK = 0,
    KT_ERR_INVALID_ARGUMENT = 1, /* reference: require(...) -> IllegalArgumentException */
    KT_ERR_NAN = 2,              /* reference: Float.roundToInt() on NaN -> IllegalArgumentException */
    KT_ERR_CUDA = 3,             /* CUDA runtime failure -> IllegalStateException */
    KT_ERR_OUT_OF_MEMORY = 4,
    KT_ERR_UNSUPPORTED = 5,
    KT_ERR_NCCL = 6,
    KT_ERR_IO = 7                /* reference: IOException / FileNotFoundException */
};

typedef struct kt_ctx kt_ctx;
typedef struct kt_qweight kt_qweight;

/* Read-only view of a device-resident quantized weight. */
typedef struct {
    int32_t bits, group_size, rows, columns, groups, bytes_per_row, stored_columns;
    int64_t size_in_bytes;        /* QuantizedTensor.sizeInBytes, QuantizedTensor.kt:97-98 */
    const void* qdata;            /* device pointers */
    const float* scales;
    const uint8_t* zeros;         /* NULL for INT8 */
} kt_qweight_info;

/* ------------------------------------------------------------ library */
int32_t kt_version(void);
const char* kt_last_error(void);
/* Quantization(bits, groupSize) validation, QuantizedTensor.kt:14-17. */
kt_status kt_check_quantization(int32_t bits, int32_t group_size);

/* ------------------------------------------------------------ context (no reference counterpart:
 * the reference's MatMul is a process-wide object with a ForkJoinPool, MatMul.kt:15-57) */
kt_status kt_init(int32_t device, kt_ctx** out);
kt_status kt_destroy(kt_ctx* ctx);
kt_status kt_ctx_stream(kt_ctx* ctx, void** stream_out);
kt_status kt_alloc(kt_ctx* ctx, size_t bytes, void** out);
kt_status kt_free(kt_ctx* ctx, void* ptr);
kt_status kt_memcpy_h2d(kt_ctx* ctx, void* dst_dev, const void* src_host, size_t bytes, void* stream);
kt_status kt_memcpy_d2h(kt_ctx* ctx, void* dst_host, const void* src_dev, size_t bytes, void* stream);
kt_status kt_stream_sync(kt_ctx* ctx, void* stream);

/* ------------------------------------------------------------ quantized weights */

/* QuantizedTensor(qdata, scales, zeros, shape=[rows, columns], bits, groupSize),
 * QuantizedTensor.kt:36-70: copies host bytes in the reference layout into HBM.
 * zeros must be NULL for INT8 and non-NULL for INT4 ("4-bit tensors need zero
 * points").  Synchronous. */
kt_status kt_qweight_upload(kt_ctx* ctx, int32_t bits, int32_t group_size, int32_t rows, int32_t columns,
                            const void* qdata, const float* scales, const uint8_t* zeros, kt_qweight** out);

/* Same, from buffers already on the device (copied device-to-device on `stream`). */
kt_status kt_qweight_from_device(kt_ctx* ctx, int32_t bits, int32_t group_size, int32_t rows, int32_t columns,
                                 const void* qdata_dev, const float* scales_dev, const uint8_t* zeros_dev,
                                 void* stream, kt_qweight** out);

/* QuantizedTensor.quantize(data, rows, columns, Quantization(bits, groupSize)),
 * QuantizedTensor.kt:261-324, run on the GPU: data_dev is fp32 [rows x columns]
 * row-major on the device.  Bytes, scales and zeros are bit-identical to the
 * reference quantizer.  Synchronous on `stream` (the NaN check needs the result):
 * returns KT_ERR_NAN, and no weight, where Kotlin's roundToInt would throw. */
kt_status kt_quantize(kt_ctx* ctx, int32_t bits, int32_t group_size, int32_t rows, int32_t columns,
                      const float* data_dev, void* stream, kt_qweight** out);

kt_status kt_qweight_info_get(const kt_qweight* w, kt_qweight_info* out);

/* Copies the weight back to host buffers in the reference layout
 * (qdata: rows*bytes_per_row bytes, scales: groups*columns floats, zeros:
 * groups*columns bytes or NULL for INT8).  Synchronous. */
kt_status kt_qweight_download(const kt_qweight* w, void* qdata, float* scales, uint8_t* zeros);

kt_status kt_qweight_free(kt_qweight* w);

/* ------------------------------------------------------------ tensor parallelism
 * Shards of one weight for P ranks (no reference counterpart: the reference runs
 * on one host).  Quantization is per (row group, column), so a shard is exactly
 * the quantization of the same block of the fp32 weight: bytes, scales and
 * zeros bit-identical to quantizing the sliced fp32 weight.
 *   axis 0 (row-parallel, split K): shard `index` holds whole groups
 *     [index*G/P, (index+1)*G/P) of the G = ceil(K/groupSize) groups;
 *   axis 1 (column-parallel, split N): columns [index*N/P, (index+1)*N/P), INT4
 *     repacked with half = ceil(N_shard / 2).
 * kt_shard_bounds gives [begin, end) along that axis (host only, no GPU). */
kt_status kt_shard_bounds(int32_t axis, int32_t extent, int32_t group_size, int32_t parts, int32_t index,
                          int32_t* begin, int32_t* end);
/* A new device weight holding shard `index` of `parts` of w, built on `stream`. */
kt_status kt_qweight_shard(kt_ctx* ctx, const kt_qweight* w, int32_t axis, int32_t parts, int32_t index,
                           void* stream, kt_qweight** out);
/* A new device weight holding rows (axis 0) or columns (axis 1) [begin, end) of w;
 * a row slice must start on a group boundary and end on one or at K (the blocks
 * kt_qweight_shard takes, and e.g. q / k / v out of a fused q|k|v weight). */
kt_status kt_qweight_slice(kt_ctx* ctx, const kt_qweight* w, int32_t axis, int32_t begin, int32_t end, void* stream,
                           kt_qweight** out);

/* The inverse of column shards: one weight whose columns are those of ws[0..count-1]
 * side by side (1 <= count <= 4; same bits, group size and rows), e.g. q|k|v or
 * gate|up projections fused into one matmul.  Bytes, scales and zeros equal the
 * quantization of the concatenated fp32 columns. */
kt_status kt_qweight_concat_columns(kt_ctx* ctx, const kt_qweight* const* ws, int32_t count, void* stream,
                                    kt_qweight** out);

/* One NCCL communicator per rank (one process per GPU).  NCCL is loaded at run
 * time (libnccl.so.2, or the file named by KT_NCCL_LIBRARY); without it these
 * return KT_ERR_NCCL.  Rank 0 makes the 128-byte id, every rank passes it to
 * kt_comm_init (which blocks until all nranks have joined).  Calls on one
 * communicator must be made in the same order on every rank, each rank on one
 * stream. */
typedef struct kt_comm kt_comm;
kt_status kt_comm_unique_id(void* id_out /* 128 bytes */);
kt_status kt_comm_init(kt_ctx* ctx, int32_t nranks, int32_t rank, const void* unique_id, kt_comm** out);
kt_status kt_comm_destroy(kt_comm* comm);

/* A communicator of nranks (2..8) in which only `rank` exists: no NCCL, every
 * rank's exchange area allocated on this GPU, the exchange ready at once.  A
 * row-parallel call whose exchange runs over peer memory (the fused m = 1
 * GEMV; the small-product exchange) stores its partials and then waits for
 * ranks that never arrive until the wait limit runs out
 * (kt_comm_set_wait_limit), sets the context error word and returns; the
 * context stays usable.  Calls that need NCCL (larger row-parallel products,
 * kt_allgather_columns, kt_argmax_column_parallel) fail with
 * KT_ERR_INVALID_ARGUMENT.  It exists to test the failure path of the fused
 * exchange on one GPU; it has no counterpart in the reference, whose
 * multi-rank path is not part of this library. */
kt_status kt_comm_init_detached(kt_ctx* ctx, int32_t nranks, int32_t rank, kt_comm** out);

/* Row-parallel multiplyQuantized: w_shard = kt_qweight_shard(W, axis 0, P, rank),
 * a_shard = the matching columns of a, contiguous [m x K_rank] on the device:
 *   c[m x N] = (accumulate ? c : 0) + alpha * sum_ranks a_shard . dequant(w_shard) + bias
 * on every rank (ncclAllReduce of the fp32 partial products, bias added once).
 * At m = 1 on INT4 shards the exchange runs inside the GEMV's epilogue over peer
 * memory (CUDA IPC areas set up on the first such call -- a collective -- and
 * agreed once per shard by every rank); KT_TP_FUSED=0 keeps the NCCL path.
 * Its waits for the other ranks are bounded: ranks that reach the same call more
 * than the communicator's wait limit apart (2 s unless kt_comm_set_wait_limit)
 * make it fail (context error word set, kt_ctx_take_error), where NCCL would
 * wait indefinitely; so does a rank whose flag shows a call other than this one.
 * After such a failure the ranks' call counters disagree: call
 * kt_comm_exchange_reset on every rank before the next fused call. */
kt_status kt_qmatmul_row_parallel(kt_ctx* ctx, kt_comm* comm, const kt_qweight* w_shard, const float* a_shard_dev,
                                  float* c_dev, int32_t m, int32_t accumulate, float alpha, const float* bias_dev,
                                  void* stream);

/* 1 in *ready once this communicator's peer-memory exchange areas are set up
 * and every rank agreed to use them (the fused m = 1 row-parallel GEMV), else 0. */
kt_status kt_comm_exchange_ready(const kt_comm* comm, int32_t* ready);

/* Limit, in seconds (0 < seconds <= 3600), of a fused row-parallel call's wait
 * for the other ranks' partials (no reference counterpart; default 2 s).
 * Applies to calls launched after it; the context's other bounded waits (TMA
 * copies inside a kernel) keep their 2 s limit. */
kt_status kt_comm_set_wait_limit(kt_comm* comm, double seconds);

/* Collective (every rank, same call order; no reference counterpart): waits
 * until this rank's device is idle, agrees with every rank that all are, zeroes
 * this rank's exchange area (call counter, flags, receive rows) and agrees
 * again, so the next fused call starts from the same call number everywhere.
 * Needed after a fused call failed (kt_ctx_take_error != 0); a no-op on a
 * communicator whose exchange is not set up, apart from the agreements. */
kt_status kt_comm_exchange_reset(kt_comm* comm, void* stream);

/* Column-parallel outputs (kt_qmatmul on w_shard = kt_qweight_shard(W, axis 1,
 * P, rank), equal widths n_shard = N / P) gathered into y_full [m x N] on every rank. */
kt_status kt_allgather_columns(kt_comm* comm, const float* y_shard_dev, float* y_full_dev, int32_t m,
                               int32_t n_shard, void* stream);

/* Greedy decoding over a column-parallel lm head (argmaxOfLastToken,
 * Transformer.kt:255-266, across shards): logits_shard_dev [rows x n_shard] holds
 * global columns [col_begin, col_begin + n_shard) of the logits on this rank;
 * out_dev[row] (device int32) receives, on every rank, the column of the largest
 * logit above -1e9 over all ranks, the lowest column among equal ones, 0 if none
 * -- what kt_argmax gives on the whole row.  One ncclAllGather of rows x 8 bytes. */
kt_status kt_argmax_column_parallel(kt_comm* comm, const float* logits_shard_dev, int32_t rows, int32_t n_shard,
                                    int32_t col_begin, int32_t* out_dev, void* stream);

/* QuantizedTensor.dequantize(), QuantizedTensor.kt:243-249: out_dev fp32 [rows x columns]. */
kt_status kt_dequantize(kt_ctx* ctx, const kt_qweight* w, float* out_dev, void* stream);

/* QuantizedTensor.dequantizeRow(row, dest) for `count` rows gathered by index
 * (the quantized-embedding lookup, Embedding.kt:96-101): out_dev [count x columns].
 * Row indices out of range set KT_ERR_INVALID_ARGUMENT in *status_dev (device
 * int32, may be NULL) and leave that output row untouched. */
kt_status kt_dequantize_rows(kt_ctx* ctx, const kt_qweight* w, const int32_t* rows_dev, int32_t count,
                             float* out_dev, int32_t* status_dev, void* stream);

/* ------------------------------------------------------------ matmul */

/* MatMul.multiplyQuantized(a, W, c, m, accumulate, alpha), MatMul.kt:460-486,
 * followed by QuantizedLinear's `+ bias` (QuantizedLinear.kt:18-25):
 *   c[m x N] = (accumulate ? c : 0) + alpha * a[m x K] . dequant(W) + bias
 * bias_dev (fp32 [N]) may be NULL.  m == 0 is a no-op.  Device pointers.
 * Tolerance against the reference fp32 result: 1e-3 relative to max|c| on the
 * fp32-accumulate kernels (m <= 8), 2e-2 on the bf16 tensor-core kernel (m >= 9). */
kt_status kt_qmatmul(kt_ctx* ctx, const kt_qweight* w, const float* a_dev, float* c_dev, int32_t m,
                     int32_t accumulate, float alpha, const float* bias_dev, void* stream);

/* kt_qmatmul for callers that must not have the library allocate device
 * memory (no counterpart in the reference, whose MatMul works in host
 * memory): a decode loop on a fixed memory budget, or a host runtime that
 * accounts for every device byte itself.  The same kernels as kt_qmatmul for
 * every m, with bit-identical results; their scratch (split-K counters and
 * partial tiles of the INT4 tensor-core GEMVs, the bf16 activations and split-K
 * partials of the tcgen05 GEMM) is a 16 MiB array inside the library image
 * instead of a buffer allocated on first use.  The first call on a device
 * looks up that array's address: make it before capturing a stream.  One array
 * per device: calls that overlap in time on a device race on it, so order them
 * on one stream.  Shapes whose scratch exceeds 16 MiB (e.g. the GEMM at
 * m x K > 8 Mi activations) return KT_ERR_INVALID_ARGUMENT; kt_qmatmul takes them. */
kt_status kt_qmatmul_noalloc(kt_ctx* ctx, const kt_qweight* w, const float* a_dev, float* c_dev, int32_t m,
                             int32_t accumulate, float alpha, const float* bias_dev, void* stream);

/* Which kernel family kt_qmatmul runs for this weight and m (for a 16-byte
 * aligned a), and so which tolerance applies: KT_PATH_GEMV (fp32 CUDA-core
 * streaming kernel), KT_PATH_GENERIC (fp32 kernel for unaligned shapes),
 * KT_PATH_TENSOR_CORE (bf16 tcgen05 kernel, 2e-2), KT_PATH_GEMV_MMA (INT4
 * m <= 8, INT8 m = 1: exact integer weights on tensor cores with x as three
 * integer parts (m = 1) or two fp16 terms (m >= 2; m = 5..8 as two groups of
 * tokens in one launch), fp32 group combine, 1e-3). */
enum { KT_PATH_GEMV = 0, KT_PATH_GENERIC = 1, KT_PATH_TENSOR_CORE = 2, KT_PATH_GEMV_MMA = 3 };
kt_status kt_qmatmul_path(const kt_qweight* w, int32_t m, int32_t* path_out);
/* The same for kt_qmatmul_t: KT_PATH_TENSOR_CORE (bf16 tcgen05, 2e-2) or
 * KT_PATH_GENERIC (fp32 CUDA cores, 1e-3). */
kt_status kt_qmatmul_t_path(const kt_qweight* w, int32_t m, int32_t* path_out);

/* Pins the number of K-splits per column tile (>= 1; raised to the minimum
 * the shape needs) of the INT4 tensor-core GEMV; 0 restores the built-in
 * choice (no reference counterpart). */
kt_status kt_set_gemv_mma_tuning(int32_t k_splits);

/* Pins the launch shape of the fp32 streaming kernel (no reference counterpart;
 * the reference's knobs are MatMul.numThreads / parallelThreshold,
 * MatMul.kt:30-43): packed bytes per lane and row (4, 8 or 16) and CTAs per
 * thread-block cluster along K (1..8).  0 restores the built-in choice for that
 * field.  Process-wide; results stay within the same tolerance for every
 * setting. */
kt_status kt_set_gemv_tuning(int32_t lane_bytes, int32_t cluster_k);

/* Reads and clears the context's sticky device error word (no reference
 * counterpart): non-zero means a kernel's bounded wait on a TMA transfer ran
 * out of time and that call's output is not valid.  Synchronizes the device. */
kt_status kt_ctx_take_error(kt_ctx* ctx, int32_t* error_out);

/* The literal FloatArray signature: host a / c / bias, copied through the
 * context's staging buffers on its own stream.  Synchronous. */
kt_status kt_qmatmul_host(kt_ctx* ctx, const kt_qweight* w, const float* a_host, float* c_host, int32_t m,
                          int32_t accumulate, float alpha, const float* bias_host);

/* MatMul.multiplyByQuantizedTransposed(dy, W, dx, m, accumulate), MatMul.kt:954-981:
 *   dx[m x K] = (accumulate ? dx : 0) + dy[m x N] . dequant(W)^T        (device pointers)
 * At m >= 16, INT4 with N % 128 == 0 or INT8 with N % 64 == 0 (group size 32, 64
 * or a multiple of 128) runs on the bf16 tcgen05 tensor cores (tolerance 2e-2 of
 * max|dx|); every other case on the fp32 CUDA-core kernels (1e-3).
 * kt_qmatmul_t_path tells which. */
kt_status kt_qmatmul_t(kt_ctx* ctx, const kt_qweight* w, const float* dy_dev, float* dx_dev, int32_t m,
                       int32_t accumulate, void* stream);

/* ------------------------------------------------------------ decode step
 * The device-resident pieces of Transformer.decode around the quantized
 * matmul (Transformer.kt:141-154, TransformerBlock.kt:40-47,
 * Attention.kt:207-239 and :295-328).  Positions and token ids are read from
 * device memory so that a whole step can be captured into a CUDA graph.
 * KV cache layout is the reference's (KVCache.kt:3-59): fp32
 * [layers][kv_heads][max_seq][head_dim] for keys and for values. */

/* RMSNorm.forwardInto (RMSNorm.kt:71-90), `rows` rows of `dim`. */
kt_status kt_rmsnorm(kt_ctx* ctx, const float* x_dev, const float* weight_dev, float* out_dev, int32_t rows,
                     int32_t dim, float eps, void* stream);
/* RoPE.applyInPlace / applyRowsInPlace (RoPE.kt:117-155): row r of v [rows x width]
 * at position *position_dev + r, heads of head_dim, pairs (i, i + head_dim/2),
 * inv_freq_dev [head_dim/2] as RoPE.invFreq (RoPE.kt:39-42, Llama-3 scaling included). */
kt_status kt_rope(kt_ctx* ctx, float* v_dev, int32_t rows, int32_t width, int32_t head_dim, const float* inv_freq_dev,
                  const int32_t* position_dev, void* stream);
/* The cache writes of Attention.decodeInto / prefillInto (Attention.kt:225-232). */
kt_status kt_kv_store(kt_ctx* ctx, const float* k_dev, const float* v_dev, float* k_cache, float* v_cache,
                      int32_t rows, int32_t kv_heads, int32_t head_dim, int32_t max_seq, int32_t layer,
                      const int32_t* position_dev, void* stream);
/* attendHead for every query head of `rows` tokens, row t at position *position_dev + t
 * attending to positions 0..that position (Attention.kt:295-328; rows > 1 is the
 * causal prefill of Attention.prefillInto, Attention.kt:241-293):
 * scores (dot * scale) over positions 0..pos, softmax from the reference's -1e9
 * initial maximum, context = weighted sum of values (split over blocks of 64
 * positions and merged with a log-sum-exp in block order).  scores_dev: scratch of
 * kt_attention_scratch_floats(rows, heads, head_dim, max_seq) floats; head_dim <= 254.
 * q_dev: rows q_stride floats apart (a fused q|k|v row is wider than the q part);
 * context_dev: [rows x heads*head_dim]. */
size_t kt_attention_scratch_floats(int32_t rows, int32_t heads, int32_t head_dim, int32_t max_seq);
/* The same for rows of several sequences (batched decode and prefill): row r
 * belongs to sequence r / rows_per_seq, whose caches start cache_stride floats
 * after the previous sequence's, and sits at position *position_dev +
 * r % rows_per_seq.  rows is a multiple of rows_per_seq. */
kt_status kt_attention_seqs(kt_ctx* ctx, const float* q_dev, const float* k_cache, const float* v_cache,
                            float* context_dev, float* scores_dev, int32_t rows, int32_t q_stride, int32_t heads,
                            int32_t kv_heads, int32_t head_dim, int32_t max_seq, int32_t layer, float scale,
                            const int32_t* position_dev, int32_t rows_per_seq, int64_t cache_stride, void* stream);
kt_status kt_attention_decode(kt_ctx* ctx, const float* q_dev, const float* k_cache, const float* v_cache,
                              float* context_dev, float* scores_dev, int32_t rows, int32_t q_stride, int32_t heads,
                              int32_t kv_heads, int32_t head_dim, int32_t max_seq, int32_t layer, float scale,
                              const int32_t* position_dev, void* stream);
/* SwiGLU.forwardInto (SwiGLU.kt:19-25) over a fused gate | up weight W
 * [K x 2H] (gate columns, then up columns; kt_qweight_concat_columns):
 *   act[m x H] = silu(g) * u,  [g | u] = alpha * a[m x K] . dequant(W) + bias
 * Where the m = 1 INT4 GEMV takes the weight, silu(g) * u is formed in its
 * epilogue (gate column j and up column H + j are the two nibbles of byte j of
 * the split-half packing) and gu_dev is not touched; elsewhere the product goes
 * through gu_dev ([m x 2H], may be NULL only on the fused path) and a separate
 * kernel.  Same results as kt_qmatmul followed by kt_silu_mul_rows. */
kt_status kt_qmatmul_swiglu(kt_ctx* ctx, const kt_qweight* w, const float* a_dev, float* gu_dev, float* act_dev,
                            int32_t m, float alpha, const float* bias_dev, void* stream);
/* RMSNorm.forwardInto (RMSNorm.kt:71-90) followed by a projection, the start
 * of both halves of TransformerBlock.decodeInto (TransformerBlock.kt:40-47):
 *   c[m x N] = (accumulate ? c : 0) + RMSNorm(x)[m x K] . dequant(W) + bias
 * with RMSNorm(x) = x * (1 / sqrt(mean(x^2) + eps)) * norm_weight per row.
 * Where an INT4 GEMV takes the weight (m = 1, or m = 2..8 with x_dev 16-byte
 * aligned; norm_weight_dev 16-byte aligned) the norm is applied while the GEMV
 * stages x -- every CTA sums the rows' squares itself -- and xn_dev is not
 * touched; elsewhere kt_rmsnorm writes xn_dev ([m x K], may be NULL only on
 * the fused path), then kt_qmatmul.  Within the fp32 tolerance of the two
 * calls. */
kt_status kt_rmsnorm_qmatmul(kt_ctx* ctx, const kt_qweight* w, const float* x_dev, const float* norm_weight_dev,
                             float eps, float* xn_dev, float* c_dev, int32_t m, int32_t accumulate,
                             const float* bias_dev, void* stream);
/* The same followed by SwiGLU over a gate | up weight (kt_qmatmul_swiglu):
 * act[m x H] = silu(g) * u, [g | u] = RMSNorm(x) . dequant(W) + bias; both the
 * norm and silu(g) * u fused into the m = 1 INT4 GEMV where it applies, the
 * norm alone into the m = 2..8 one (gu_dev then receives [g | u]). */
kt_status kt_rmsnorm_qmatmul_swiglu(kt_ctx* ctx, const kt_qweight* w, const float* x_dev,
                                    const float* norm_weight_dev, float eps, float* xn_dev, float* gu_dev,
                                    float* act_dev, int32_t m, const float* bias_dev, void* stream);
/* One decode token per sequence, the middle of Attention.decodeInto
 * (Attention.kt:207-239) in one launch: for fused q|k|v rows (row r = sequence
 * r, whose caches start cache_stride floats after the previous sequence's, at
 * position *position_dev) RoPE of the query and key heads (RoPE.kt:117-137),
 * key and value into the cache (Attention.kt:225-232), attendHead for every
 * query head (Attention.kt:295-328) and the merge of the position blocks --
 * kt_rope_kv_seqs followed by kt_attention_seqs at rows_per_seq = 1, with the
 * query rotated in registers (qkv_dev is not written).  scratch_dev: the
 * kt_attention_scratch_floats(rows, heads, head_dim, max_seq) floats of the
 * attention, zero-filled before the first call (its last rows x heads words
 * are merge counters that every call leaves at zero).  heads / kv_heads <= 8,
 * head_dim 64 or 128, max_seq <= 16384, else KT_ERR_UNSUPPORTED. */
kt_status kt_attention_rope_decode(kt_ctx* ctx, const float* qkv_dev, int32_t rows, int32_t q_width, int32_t heads,
                                   int32_t kv_heads, int32_t head_dim, const float* inv_freq_dev, float* k_cache,
                                   float* v_cache, float* context_dev, float* scratch_dev, int32_t max_seq,
                                   int32_t layer, float scale, const int32_t* position_dev, int64_t cache_stride,
                                   void* stream);
/* gate = silu(gate) * up (SwiGLU.forwardInto, Tensor.kt:231-237). */
kt_status kt_silu_mul(kt_ctx* ctx, float* gate_dev, const float* up_dev, int64_t n, void* stream);
/* x += y, then out = RMSNorm(x) with `weight` (the residual add of
 * TransformerBlock.decodeInto fused with the norm that follows it). */
kt_status kt_add_rmsnorm(kt_ctx* ctx, float* x_dev, const float* y_dev, const float* weight_dev, float* out_dev,
                         int32_t rows, int32_t dim, float eps, void* stream);
/* RoPE on the q and k parts of fused q|k|v rows (widths q_width and
 * kv_heads*head_dim; row r at position *position_dev + r), then k and v into the cache. */
kt_status kt_rope_kv(kt_ctx* ctx, float* qkv_dev, int32_t rows, int32_t q_width, int32_t kv_heads, int32_t head_dim,
                     const float* inv_freq_dev, float* k_cache, float* v_cache, int32_t max_seq, int32_t layer,
                     const int32_t* position_dev, void* stream);
/* kt_rope_kv for rows of several sequences (row r: sequence r / rows_per_seq at
 * position *position_dev + r % rows_per_seq, caches cache_stride floats apart). */
kt_status kt_rope_kv_seqs(kt_ctx* ctx, float* qkv_dev, int32_t rows, int32_t q_width, int32_t kv_heads,
                          int32_t head_dim, const float* inv_freq_dev, float* k_cache, float* v_cache, int32_t max_seq,
                          int32_t layer, const int32_t* position_dev, int32_t rows_per_seq, int64_t cache_stride,
                          void* stream);
/* out[t][j] = silu(gu[t][j]) * gu[t][hidden + j] for fused gate|up rows [rows x 2*hidden]. */
kt_status kt_silu_mul_rows(kt_ctx* ctx, const float* gu_dev, float* out_dev, int32_t rows, int32_t hidden,
                           void* stream);
/* x += y (Tensor.addInPlace). */
kt_status kt_add(kt_ctx* ctx, float* x_dev, const float* y_dev, int64_t n, void* stream);
/* argmaxOfLastToken per row (Transformer.kt:255-266): the largest logit above
 * -1e9, the lowest index among equal ones, 0 if none. */
kt_status kt_argmax(kt_ctx* ctx, const float* logits_dev, int32_t rows, int32_t n, int32_t* out_dev, void* stream);
/* QuantizedTensor.dequantizeColumn for `count` columns (the tied embedding lookup,
 * Embedding.kt:119-135): out_dev [count x rows]; an out-of-range column sets
 * KT_ERR_INVALID_ARGUMENT in *status_dev and leaves its output row untouched. */
kt_status kt_dequantize_column(kt_ctx* ctx, const kt_qweight* w, const int32_t* columns_dev, int32_t count,
                               float* out_dev, int32_t* status_dev, void* stream);
/* dst_dev[i] = src_dev[rows_dev[i]] for i < count, rows of `width` floats (e.g.
 * the last prompt row of every sequence before the head). */
kt_status kt_gather_rows(kt_ctx* ctx, const float* src_dev, const int32_t* rows_dev, int32_t count, int32_t width,
                         float* dst_dev, void* stream);
/* *value_dev += delta on `stream` (advances a captured step's position). */
kt_status kt_increment(kt_ctx* ctx, int32_t* value_dev, int32_t delta, void* stream);

/* ------------------------------------------------------------ LoRA adapters over a quantized base
 * LoRALinear (LoRA.kt:7-57) with a QuantizedLinear base: lora_a fp32 [K x rank],
 * lora_b fp32 [rank x N], scaling = alpha / rank, all row-major on the device;
 * 1 <= rank <= 256. */
/* projected[m x rank] = a[m x K] . lora_a (the low-rank projection of forwardInto). */
kt_status kt_lora_project(kt_ctx* ctx, const float* a_dev, int32_t m, int32_t k, const float* lora_a, int32_t rank,
                          float* projected_dev, void* stream);
/* LoRALinear.forwardInto (LoRA.kt:39-46): projected = a . A, then
 * c = (accumulate ? c : 0) + alpha * a . deq(W) + bias + scaling * projected . B,
 * the low-rank term added in the quantized matmul's own epilogue (no extra pass
 * over c).  `projected` [m x rank] is kept for the backward. */
kt_status kt_lora_qmatmul(kt_ctx* ctx, const kt_qweight* w, const float* a_dev, float* c_dev, int32_t m,
                          int32_t accumulate, float alpha, const float* bias_dev, const float* lora_a,
                          const float* lora_b, int32_t rank, float scaling, float* projected_dev, void* stream);
/* Gradients of LoRALinear.forward (LoRA.kt:31-36 through the autograd of
 * matmulDequant, Tensor.kt:171-177, and of its two matmuls).  With
 * G = dy . B^T [m x rank]:
 *   dx = (accumulate_dx ? dx : 0) + dy . deq(W)^T + scaling * G . A^T   (dx NULL: skipped)
 *   grad_a += scaling * a^T . G         [K x rank]                        (NULL: skipped)
 *   grad_b += scaling * projected^T . dy [rank x N]                       (NULL: skipped)
 * The base weight gets no gradient (frozen, LoRAAdapter, LoRA.kt:86-91). */
kt_status kt_lora_backward(kt_ctx* ctx, const kt_qweight* w, const float* a_dev, const float* dy_dev,
                           const float* projected_dev, const float* lora_a, const float* lora_b, int32_t rank,
                           float scaling, int32_t m, float* dx_dev, int32_t accumulate_dx, float* grad_a,
                           float* grad_b, void* stream);

/* fusedCrossEntropyLoss(hidden, head, targets, ignoreIndex) with a QuantizedLinear
 * head (Loss.kt:114-220): head = W [dim x vocab] with bias_dev [vocab] (NULL:
 * zero), hidden_dev fp32 [rows x dim], targets_host int32 [rows] in host
 * memory (ignore_index marks rows without a target; a target outside
 * 0..vocab-1 fails with the reference's message).  *loss_dev = mean over the
 * active rows of max + ln(sum exp) - logit[target] (0 with no active row, and
 * then no gradients).  With upstream gradient 1: hidden_grad_dev (NULL:
 * skipped) += the rows' gradients through the head (ignored rows untouched),
 * bias_grad_dev (NULL: skipped) += the column sums of the logit gradients.
 * Rows are processed in chunks of at most 2^26 logits; the logits come from
 * the same matmul paths as kt_qmatmul. */
kt_status kt_fused_cross_entropy(kt_ctx* ctx, const kt_qweight* head, const float* bias_dev, const float* hidden_dev,
                                 int32_t rows, const int32_t* targets_host, int32_t ignore_index, float* loss_dev,
                                 float* hidden_grad_dev, float* bias_grad_dev, void* stream);

/* ------------------------------------------------------------ safetensors files
 * The reference's model files (SafeTensors.kt:12-249, written by
 * Transformer.saveQuantized, Transformer.kt:402-431): an 8-byte little-endian
 * header length, a JSON header {name: {"dtype", "shape", "data_offsets"},
 * "__metadata__": {key: value}} padded with spaces to a multiple of 8 bytes,
 * then every tensor's bytes.  Parsing and writing run on the host (no GPU
 * needed for host data); tensor bytes move between the file and HBM through
 * two pinned staging buffers per file, so reading chunk i+1 from the file
 * overlaps the copy of chunk i.  A quantized weight is stored as
 * <name>.qweight (I8 for INT8, U8 for INT4) [K, bytesPerRow], <name>.scales
 * F32 [G, N] and, INT4 only, <name>.zeros U8 [G, N]. */
typedef struct kt_stfile kt_stfile;

typedef struct {
    char dtype[8];     /* "F32", "BF16", "U8", ... NUL-terminated */
    int32_t rank;      /* number of dimensions, at most 8 */
    int64_t shape[8];
    int64_t offset;    /* first byte, counted from the start of the data section */
    int64_t bytes;
} kt_st_entry_info;

/* SafeTensorsFile(file) (SafeTensors.kt:33-69): opens and parses the header;
 * KT_ERR_IO if the file cannot be read, KT_ERR_INVALID_ARGUMENT for a header
 * the reference rejects (length outside 1..100 MiB, not a JSON object, a
 * tensor without dtype or data_offsets, a data range past the end of file). */
kt_status kt_st_open(const char* path, kt_stfile** out);
/* close(): waits for copies in flight from or to this file's staging buffers. */
kt_status kt_st_close(kt_stfile* f);
/* names (header order) and entry(name); kt_st_entry fails for a missing name. */
int32_t kt_st_tensor_count(const kt_stfile* f);
const char* kt_st_tensor_name(const kt_stfile* f, int32_t index);  /* NULL when out of range */
kt_status kt_st_entry(const kt_stfile* f, const char* name, kt_st_entry_info* out);
/* metadata, in header order; the strings live until kt_st_close. */
int32_t kt_st_metadata_count(const kt_stfile* f);
kt_status kt_st_metadata_at(const kt_stfile* f, int32_t index, const char** key, const char** value);
/* readRaw(name, dest) (SafeTensors.kt:90-98): the tensor's bytes into host
 * memory of `capacity` bytes.  Synchronous. */
kt_status kt_st_read_raw(kt_stfile* f, const char* name, void* dst_host, int64_t capacity);
/* The tensor's bytes straight into device memory of `capacity` bytes, ordered
 * on `stream` (the host returns once the last chunk is queued). */
kt_status kt_st_read_raw_device(kt_ctx* ctx, kt_stfile* f, const char* name, void* dst_dev, int64_t capacity,
                                void* stream);
/* readInto(name, dest) (SafeTensors.kt:86-88, :110-170): the tensor as float32
 * into device memory of `capacity` floats, converted on the GPU from F32, F16,
 * BF16, F64, I8, U8, BOOL, I16, I32 or I64 with the reference's rounding
 * (round to nearest even for F64, I32 and I64; the others are exact). */
kt_status kt_st_read_f32_device(kt_ctx* ctx, kt_stfile* f, const char* name, float* dst_dev, int64_t capacity,
                                void* stream);
/* QuantizedTensor.mapFrom(reader, name) (QuantizedTensor.kt:109-126) into HBM:
 * a new device weight of the given quantization and shape from <name>.qweight,
 * <name>.scales and (INT4) <name>.zeros, with the reference's size checks. */
kt_status kt_qweight_load(kt_ctx* ctx, kt_stfile* f, const char* name, int32_t bits, int32_t group_size,
                          int32_t rows, int32_t columns, void* stream, kt_qweight** out);

/* One tensor to write: `data` is host memory, or device memory when on_device != 0. */
typedef struct {
    const char* name;
    const char* dtype;
    int32_t rank;
    const int64_t* shape;
    const void* data;
    int64_t bytes;
    int32_t on_device;
} kt_st_tensor;
/* SafeTensors.saveEntries(file, entries, metadata) (SafeTensors.kt:220-249):
 * the same bytes as the reference writes (header key order, JSON escaping,
 * space padding, data in entry order).  Device tensors are copied out on
 * `stream` through the staging buffers; ctx may be NULL when every tensor is
 * host memory.  Synchronous. */
kt_status kt_st_write(kt_ctx* ctx, const char* path, const kt_st_tensor* tensors, int32_t count,
                      const char* const* meta_keys, const char* const* meta_values, int32_t meta_count,
                      void* stream);

#ifdef __cplusplus
}
#endif
#endif /* KT_CUDA_H */
