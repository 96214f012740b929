// kt_tp.cu -- tensor parallelism over NCCL for the quantized matmul: one
// process per GPU, weights sharded with kt_qweight_shard (kt_shard.cu).
//
//   row-parallel    (split K, e.g. attention out / FFN down): each rank computes
//                   alpha * a[:, K_r] . W_r, the partial products are summed with
//                   ncclAllReduce, then c = (acc ? c : 0) + sum + bias on every rank.
//   column-parallel (split N, e.g. q/k/v, gate/up, lm head): each rank computes
//                   its columns with kt_qmatmul, no exchange; kt_allgather_columns
//                   assembles [m x N] when a rank needs the whole output.
//
// Row-parallel at m = 1 (decode) with INT4 shards runs one kernel per rank
// instead: the m = 1 GEMV with the exchange fused into its epilogue (one-shot
// all-reduce over peer memory, kt_gemv_imma.cu).  Each rank owns an exchange
// area -- receive rows [2][P][kTpNCap] of 64-bit words {call number, value} --
// mapped into every other rank's process with CUDA IPC (handles all-gathered
// through NCCL); the thread finishing an output column stores its word into
// every rank's area, then polls the column's word of every rank until each
// carries this call's number and sums the values in rank order.  Set up on the first such call (a collective:
// every rank takes part and all use the fused kernel or none), and agreed once
// per shard; KT_TP_FUSED=0 keeps the NCCL path.
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, or KT_NCCL_LIBRARY): the
// rest of the library does not depend on it.  Calls on one communicator must be
// issued in the same order on every rank, on one stream per rank.
#include <dlfcn.h>

#include <algorithm>
#include <vector>

#include <cstdlib>
#include <cstring>
#include <new>
#include <mutex>
#include <string>

#include "kt_device.cuh"
#include "kt_internal.h"

namespace {

// The few NCCL types and constants this file uses (nccl.h, NCCL 2.x ABI).
typedef struct ncclComm* ncclComm_t;
typedef struct {
    char internal[128];
} ncclUniqueId;
typedef int ncclResult_t;
constexpr int kNcclFloat32 = 7;
constexpr int kNcclSum = 0;

struct NcclApi {
    bool ok = false;
    std::string why;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, int, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, int, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        const char* names[] = {std::getenv("KT_NCCL_LIBRARY"), "libnccl.so.2", "libnccl.so"};
        void* h = nullptr;
        for (const char* n : names)
            if (n != nullptr && (h = dlopen(n, RTLD_NOW | RTLD_LOCAL)) != nullptr) break;
        if (h == nullptr) {
            api.why = "libnccl.so.2 not found (set KT_NCCL_LIBRARY)";
            return;
        }
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_reduce && api.all_gather &&
                 api.error_string;
        if (!api.ok) api.why = "libnccl.so.2 lacks an expected symbol";
    });
    return api;
}

kt_status fail_tp(kt_status st, const std::string& msg) {
    kt::set_error(msg);
    return st;
}

kt_status nccl_fail(ncclResult_t r, const char* what) {
    return fail_tp(KT_ERR_NCCL, std::string(what) + ": " + nccl().error_string(r));
}

// c = (accumulate ? c : 0) + sum + bias[col]
__global__ void row_parallel_epilogue_kernel(float* __restrict__ c, const float* __restrict__ sum,
                                             const float* __restrict__ bias, int64_t total, int32_t n,
                                             int32_t accumulate) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float r = sum[i] + (accumulate ? c[i] : 0.0f);
        if (bias != nullptr) r += bias[i % n];
        c[i] = r;
    }
}

// gathered [P][m][ns] -> y [m][P * ns]
__global__ void gather_columns_kernel(const float* __restrict__ gathered, float* __restrict__ y, int32_t parts,
                                      int32_t m, int32_t ns) {
    const int64_t total = static_cast<int64_t>(parts) * m * ns;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t p = i / (static_cast<int64_t>(m) * ns);
        const int64_t rem = i - p * m * ns;
        const int64_t t = rem / ns, j = rem - t * ns;
        y[t * parts * ns + p * ns + j] = gathered[i];
    }
}

int blocks_for(int64_t total) { return static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 16)); }

// Row-parallel above m = 1 (or on shards the fused GEMV does not take): the
// partial product sits in the communicator's scratch; one kernel exchanges it
// over peer memory the way the fused GEMV's epilogue does -- every thread
// stores {call number, value} words for its elements into every rank's receive
// row, then reads every rank's word of each of its elements in rank order until
// it carries this call's number (bounded; a later number fails at once) and
// writes c = sum + (accumulate ? c : 0) + bias -- and the grid's last CTA
// advances this rank's call counter.  The grid is small enough to be resident
// at once (a thread never waits for a CTA of its own grid).
struct LLExchange {
    unsigned long long* const* recv;  // [P] receive areas ([2][P][cap] words), mapped here
    uint32_t* state;                  // this rank's {calls completed, CTAs exited in this call}
    int32_t nranks, rank, cap;
    uint64_t wait_ns;
    int32_t* err;
};
__global__ void __launch_bounds__(256) ll_allreduce_kernel(const float* __restrict__ part, float* __restrict__ c,
                                                           const float* __restrict__ bias, int64_t total, int32_t n,
                                                           int32_t accumulate, LLExchange x) {
    const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(x.state) + 1u;
    const int64_t slot_base = static_cast<int64_t>(epoch & 1u) * x.nranks * x.cap;
    const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t first = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (int64_t i = first; i < total; i += step) {
        const unsigned long long word = (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(part[i]);
        for (int q = 0; q < x.nranks; ++q)
            kt::dev::st_relaxed_sys_u64(x.recv[q] + slot_base + static_cast<int64_t>(x.rank) * x.cap + i, word);
    }
    bool ok = true;
    for (int64_t i = first; i < total && ok; i += step) {
        const unsigned long long* mine = x.recv[x.rank] + slot_base + i;
        float sum = 0.0f;
        for (int src = 0; src < x.nranks && ok; ++src) {
            float v = 0.0f;
            ok = kt::dev::wait_word_sys(mine + static_cast<int64_t>(src) * x.cap, epoch, x.wait_ns, &v);
            sum += v;
        }
        if (ok) {
            float r = sum + (accumulate ? c[i] : 0.0f);
            if (bias != nullptr) r += bias[i % n];
            c[i] = r;
        }
    }
    if (!ok) atomicOr(x.err, 1);
    __syncthreads();  // every thread of the CTA has read this call's number
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(x.state + 1, 1u) == gridDim.x - 1) {  // the grid's last CTA
            x.state[1] = 0;
            x.state[0] += 1;
            __threadfence();
        }
    }
}

bool tp_ll_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("KT_TP_LL");
        return v == nullptr || std::atoi(v) != 0;
    }();
    return on;
}

// Greedy decoding over an lm head split along N (argmaxOfLastToken,
// Transformer.kt:255-266, kept across shards): per row the largest logit above
// -1e9 and, among equal ones, the lowest column.  Stage 1 on every rank: the
// best of its shard as the pair {value bits, global column} (column INT_MAX
// when no logit is above -1e9).  Stage 2, after an all-gather of the pairs:
// the ranks' pairs merged in rank order with the same rule, 0 when none.
constexpr int kArgmaxThreads = 256;
constexpr int32_t kNoColumn = 0x7fffffff;
__device__ __forceinline__ void better_pair(float& bv, int32_t& bi, float ov, int32_t oi) {
    if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
    }
}
__global__ void __launch_bounds__(kArgmaxThreads) shard_argmax_kernel(const float* __restrict__ logits, int32_t n_shard,
                                                                      int32_t col_begin, int32_t* __restrict__ pairs) {
    __shared__ float sv[kArgmaxThreads];
    __shared__ int32_t si[kArgmaxThreads];
    const int row = blockIdx.x;
    float best = -1e9f;
    int32_t idx = kNoColumn;
    for (int v = threadIdx.x; v < n_shard; v += kArgmaxThreads) {
        const float x = logits[static_cast<int64_t>(row) * n_shard + v];
        if (x > best) {  // strictly greater: the first (lowest) column of a tie stays
            best = x;
            idx = col_begin + v;
        }
    }
    sv[threadIdx.x] = best;
    si[threadIdx.x] = idx;
    __syncthreads();
    for (int st = kArgmaxThreads / 2; st > 0; st >>= 1) {
        if (threadIdx.x < st) better_pair(sv[threadIdx.x], si[threadIdx.x], sv[threadIdx.x + st], si[threadIdx.x + st]);
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        pairs[2 * row] = __float_as_int(sv[0]);
        pairs[2 * row + 1] = si[0];
    }
}
// gathered [P][rows][2] -> out[row]
__global__ void merge_argmax_kernel(const int32_t* __restrict__ gathered, int32_t parts, int32_t rows,
                                    int32_t* __restrict__ out) {
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= rows) return;
    float best = -1e9f;
    int32_t idx = kNoColumn;
    for (int p = 0; p < parts; ++p) {
        const int64_t o = (static_cast<int64_t>(p) * rows + row) * 2;
        better_pair(best, idx, __int_as_float(gathered[o]), gathered[o + 1]);
    }
    out[row] = idx == kNoColumn ? 0 : idx;
}

}  // namespace

constexpr int kTpMaxRanks = 8;
constexpr int32_t kTpNCap = 262144;    // words of a rank's receive row: m x N of one exchange

struct kt_comm {
    kt_ctx* ctx = nullptr;
    ncclComm_t comm = nullptr;
    int32_t nranks = 0, rank = 0;
    float* scratch = nullptr;  // partial sums / gathered columns, grown on demand
    size_t scratch_floats = 0;
    // exchange areas of the fused row-parallel GEMV
    int p2p_state = 0;                  // 0 not set up, 1 ready, 2 unavailable
    void* area = nullptr;               // this rank's area (cudaMalloc)
    void* peers[kTpMaxRanks] = {};      // every rank's area as mapped here (own at [rank])
    unsigned long long** d_recv = nullptr;  // device array of the P receive-area pointers
    uint64_t wait_ns = 2000000000ull;   // limit of a fused call's wait for the other ranks (2 s)
    bool detached = false;              // kt_comm_init_detached: no NCCL, every area local
};

namespace {

// Scratch of the communicator (calls on one communicator are ordered on one
// stream, so they may share it).  Allocation is not a stream operation; it is
// allowed in relaxed capture mode while that stream is being captured.
cudaError_t comm_scratch(kt_comm* c, size_t floats, float** out) {
    if (c->scratch_floats < floats) {
        cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
        cudaThreadExchangeStreamCaptureMode(&mode);
        float* p = nullptr;
        cudaError_t e = cudaMalloc(&p, floats * sizeof(float));
        cudaThreadExchangeStreamCaptureMode(&mode);
        if (e != cudaSuccess) return e;
        if (c->scratch != nullptr) {
            cudaDeviceSynchronize();  // queued collectives may still use the old buffer
            cudaFree(c->scratch);
        }
        c->scratch = p;
        c->scratch_floats = floats;
    }
    *out = c->scratch;
    return cudaSuccess;
}

size_t tp_recv_bytes(int P) { return static_cast<size_t>(2) * P * kTpNCap * sizeof(unsigned long long); }
// receive rows | this rank's own call counter and CTA exit count
size_t tp_area_bytes(int P) { return tp_recv_bytes(P) + 16; }

bool tp_fused_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("KT_TP_FUSED");
        return v == nullptr || std::atoi(v) != 0;
    }();
    return on;
}

// Every rank's agreement on a local yes / no (sum of ones over NCCL).
kt_status all_agree(kt_comm* c, bool mine, cudaStream_t s, bool* all) {
    if (c->detached) {  // the ranks that never run take this rank's answer
        *all = mine;
        return KT_OK;
    }
    float* f = nullptr;
    cudaError_t e = comm_scratch(c, 1, &f);
    if (e != cudaSuccess) return fail_tp(KT_ERR_OUT_OF_MEMORY, std::string("TP scratch: ") + cudaGetErrorString(e));
    const float one = mine ? 1.0f : 0.0f;
    e = cudaMemcpyAsync(f, &one, sizeof(float), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return fail_tp(KT_ERR_CUDA, std::string("agreement copy: ") + cudaGetErrorString(e));
    const ncclResult_t r = nccl().all_reduce(f, f, 1, kNcclFloat32, kNcclSum, c->comm, s);
    if (r != 0) return nccl_fail(r, "ncclAllReduce (agreement)");
    float sum = 0.0f;
    e = cudaMemcpyAsync(&sum, f, sizeof(float), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail_tp(KT_ERR_CUDA, std::string("agreement copy: ") + cudaGetErrorString(e));
    *all = sum == static_cast<float>(c->nranks);
    return KT_OK;
}

void release_p2p(kt_comm* c) {
    for (int q = 0; q < c->nranks && q < kTpMaxRanks; ++q)
        if (q != c->rank && c->peers[q] != nullptr) {
            if (c->detached) cudaFree(c->peers[q]);  // allocated here, not mapped
            else cudaIpcCloseMemHandle(c->peers[q]);
        }
    cudaFree(c->area);
    cudaFree(c->d_recv);
    c->area = nullptr;
    c->d_recv = nullptr;
    for (void*& p : c->peers) p = nullptr;
    cudaGetLastError();
}

// Collective: every rank allocates and zeroes its area, the IPC handles are
// all-gathered through NCCL, every rank maps the others', and all of them
// agree (or none uses the fused path).
kt_status setup_p2p(kt_comm* c, cudaStream_t s) {
    const int P = c->nranks;
    bool ok = P <= kTpMaxRanks;
    cudaIpcMemHandle_t mine{};
    const size_t bytes = tp_area_bytes(std::min(P, kTpMaxRanks));
    if (ok) ok = cudaMalloc(&c->area, bytes) == cudaSuccess;
    if (ok) ok = cudaMemset(c->area, 0, bytes) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
    if (ok) ok = cudaIpcGetMemHandle(&mine, c->area) == cudaSuccess;
    cudaGetLastError();
    // handles: 64 bytes = 16 32-bit words per rank (a float32 all-gather copies bits)
    constexpr int kWords = sizeof(cudaIpcMemHandle_t) / 4;
    static_assert(sizeof(cudaIpcMemHandle_t) % 4 == 0, "IPC handle size");
    float* f = nullptr;
    cudaError_t e = comm_scratch(c, static_cast<size_t>(kWords) * (P + 1), &f);
    if (e != cudaSuccess) return fail_tp(KT_ERR_OUT_OF_MEMORY, std::string("TP scratch: ") + cudaGetErrorString(e));
    e = cudaMemcpyAsync(f, &mine, sizeof(mine), cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return fail_tp(KT_ERR_CUDA, std::string("IPC handle copy: ") + cudaGetErrorString(e));
    const ncclResult_t r = nccl().all_gather(f, f + kWords, kWords, kNcclFloat32, c->comm, s);
    if (r != 0) return nccl_fail(r, "ncclAllGather (IPC handles)");
    std::vector<cudaIpcMemHandle_t> all(P);
    e = cudaMemcpyAsync(all.data(), f + kWords, sizeof(cudaIpcMemHandle_t) * P, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail_tp(KT_ERR_CUDA, std::string("IPC handle copy: ") + cudaGetErrorString(e));
    if (ok) {
        c->peers[c->rank] = c->area;
        for (int q = 0; q < P && ok; ++q)
            if (q != c->rank)
                ok = cudaIpcOpenMemHandle(&c->peers[q], all[q], cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    }
    if (ok) {
        unsigned long long* recv[kTpMaxRanks];
        for (int q = 0; q < P; ++q) recv[q] = static_cast<unsigned long long*>(c->peers[q]);
        ok = cudaMalloc(&c->d_recv, sizeof(unsigned long long*) * P) == cudaSuccess &&
             cudaMemcpy(c->d_recv, recv, sizeof(unsigned long long*) * P, cudaMemcpyHostToDevice) == cudaSuccess;
    }
    cudaGetLastError();
    bool every = false;
    const kt_status st = all_agree(c, ok, s, &every);
    if (st != KT_OK) return st;
    if (!every) release_p2p(c);
    c->p2p_state = every ? 1 : 2;
    return KT_OK;
}

}  // namespace

extern "C" {

kt_status kt_comm_unique_id(void* id_out) {
    if (!id_out) return fail_tp(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    const NcclApi& api = nccl();
    if (!api.ok) return fail_tp(KT_ERR_NCCL, api.why);
    ncclUniqueId id;
    const ncclResult_t r = api.get_unique_id(&id);
    if (r != 0) return nccl_fail(r, "ncclGetUniqueId");
    std::memcpy(id_out, &id, sizeof(id));
    return KT_OK;
}

kt_status kt_comm_init(kt_ctx* ctx, int32_t nranks, int32_t rank, const void* unique_id, kt_comm** out) {
    if (!ctx || !unique_id || !out) return fail_tp(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    if (nranks <= 0 || rank < 0 || rank >= nranks)
        return fail_tp(KT_ERR_INVALID_ARGUMENT, "rank " + std::to_string(rank) + " of " + std::to_string(nranks));
    const NcclApi& api = nccl();
    if (!api.ok) return fail_tp(KT_ERR_NCCL, api.why);
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return fail_tp(KT_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof(id));
    auto* c = new (std::nothrow) kt_comm();
    if (!c) return fail_tp(KT_ERR_OUT_OF_MEMORY, "host allocation failed");
    const ncclResult_t r = api.comm_init_rank(&c->comm, nranks, id, rank);
    if (r != 0) {
        delete c;
        return nccl_fail(r, "ncclCommInitRank");
    }
    c->ctx = ctx;
    c->nranks = nranks;
    c->rank = rank;
    *out = c;
    return KT_OK;
}

// Only `rank` of nranks exists: every rank's exchange area is allocated and
// zeroed on this GPU, so the fused exchange is ready without a collective and
// its waits for the absent ranks run into the wait limit.
kt_status kt_comm_init_detached(kt_ctx* ctx, int32_t nranks, int32_t rank, kt_comm** out) {
    if (!ctx || !out) return fail_tp(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    if (nranks < 2 || nranks > kTpMaxRanks || rank < 0 || rank >= nranks)
        return fail_tp(KT_ERR_INVALID_ARGUMENT, "rank " + std::to_string(rank) + " of " + std::to_string(nranks) +
                                                    " (a detached communicator has 2.." +
                                                    std::to_string(kTpMaxRanks) + " ranks)");
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return fail_tp(KT_ERR_CUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
    auto* c = new (std::nothrow) kt_comm();
    if (!c) return fail_tp(KT_ERR_OUT_OF_MEMORY, "host allocation failed");
    c->ctx = ctx;
    c->nranks = nranks;
    c->rank = rank;
    c->detached = true;
    const size_t bytes = tp_area_bytes(nranks);
    unsigned long long* recv[kTpMaxRanks] = {};
    for (int q = 0; q < nranks && e == cudaSuccess; ++q) {
        e = cudaMalloc(&c->peers[q], bytes);
        if (e == cudaSuccess) e = cudaMemset(c->peers[q], 0, bytes);
        recv[q] = static_cast<unsigned long long*>(c->peers[q]);
    }
    c->area = c->peers[rank];
    if (e == cudaSuccess) e = cudaMalloc(&c->d_recv, sizeof(unsigned long long*) * nranks);
    if (e == cudaSuccess)
        e = cudaMemcpy(c->d_recv, recv, sizeof(unsigned long long*) * nranks, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        for (void* p : c->peers) cudaFree(p);
        cudaFree(c->d_recv);
        cudaGetLastError();
        delete c;
        return fail_tp(KT_ERR_OUT_OF_MEMORY, std::string("exchange areas: ") + cudaGetErrorString(e));
    }
    c->p2p_state = 1;
    *out = c;
    return KT_OK;
}

kt_status kt_comm_destroy(kt_comm* c) {
    if (!c) return KT_OK;
    cudaSetDevice(c->ctx->device);
    cudaDeviceSynchronize();
    // Peers wrote into this rank's area only inside calls this rank also made,
    // before raising the flags its kernels waited for: nothing is in flight now.
    if (c->p2p_state == 1) release_p2p(c);
    if (c->comm != nullptr) nccl().comm_destroy(c->comm);
    cudaFree(c->scratch);
    delete c;
    return KT_OK;
}

kt_status kt_qmatmul_row_parallel(kt_ctx* ctx, kt_comm* comm, const kt_qweight* w_shard, const float* a_shard,
                                  float* c, int32_t m, int32_t accumulate, float alpha, const float* bias,
                                  void* stream) {
    if (!ctx || !comm || !w_shard) return fail_tp(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (m < 0) return fail_tp(KT_ERR_INVALID_ARGUMENT, "Negative row count " + std::to_string(m));
    if (m == 0) return KT_OK;
    if (!a_shard || !c) return fail_tp(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (m == 1 && tp_fused_enabled()) {
        // decided once per shard with every rank (collective, same call order everywhere)
        kt_qweight* w = const_cast<kt_qweight*>(w_shard);
        if (w->tp_fused == 0 || w->tp_comm != comm) {
            if (comm->p2p_state == 0) {
                const kt_status st = setup_p2p(comm, s);
                if (st != KT_OK) return st;
            }
            const kt::QView v = kt::view(w);
            const bool mine = comm->p2p_state == 1 && w->columns <= kTpNCap &&
                              kt::gemv_imma_tp_supported(v, ctx->sm_count);
            bool every = false;
            const kt_status st = all_agree(comm, mine, s, &every);
            if (st != KT_OK) return st;
            w->tp_fused = every ? 1 : 2;
            w->tp_comm = comm;
        }
        if (w->tp_fused == 1) {
            const kt::QView v = kt::view(w);
            const float* a = a_shard;
            if (reinterpret_cast<uintptr_t>(a) % 16 != 0) {  // the kernel loads x in 16-byte vectors
                float* copy = nullptr;
                cudaError_t e = comm_scratch(comm, static_cast<size_t>(w->rows) + 4, &copy);
                if (e == cudaSuccess)
                    e = cudaMemcpyAsync(copy, a_shard, sizeof(float) * w->rows, cudaMemcpyDeviceToDevice, s);
                if (e != cudaSuccess) return fail_tp(KT_ERR_CUDA, std::string("x copy: ") + cudaGetErrorString(e));
                a = copy;
            }
            kt::MatmulArgs args{a, c, bias, 1, accumulate, alpha, ctx->d_error};
            args.tp.recv = comm->d_recv;
            args.tp.nranks = comm->nranks;
            args.tp.rank = comm->rank;
            args.tp.n_cap = kTpNCap;
            args.tp.wait_ns = comm->wait_ns;
            args.tp.state = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(comm->area) +
                                                        tp_recv_bytes(comm->nranks));
            const size_t need = kt::gemv_imma_workspace_bytes(v, ctx->sm_count, true);
            void* ws = nullptr;
            cudaError_t e = cudaSuccess;
            if (need > 0) e = kt::stream_workspace(ctx, s, need, &ws);
            if (e == cudaSuccess) e = kt::launch_gemv_imma(v, args, ctx->sm_count, s, ws, need);
            if (e != cudaSuccess) return fail_tp(KT_ERR_CUDA, std::string("fused row-parallel GEMV: ") + cudaGetErrorString(e));
            return KT_OK;
        }
    }
    const int64_t total = static_cast<int64_t>(m) * w_shard->columns;
    if (tp_fused_enabled() && tp_ll_enabled() && total <= kTpNCap && comm->p2p_state != 2) {
        if (comm->p2p_state == 0) {  // collective, same call order everywhere
            const kt_status st = setup_p2p(comm, s);
            if (st != KT_OK) return st;
        }
        if (comm->p2p_state == 1) {
            float* part = nullptr;
            cudaError_t e = comm_scratch(comm, static_cast<size_t>(total), &part);
            if (e != cudaSuccess)
                return fail_tp(KT_ERR_OUT_OF_MEMORY, std::string("TP scratch: ") + cudaGetErrorString(e));
            kt_status st = kt::run_qmatmul(ctx, w_shard, a_shard, part, m, 0, alpha, nullptr, s);
            if (st != KT_OK) return st;
            LLExchange x{comm->d_recv,
                         reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(comm->area) + tp_recv_bytes(comm->nranks)),
                         comm->nranks, comm->rank, kTpNCap, comm->wait_ns, ctx->d_error};
            const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, ctx->sm_count));
            ll_allreduce_kernel<<<blocks, 256, 0, s>>>(part, c, bias, total, w_shard->columns, accumulate, x);
            e = cudaGetLastError();
            if (e != cudaSuccess) return fail_tp(KT_ERR_CUDA, std::string("exchange: ") + cudaGetErrorString(e));
            return KT_OK;
        }
    }
    if (comm->detached) return fail_tp(KT_ERR_INVALID_ARGUMENT, "a detached communicator has no collective");
    float* sum = nullptr;
    cudaError_t e = comm_scratch(comm, static_cast<size_t>(total), &sum);
    if (e != cudaSuccess) return fail_tp(KT_ERR_OUT_OF_MEMORY, std::string("TP scratch: ") + cudaGetErrorString(e));
    // partial = alpha * a_shard . W_shard
    kt_status st = kt::run_qmatmul(ctx, w_shard, a_shard, sum, m, 0, alpha, nullptr, s);
    if (st != KT_OK) return st;
    const ncclResult_t r = nccl().all_reduce(sum, sum, static_cast<size_t>(total), kNcclFloat32, kNcclSum, comm->comm, s);
    if (r != 0) return nccl_fail(r, "ncclAllReduce");
    row_parallel_epilogue_kernel<<<blocks_for(total), 256, 0, s>>>(c, sum, bias, total, w_shard->columns, accumulate);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_tp(KT_ERR_CUDA, std::string("row-parallel epilogue: ") + cudaGetErrorString(e));
    return KT_OK;
}

kt_status kt_allgather_columns(kt_comm* comm, const float* y_shard, float* y_full, int32_t m, int32_t n_shard,
                               void* stream) {
    if (!comm || !y_shard || !y_full) return fail_tp(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (m <= 0 || n_shard <= 0) return fail_tp(KT_ERR_INVALID_ARGUMENT, "empty shard");
    if (comm->detached) return fail_tp(KT_ERR_INVALID_ARGUMENT, "a detached communicator has no collective");
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t per = static_cast<int64_t>(m) * n_shard;
    float* gathered = nullptr;
    cudaError_t e = comm_scratch(comm, static_cast<size_t>(per * comm->nranks), &gathered);
    if (e != cudaSuccess) return fail_tp(KT_ERR_OUT_OF_MEMORY, std::string("TP scratch: ") + cudaGetErrorString(e));
    const ncclResult_t r = nccl().all_gather(y_shard, gathered, static_cast<size_t>(per), kNcclFloat32, comm->comm, s);
    if (r != 0) return nccl_fail(r, "ncclAllGather");
    gather_columns_kernel<<<blocks_for(per * comm->nranks), 256, 0, s>>>(gathered, y_full, comm->nranks, m, n_shard);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_tp(KT_ERR_CUDA, std::string("gather columns: ") + cudaGetErrorString(e));
    return KT_OK;
}

kt_status kt_comm_set_wait_limit(kt_comm* comm, double seconds) {
    if (!comm) return fail_tp(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (!(seconds > 0.0) || seconds > 3600.0)
        return fail_tp(KT_ERR_INVALID_ARGUMENT, "wait limit must be in (0, 3600] seconds");
    comm->wait_ns = static_cast<uint64_t>(seconds * 1e9);
    return KT_OK;
}

// Collective: after a fused call timed out, the ranks' call counters and flags
// disagree.  Every rank waits for its own work, all ranks agree that they are
// idle, each zeroes its exchange area (counters, flags, receive rows), and a
// second agreement makes sure no rank starts a call before every area is clear.
kt_status kt_comm_exchange_reset(kt_comm* comm, void* stream) {
    if (!comm) return fail_tp(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSetDevice(comm->ctx->device);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return fail_tp(KT_ERR_CUDA, std::string("exchange reset: ") + cudaGetErrorString(e));
    bool every = false;
    kt_status st = all_agree(comm, true, s, &every);
    if (st != KT_OK) return st;
    if (comm->p2p_state == 1) {
        // a detached communicator clears every area (all of them are written here)
        for (int q = 0; q < comm->nranks && e == cudaSuccess; ++q)
            if (q == comm->rank || comm->detached)
                e = cudaMemsetAsync(comm->peers[q], 0, tp_area_bytes(comm->nranks), s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return fail_tp(KT_ERR_CUDA, std::string("exchange reset: ") + cudaGetErrorString(e));
    }
    return all_agree(comm, true, s, &every);
}

kt_status kt_comm_exchange_ready(const kt_comm* comm, int32_t* ready) {
    if (!comm || !ready) return fail_tp(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    *ready = comm->p2p_state == 1 ? 1 : 0;
    return KT_OK;
}

kt_status kt_argmax_column_parallel(kt_comm* comm, const float* logits_shard, int32_t rows, int32_t n_shard,
                                    int32_t col_begin, int32_t* out, void* stream) {
    if (!comm || !logits_shard || !out) return fail_tp(KT_ERR_INVALID_ARGUMENT, "NULL argument");
    if (rows <= 0 || n_shard <= 0 || col_begin < 0 || static_cast<int64_t>(col_begin) + n_shard > kNoColumn)
        return fail_tp(KT_ERR_INVALID_ARGUMENT, "bad column-parallel argmax arguments");
    if (comm->detached) return fail_tp(KT_ERR_INVALID_ARGUMENT, "a detached communicator has no collective");
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* scratch = nullptr;
    const size_t pair_words = 2 * static_cast<size_t>(rows);
    cudaError_t e = comm_scratch(comm, pair_words * (1 + comm->nranks), &scratch);
    if (e != cudaSuccess) return fail_tp(KT_ERR_OUT_OF_MEMORY, std::string("TP scratch: ") + cudaGetErrorString(e));
    int32_t* mine = reinterpret_cast<int32_t*>(scratch);
    int32_t* gathered = mine + pair_words;
    shard_argmax_kernel<<<rows, kArgmaxThreads, 0, s>>>(logits_shard, n_shard, col_begin, mine);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_tp(KT_ERR_CUDA, std::string("shard argmax: ") + cudaGetErrorString(e));
    // the pairs travel as 32-bit words (a float32 all-gather copies bits)
    const ncclResult_t r = nccl().all_gather(mine, gathered, pair_words, kNcclFloat32, comm->comm, s);
    if (r != 0) return nccl_fail(r, "ncclAllGather");
    merge_argmax_kernel<<<(rows + 127) / 128, 128, 0, s>>>(gathered, comm->nranks, rows, out);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail_tp(KT_ERR_CUDA, std::string("merge argmax: ") + cudaGetErrorString(e));
    return KT_OK;
}

}  // extern "C"
