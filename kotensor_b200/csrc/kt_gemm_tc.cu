// kt_gemm_tc.cu -- INT4 / INT8 dequantizing GEMM on the 5th-generation tensor cores:
// MatMul.multiplyQuantized (Engine/kotensor/src/main/kotlin/MatMul.kt:460-486)
// for m >= 9, the tile path of the reference (computeQuantizedTile,
// MatMul.kt:830-952) used by prefill and batched decode.
//
// Product.  c[m x N] = (accumulate ? c : 0) + alpha * a[m x K] . dequant(W) + bias,
// with W dequantized as in the reference (scale * (q - zero), fp32) and then
// rounded to bf16, a rounded to bf16, bf16 x bf16 products accumulated in fp32
// by tcgen05.mma (kind::f16) in tensor memory.  Tolerance 2e-2 relative to
// max|c| against the reference's fp32 result.
//
// Mapping.  The MMA computes D[128 x nt] = A[128 x K] . B[nt x K]^T with
//   A = dequantized weights, one row per output column (K-major, 128-byte swizzle)
//   B = bf16 activations, one row per token (K-major, 128-byte swizzle)
// so tokens are the MMA's N (16..256 per CTA, any m) and the 128 output
// columns its M.  A CTA owns 128 packed bytes of every weight row: INT4 packs
// column c and column c + half into one byte, so those bytes feed two A tiles
// (low and high nibble columns) and two accumulators of nt TMEM columns each.
//
// Pipeline per 64-row K-block, kStages deep:
//   warp 8  (one lane): TMA of the packed bytes [64 x 128] and the block's
//                       group scales / zero points -> "full_w"; TMA of the
//                       bf16 x tile [nt x 64] (128-byte swizzle) -> "full_x"
//   warps 0-7         : dequantize the packed bytes into the two A tiles
//                       (swizzled 16-byte stores), fence.proxy.async -> "full_a"
//   warp 9  (one lane): 2 x 4 tcgen05.mma (K = 16 each), tcgen05.commit -> "empty"
// then tcgen05.commit -> "done", and warps 0-7 read the accumulators with
// tcgen05.ld and write c.  Every mbarrier wait is bounded (globaltimer); a
// timeout sets the context's error word.
//
// The activations are converted to bf16 once per call by a small pre-pass
// kernel into the stream's workspace (after its reserved front).  Pre-pass,
// GEMM and split-K reduction are chained by programmatic dependent launch: the
// GEMM's CTAs start while the kernel before them runs, allocate tensor memory,
// load and dequantize the first stages of weights (which no kernel of the
// chain writes) and wait (griddepcontrol.wait) only before the first x tile.
//
// Split-K (when column x token tiles leave SMs idle): every split writes its
// fp32 partial tile to the workspace; the partials are summed in split order
// (deterministic) by the last CTA of the tile to arrive when they are small,
// or by a separate reduction kernel spread over the whole GPU when they are
// large (one CTA reading megabytes of partials would take tens of us).
#include <cuda_bf16.h>

#include <algorithm>
#include <cstdlib>

#include "kt_device.cuh"
#include "kt_internal.h"

namespace kt {
namespace {

constexpr int kBK = 64;                 // K rows per stage
constexpr int kTileBytes = 128;         // packed bytes per CTA (256 INT4 output columns)
constexpr int kMaxNT = 256;             // tokens per CTA (MMA N)
constexpr int kStages = 3;
constexpr int kWorkers = 8;             // dequantizing warps, then the epilogue
constexpr int kProducerWarp = kWorkers;
constexpr int kMmaWarp = kWorkers + 1;
constexpr int kThreads = (kWorkers + 2) * 32;
constexpr uint64_t kWaitLimitNs = 2000000000ull;

constexpr int kRawBytes = kBK * kTileBytes;          // 8 KiB packed
constexpr int kXBytes = kMaxNT * kBK * 2;            // 32 KiB bf16 activations
constexpr int kABytes = 128 * kBK * 2;               // 16 KiB bf16 weights per nibble half
constexpr int kStageBytes = kRawBytes + kXBytes + 2 * kABytes;
// per stage, the scales and zero points of the (at most two) groups its rows touch:
// scales low [128] | scales high [128] | zeros low [128] | zeros high [128]
constexpr int kGroupSlotBytes = 2 * kTileBytes * 4 + 2 * kTileBytes;
constexpr int kMaxGroupsPerStage = 2;
constexpr int kScaleStageBytes = kMaxGroupsPerStage * kGroupSlotBytes;
constexpr int kBarBytes = 128;
constexpr size_t kSmemBytes =
    1024 + static_cast<size_t>(kStages) * (kStageBytes + kScaleStageBytes) + kBarBytes;
static_assert(kStageBytes % 1024 == 0 && kRawBytes % 1024 == 0 && kXBytes % 1024 == 0 && kABytes % 1024 == 0,
              "swizzled tiles start on 1024-byte boundaries");
static_assert(kSmemBytes <= 232448, "shared memory per CTA");

struct GemmParams {
    const float* scales;
    const uint8_t* zeros;
    float* y;
    const float* bias;
    int32_t* err;
    int32_t M, K, N, R, gs, G;
    int32_t nt;        // tokens per CTA: multiple of 16, <= kMaxNT
    int32_t nt_cols;   // TMEM columns between the two accumulators
    int32_t tmem_cols; // TMEM columns allocated (power of two >= 32)
    uint32_t idesc;    // instruction descriptor of the MMA
    float alpha;
    int32_t accumulate;
    LoraEpilogue lora;
    // split-K (gridDim.z > 1): partial tiles and per-tile arrival counters
    float* partials;   // [tile][split][nt][256]
    int32_t* tickets;  // [tile], zero between launches
    int32_t reduce_kernel;  // 1: the partials are summed by split_reduce_kernel, not the last CTA
    // SwiGLU in split_reduce_kernel (INT4 gate | up weight, N = 2R): y receives
    // [M x R] silu(gate) * up, gate column b the low and up column R + b the
    // high nibble of byte b (accumulate 0)
    int32_t swiglu;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > kWaitLimitNs) return false;
    }
    return true;
}
// 1-D bulk copy global -> this CTA's shared memory (no multicast).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// 2-D TMA tile load into this CTA's shared memory (no multicast).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Shared-memory matrix descriptor of a K-major bf16 tile with 128-byte rows,
// 128-byte swizzle, 8-row atoms 1024 bytes apart (start address in 16-byte
// units; leading byte offset 1 (unused when swizzled); descriptor version 1).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t addr) {
    return static_cast<uint64_t>((addr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive fp32 columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(mask), "r"(c));
    return d;
}
// bf16x2 (a - b) * s, each lane of the pair rounded once to bf16 (a - b is exact here)
__device__ __forceinline__ uint32_t bf2_sub_mul(uint32_t a, uint32_t b, uint32_t s) {
    const __nv_bfloat162 r = __hmul2(__hsub2(*reinterpret_cast<const __nv_bfloat162*>(&a),
                                             *reinterpret_cast<const __nv_bfloat162*>(&b)),
                                     *reinterpret_cast<const __nv_bfloat162*>(&s));
    return *reinterpret_cast<const uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t bf2_splat(float v) {
    const __nv_bfloat162 h = __float2bfloat162_rn(v);
    return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ int atomic_add_acq_rel(int32_t* p, int v) {
    int old;
    asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void workers_barrier() { asm volatile("bar.sync 1, %0;" ::"n"(kWorkers * 32) : "memory"); }

// Epilogue of the worker warps (0-7): warp w reads TMEM lanes 32 (w % 4) .. +32
// of the low (w < 4) or high (w >= 4) accumulator (INT8: even / odd token
// chunks of the one accumulator), one tile column per thread, and writes c --
// or, split-K, its partial tile (summed by the tile's last CTA or by
// split_reduce_kernel).  acc_hi: TMEM column of the high-nibble accumulator.
template <int BITS>
__device__ __forceinline__ void gemm_epilogue(const GemmParams& p, uint32_t tmem, uint32_t acc_hi, uint32_t done,
                                              bool ok, int tile_b0, int tok0, int* s_last) {
    constexpr int kCT = BITS == 4 ? 2 * kTileBytes : kTileBytes;  // output columns per CTA
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    dev::pdl_wait();  // c may be read or written by the kernel before this one
    const bool have = ok && mbar_wait_bounded(done, 0);
    if (!have && lane == 0) atomicOr(p.err, 1);
    tc_fence_after();
    const int quarter = warp & 3;
    const int half_w = warp >> 2;  // INT4: low / high accumulator; INT8: even / odd token chunks
    const int c = 32 * quarter + lane;  // 0..127 in the accumulator
    const int colt = BITS == 4 ? half_w * 128 + c : c;  // column of the CTA's partial tile
    const uint32_t taddr =
        tmem + (static_cast<uint32_t>(32 * quarter) << 16) + (BITS == 4 && half_w ? acc_hi : 0);
    auto emit = [&](int tok, int col, float v) {
        const int cb = tile_b0 + (col & 127);
        const int oc = (BITS == 4 && col >= 128) ? p.R + cb : cb;
        if (!have || cb >= p.R || oc >= p.N || tok >= p.M) return;
        float* out = p.y + static_cast<int64_t>(tok) * p.N + oc;
        float r = fmaf(p.alpha, v, p.accumulate ? *out : 0.0f);
        if (p.bias != nullptr) r += p.bias[oc];
        if (p.lora.p != nullptr) r += lora_term(p.lora, tok, oc, p.N);
        *out = r;
    };
    const int S = gridDim.z;
    const int64_t tile_id = static_cast<int64_t>(blockIdx.y) * gridDim.x + blockIdx.x;
    float* parts = p.partials + tile_id * S * (static_cast<int64_t>(p.nt) * kCT);  // [S][nt][kCT]
    for (int t0 = (BITS == 4 ? 0 : 16 * half_w); t0 < p.nt; t0 += (BITS == 4 ? 16 : 32)) {
        float v[16];
        tmem_ld16(taddr + t0, v);  // every lane of the warp takes part (.sync.aligned)
        if (S == 1) {
#pragma unroll
            for (int j = 0; j < 16; ++j) emit(tok0 + t0 + j, colt, v[j]);
        } else {
            float* mine = parts + static_cast<int64_t>(blockIdx.z) * p.nt * kCT;
#pragma unroll
            for (int j = 0; j < 16; ++j) __stcg(mine + (t0 + j) * kCT + colt, v[j]);
        }
    }
    if (S > 1 && !p.reduce_kernel) {
        // split-K: the last CTA of the tile to arrive sums the partial tiles in
        // split order (the worker barrier orders every worker's stores before
        // thread 0's acq_rel atomic, which publishes them at GPU scope).
        workers_barrier();
        if (threadIdx.x == 0)
            *s_last = atomic_add_acq_rel(p.tickets + tile_id, 1) == S - 1;
        workers_barrier();
        if (*s_last) {
            // thread: 4 adjacent columns of one token at a time, tokens strided
            constexpr int kQuads = kCT / 4;
            const int q4 = (threadIdx.x % kQuads) * 4;
#pragma unroll 2
            for (int t = threadIdx.x / kQuads; t < p.nt; t += kWorkers * 32 / kQuads) {
                float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int sp = 0; sp < S; ++sp) {
                    const float4 u = __ldcg(reinterpret_cast<const float4*>(
                        parts + (static_cast<int64_t>(sp) * p.nt + t) * kCT + q4));
                    a0.x += u.x; a0.y += u.y; a0.z += u.z; a0.w += u.w;
                }
                emit(tok0 + t, q4, a0.x); emit(tok0 + t, q4 + 1, a0.y);
                emit(tok0 + t, q4 + 2, a0.z); emit(tok0 + t, q4 + 3, a0.w);
            }
            if (threadIdx.x == 0) p.tickets[tile_id] = 0;  // ready for the next launch on this workspace
        }
    }
}

// BITS = 4: a CTA's 128 packed bytes are 256 output columns (two A tiles, two
// accumulators); BITS = 8: 128 output columns (one A tile, one accumulator).
template <int BITS>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                   GemmParams p) {
    constexpr int kCT = BITS == 4 ? 2 * kTileBytes : kTileBytes;  // output columns per CTA
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tile_b0 = blockIdx.x * kTileBytes;
    const int tok0 = blockIdx.y * p.nt;
    // this CTA's K-blocks: split blockIdx.z of gridDim.z, spread evenly
    const int kb_total = (p.K + kBK - 1) / kBK;
    const int kb_begin = static_cast<int>(static_cast<int64_t>(blockIdx.z) * kb_total / gridDim.z);
    const int kb_end = static_cast<int>(static_cast<int64_t>(blockIdx.z + 1) * kb_total / gridDim.z);
    const int n_kb = kb_end - kb_begin;  // >= 1 (the host keeps splits <= kb_total)

    // 1024-aligned base for the swizzled tiles
    const uint32_t raw_s = smem_u32(smem_raw);
    const uint32_t base = (raw_s + 1023u) & ~1023u;
    unsigned char* gbase = smem_raw + (base - raw_s);
    const uint32_t scl = base + kStages * kStageBytes;  // scale slots [stage][group]
    const uint32_t bars = scl + kStages * kScaleStageBytes;
    auto full_w = [&](int s) { return bars + 8 * s; };
    auto full_x = [&](int s) { return bars + 8 * (kStages + s); };
    auto full_a = [&](int s) { return bars + 8 * (2 * kStages + s); };
    auto empty = [&](int s) { return bars + 8 * (3 * kStages + s); };
    const uint32_t done = bars + 8 * (4 * kStages);
    uint32_t* tmem_slot =
        reinterpret_cast<uint32_t*>(gbase + kStages * (kStageBytes + kScaleStageBytes) + 8 * (4 * kStages + 1));
    const int tile_cols = min(kTileBytes, p.R - tile_b0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full_w(s), 1);
            mbar_init(full_x(s), 1);
            mbar_init(full_a(s), kWorkers);
            mbar_init(empty(s), 1);
        }
        mbar_init(done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(p.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    dev::pdl_launch_dependents();
    if (warp == kProducerWarp) {
        if (lane == 0) {
            const uint32_t xtx = static_cast<uint32_t>(p.nt * kBK * 2);
            const uint32_t gbytes = static_cast<uint32_t>(tile_cols) * (BITS == 4 ? 10 : 4);
            // the packed bytes and group constants of block i -> full_w(i % NS)
            auto issue_w = [&](int i) {
                const int s = i % kStages;
                const uint32_t st = base + s * kStageBytes;
                const int kb = kb_begin + i;
                const int ga = min(kb * kBK / p.gs, p.G - 1);
                const int gb = min((kb * kBK + kBK - 1) / p.gs, p.G - 1);
                mbar_expect_tx(full_w(s), kRawBytes + (gb - ga + 1) * gbytes);
                tma_load_2d(st, &tmap_w, tile_b0, kb * kBK, full_w(s));
                for (int g = ga; g <= gb; ++g) {
                    const uint32_t dst = scl + s * kScaleStageBytes + (g - ga) * kGroupSlotBytes;
                    const int64_t go = static_cast<int64_t>(g) * p.N;
                    bulk_load(dst, p.scales + go + tile_b0, tile_cols * 4, full_w(s));
                    if constexpr (BITS == 4) {
                        bulk_load(dst + kTileBytes * 4, p.scales + go + p.R + tile_b0, tile_cols * 4, full_w(s));
                        bulk_load(dst + kTileBytes * 8, p.zeros + go + tile_b0, tile_cols, full_w(s));
                        bulk_load(dst + kTileBytes * 9, p.zeros + go + p.R + tile_b0, tile_cols, full_w(s));
                    }
                }
            };
            // the bf16 x tile of block i -> full_x(i % NS)
            auto issue_x = [&](int i) {
                const int s = i % kStages;
                mbar_expect_tx(full_x(s), xtx);
                tma_load_2d(base + s * kStageBytes + kRawBytes, &tmap_x, (kb_begin + i) * kBK, tok0, full_x(s));
            };
            // Weights of the first stages before the wait (no kernel of the
            // chain writes them), x only after it: x is the previous kernel's output.
            const int pre = min(n_kb, kStages);
            for (int i = 0; i < pre; ++i) issue_w(i);
            dev::pdl_wait();
            for (int i = 0; i < pre; ++i) issue_x(i);
            int issued = pre;
            for (int i = pre; i < n_kb; ++i) {
                const int s = i % kStages;
                if (!mbar_wait_bounded(empty(s), ((i / kStages) - 1) & 1)) {
                    atomicOr(p.err, 1);
                    break;
                }
                issue_w(i);
                issue_x(i);
                ++issued;
            }
            // the last copies issued into each slot have landed before the CTA may exit
            for (int i = max(0, issued - kStages); i < issued; ++i) {
                if (!mbar_wait_bounded(full_w(i % kStages), (i / kStages) & 1)) break;
                if (!mbar_wait_bounded(full_x(i % kStages), (i / kStages) & 1)) break;
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            for (int i = 0; i < n_kb; ++i) {
                const int s = i % kStages;
                const uint32_t par = (i / kStages) & 1;
                if (!mbar_wait_bounded(full_x(s), par) || !mbar_wait_bounded(full_a(s), par)) {
                    atomicOr(p.err, 1);
                    break;
                }
                tc_fence_after();
                const uint32_t st = base + s * kStageBytes;
                const uint32_t xs = st + kRawBytes, alo = xs + kXBytes, ahi = alo + kABytes;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    const uint64_t bdesc = umma_desc_sw128(xs + kk * 32);
                    const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
                    umma_bf16(tmem, umma_desc_sw128(alo + kk * 32), bdesc, p.idesc, acc);
                    if constexpr (BITS == 4)
                        umma_bf16(tmem + p.nt_cols, umma_desc_sw128(ahi + kk * 32), bdesc, p.idesc, acc);
                }
                umma_commit(empty(s));  // the stage is free once these MMAs have read it
            }
            umma_commit(done);
            if (!mbar_wait_bounded(done, 0)) atomicOr(p.err, 1);  // no MMA in flight past this point
        }
    } else {
        // ---- dequantize: warp w owns rows 8w..8w+7 of each stage (one 16-byte
        // k-chunk of every A row); lane l owns tile columns l + 32 i.  The
        // next K-block's group constants are loaded while this one is
        // converted.  A pair of rows (k, k+1) of one column becomes one bf16x2
        // word: PRMT puts the two bytes in the two halves, LOP3 ORs each nibble
        // into the mantissa of 128.0 (0x4300), and (128 + q) - (128 + zero)
        // is exact before the one rounding of the scale multiply.
        bool ok = true;
        for (int i = 0; i < n_kb; ++i) {
            const int s = i % kStages;
            const int kb = kb_begin + i;
            if (!mbar_wait_bounded(full_w(s), (i / kStages) & 1)) {
                if (lane == 0) atomicOr(p.err, 1);
                ok = false;
                break;
            }
            const unsigned char* raw = gbase + s * kStageBytes;
            unsigned char* alo = gbase + s * kStageBytes + kRawBytes + kXBytes;
            unsigned char* ahi = alo + kABytes;
            // this warp's rows (8 of them, gs % 32 == 0) lie in one group
            const int ga = min(kb * kBK / p.gs, p.G - 1);
            const int gw = min((kb * kBK + 8 * warp) / p.gs, p.G - 1);
            const unsigned char* slot = gbase + kStages * kStageBytes + s * kScaleStageBytes + (gw - ga) * kGroupSlotBytes;
            const float* sc_lo = reinterpret_cast<const float*>(slot);
            const float* sc_hi = sc_lo + kTileBytes;
            const unsigned char* z_lo = slot + kTileBytes * 8;
            const unsigned char* z_hi = slot + kTileBytes * 9;
#pragma unroll
            for (int c4 = 0; c4 < 4; ++c4) {
                const int c = lane + 32 * c4;
                // columns beyond the tile's bytes read stale slot data; their A rows
                // only reach accumulator rows that are never stored
                uint32_t b[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) b[j] = raw[(8 * warp + j) * kTileBytes + c];
                const uint32_t off = static_cast<uint32_t>(c * 128 + ((warp ^ (c & 7)) << 4));
                if constexpr (BITS == 4) {
                    const uint32_t s2_lo = bf2_splat(sc_lo[c]), s2_hi = bf2_splat(sc_hi[c]);
                    const uint32_t zb_lo = bf2_splat(128.0f + static_cast<float>(z_lo[c]));
                    const uint32_t zb_hi = bf2_splat(128.0f + static_cast<float>(z_hi[c]));
                    uint4 vlo, vhi;
                    uint32_t* wl = &vlo.x;
                    uint32_t* wh = &vhi.x;
#pragma unroll
                    for (int jp = 0; jp < 4; ++jp) {
                        const uint32_t pr = prmt(b[2 * jp], b[2 * jp + 1], 0x5410u);  // rows 2jp, 2jp+1 in the halves
                        const uint32_t ql = lop3_and_or(pr, 0x000F000Fu, 0x43004300u);
                        const uint32_t qh = lop3_and_or(pr >> 4, 0x000F000Fu, 0x43004300u);
                        wl[jp] = bf2_sub_mul(ql, zb_lo, s2_lo);
                        wh[jp] = bf2_sub_mul(qh, zb_hi, s2_hi);
                    }
                    *reinterpret_cast<uint4*>(alo + off) = vlo;
                    *reinterpret_cast<uint4*>(ahi + off) = vhi;
                } else {
                    // signed byte q: 2^23 + (q + 128) as a float (byte ^ 0x80 in the
                    // mantissa) minus 2^23 + 128 is exactly q; one fp32 multiply by
                    // the scale as the reference (QuantizedTensor.kt:201), then bf16
                    const float sc = sc_lo[c];
                    uint4 v;
                    uint32_t* wv = &v.x;
#pragma unroll
                    for (int jp = 0; jp < 4; ++jp) {
                        const float q0 = __uint_as_float(b[2 * jp] ^ 0x4B000080u) - 8388736.0f;
                        const float q1 = __uint_as_float(b[2 * jp + 1] ^ 0x4B000080u) - 8388736.0f;
                        wv[jp] = pack_bf16(__fmul_rn(sc, q0), __fmul_rn(sc, q1));
                    }
                    *reinterpret_cast<uint4*>(alo + off) = v;
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic stores -> MMA reads
            __syncwarp();
            if (lane == 0) mbar_arrive(full_a(s));
        }
        gemm_epilogue<BITS>(p, tmem, p.nt_cols, done, ok, tile_b0, tok0, &s_last);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols)
                     : "memory");
    }
}

// ---------------------------------------------------------------------------
// INT4 with the dequantized weights in tensor memory (the "A from TMEM" form of
// tcgen05.mma), for tiles of at most 128 tokens.  Same mapping, split-K and
// epilogue as gemm_tc_kernel; what changes is where the A tiles live and how
// the pipeline is cut.  In gemm_tc_kernel every 64-row K-block costs ~1,000
// shared-memory wavefronts (byte loads of the packed tile, scale loads by all
// eight warps, 32 KB of A stores and the MMA's A reads) and its 3-stage ring
// exposes the TMA latency (~1 us) on every block.  Here:
//   * an 8-stage shared-memory ring of packed bytes + x tiles, decoupled from
//     a 4-stage ring of A tiles in tensor memory (own full / free barriers);
//   * 16 dequantizing warps in two groups of 8 that take alternate K-blocks
//     (a warp's chain of loads, shuffles, conversions and tcgen05.st takes
//     ~0.5 us; two blocks in flight hide half of it).  They write A with
//     tcgen05.st (TMEM lane L = A row L = byte column L of the tile): warp w of
//     a group takes TMEM lanes 32 (w % 4) .. +32 and rows 32 (w / 4) .. +32;
//   * the group scales and zero points are read by the dequantizing lanes
//     straight from global memory (one block of their own ahead): issuing them
//     as four small bulk copies per block cost the single producer thread
//     ~0.3 us per block, which bounded the pipeline;
//   * conflict-free 32-bit loads of the packed bytes: lane (i = lane % 4,
//     j = lane / 4) loads word 8 (w % 4) + j of rows b + 2i (b = 0, 1) of an
//     8-row atom -- with the 128-byte swizzle the 32 lanes hit 32 distinct
//     banks -- and a 4 x 4 byte transpose across lanes 4j .. 4j + 3 (two
//     shuffles, two PRMT) leaves lane L with byte column L of rows b, b + 2,
//     b + 4, b + 6.  A PRMT pairs rows (2p, 2p + 1) into the two halves of a
//     word and the nibbles become bf16 exactly as in gemm_tc_kernel.
// TMEM columns: low accumulator 0 .. nt, high 128 .. 128 + nt, A tiles of A-stage
// a at 256 + 64 a (low nibbles) and 256 + 64 a + 32 (high): all 512 columns, so
// one CTA per SM (its shared memory is more than half an SM's).
constexpr int kTsMaxNT = 128;
constexpr int kTsRing = 8;             // shared-memory stages (packed bytes + x)
constexpr int kTsAStages = 4;          // tensor-memory stages (A tiles)
constexpr int kTsDequant = 16;         // dequantizing warps, two groups of 8 (the first 8 also run the epilogue)
constexpr int kTsGroupWarps = kTsDequant / 2;
constexpr int kTsProducerWarp = kTsDequant;
constexpr int kTsMmaWarp = kTsDequant + 1;
constexpr int kTsThreads = (kTsDequant + 2) * 32;
constexpr int kTsRawBytes = kBK * kTileBytes;        // two 32-row TMA boxes, 128-byte swizzle
constexpr int kTsXBytes = kTsMaxNT * kBK * 2;
constexpr int kTsStageBytes = kTsRawBytes + kTsXBytes;
constexpr uint32_t kTsAccHi = 128;
constexpr uint32_t kTsACol = 256;
constexpr int kTsBarBytes = 512;
constexpr size_t kTsSmemBytes = 1024 + static_cast<size_t>(kTsRing) * kTsStageBytes + kTsBarBytes;
static_assert(kTsStageBytes % 1024 == 0 && kTsRawBytes % 1024 == 0, "swizzled tiles start on 1024-byte boundaries");
static_assert(2 * kTsSmemBytes > 233472 && kTsSmemBytes <= 232448, "exactly one CTA per SM");
static_assert(kTsACol + 64 * kTsAStages <= 512, "tensor memory columns");
static_assert(8 * (3 * kTsRing + 2 * kTsAStages + 1) + 4 <= kTsBarBytes, "barrier area");

// A from tensor memory: D (TMEM) += A (TMEM) . B (shared memory descriptor).
__device__ __forceinline__ void umma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 16 consecutive 32-bit TMEM columns of this warp's 32 lanes from registers.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
// The group constants one dequantizing lane needs for a K-block: scale and
// zero point of its low- and high-nibble columns.
struct ColumnConstants {
    float s_lo, s_hi;
    uint32_t z_lo, z_hi;
};
__device__ __forceinline__ ColumnConstants load_constants(const GemmParams& p, int row, int col) {
    const int64_t g = static_cast<int64_t>(min(row / p.gs, p.G - 1)) * p.N;
    ColumnConstants c;
    c.s_lo = __ldg(p.scales + g + col);
    c.s_hi = __ldg(p.scales + g + p.R + col);
    c.z_lo = __ldg(p.zeros + g + col);
    c.z_hi = __ldg(p.zeros + g + p.R + col);
    return c;
}
// 4 x 4 byte transpose across lanes 4j .. 4j + 3 (li = lane % 4): lane li holds
// bytes [a(li,0) .. a(li,3)] and returns [a(0,li) .. a(3,li)].
__device__ __forceinline__ uint32_t transpose4x4(uint32_t w, int li) {
    const uint32_t x = __shfl_xor_sync(0xffffffffu, w, 1);
    const uint32_t v = prmt(w, x, (li & 1) ? 0x3715u : 0x6240u);
    const uint32_t y = __shfl_xor_sync(0xffffffffu, v, 2);
    return prmt(v, y, (li & 2) ? 0x3276u : 0x5410u);
}

__global__ void __launch_bounds__(kTsThreads, 1)
    gemm_ts_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_x,
                   GemmParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tile_b0 = blockIdx.x * kTileBytes;
    const int tok0 = blockIdx.y * p.nt;
    const int kb_total = (p.K + kBK - 1) / kBK;
    const int kb_begin = static_cast<int>(static_cast<int64_t>(blockIdx.z) * kb_total / gridDim.z);
    const int kb_end = static_cast<int>(static_cast<int64_t>(blockIdx.z + 1) * kb_total / gridDim.z);
    const int n_kb = kb_end - kb_begin;

    const uint32_t raw_s = smem_u32(smem_raw);
    const uint32_t base = (raw_s + 1023u) & ~1023u;
    unsigned char* gbase = smem_raw + (base - raw_s);
    const uint32_t bars = base + kTsRing * kTsStageBytes;
    auto full_w = [&](int s) { return bars + 8 * s; };                       // ring slot s: packed bytes
    auto full_x = [&](int s) { return bars + 8 * (kTsRing + s); };           // ring slot s: x tile
    auto empty = [&](int s) { return bars + 8 * (2 * kTsRing + s); };        // ring slot s consumed by the MMAs
    auto full_a = [&](int a) { return bars + 8 * (3 * kTsRing + a); };       // A-stage a written
    auto free_a = [&](int a) { return bars + 8 * (3 * kTsRing + kTsAStages + a); };  // A-stage a read by the MMAs
    const uint32_t done = bars + 8 * (3 * kTsRing + 2 * kTsAStages);
    uint32_t* tmem_slot =
        reinterpret_cast<uint32_t*>(gbase + kTsRing * kTsStageBytes + 8 * (3 * kTsRing + 2 * kTsAStages + 1));
    const int tile_cols = min(kTileBytes, p.R - tile_b0);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTsRing; ++s) {
            mbar_init(full_w(s), 1);
            mbar_init(full_x(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int a = 0; a < kTsAStages; ++a) {
            mbar_init(full_a(a), kTsGroupWarps);
            mbar_init(free_a(a), 1);
        }
        mbar_init(done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(512)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    dev::pdl_launch_dependents();

    if (warp == kTsProducerWarp) {
        // lane 0 arms full_w and loads rows 0-31 of the packed tile, lane 1 rows
        // 32-63 (a copy landing before lane 0's arming arrive cannot complete the
        // phase: that arrive is still pending), lane 2 arms full_x and loads x
        const uint32_t xtx = static_cast<uint32_t>(p.nt * kBK * 2);
        auto issue = [&](int i, bool w, bool x) {
            const int s = i % kTsRing;
            const uint32_t st = base + s * kTsStageBytes;
            const int kb = kb_begin + i;
            if (w) {
                if (lane == 0) {
                    mbar_expect_tx(full_w(s), kTsRawBytes);
                    tma_load_2d(st, &tmap_w, tile_b0, kb * kBK, full_w(s));
                } else if (lane == 1) {
                    tma_load_2d(st + kTsRawBytes / 2, &tmap_w, tile_b0, kb * kBK + kBK / 2, full_w(s));
                }
            }
            if (x && lane == 2) {
                mbar_expect_tx(full_x(s), xtx);
                tma_load_2d(st + kTsRawBytes, &tmap_x, kb * kBK, tok0, full_x(s));
            }
        };
        // weights of the first stages before the wait (no kernel of the chain
        // writes them), x only after it
        const int pre = min(n_kb, kTsRing);
        for (int i = 0; i < pre; ++i) issue(i, true, false);
        dev::pdl_wait();
        for (int i = 0; i < pre; ++i) issue(i, false, true);
        int issued = pre;
        for (int i = pre; i < n_kb; ++i) {
            const int s = i % kTsRing;
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(empty(s), ((i / kTsRing) - 1) & 1))) {
                if (lane == 0) atomicOr(p.err, 1);
                break;
            }
            issue(i, true, true);
            ++issued;
        }
        // the last copies issued into each slot have landed before the CTA may exit
        if (lane == 0) {
            for (int i = max(0, issued - kTsRing); i < issued; ++i) {
                if (!mbar_wait_bounded(full_w(i % kTsRing), (i / kTsRing) & 1)) break;
                if (!mbar_wait_bounded(full_x(i % kTsRing), (i / kTsRing) & 1)) break;
            }
        }
    } else if (warp == kTsMmaWarp) {
        if (lane == 0) {
            for (int i = 0; i < n_kb; ++i) {
                const int s = i % kTsRing, a = i % kTsAStages;
                if (!mbar_wait_bounded(full_x(s), (i / kTsRing) & 1) ||
                    !mbar_wait_bounded(full_a(a), (i / kTsAStages) & 1)) {
                    atomicOr(p.err, 1);
                    break;
                }
                tc_fence_after();
                const uint32_t xs = base + s * kTsStageBytes + kTsRawBytes;
                const uint32_t a_lo = tmem + kTsACol + 64 * a;
#pragma unroll
                for (int kk = 0; kk < kBK / 16; ++kk) {
                    const uint64_t bdesc = umma_desc_sw128(xs + kk * 32);
                    const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
                    umma_bf16_ts(tmem, a_lo + 8 * kk, bdesc, p.idesc, acc);
                    umma_bf16_ts(tmem + kTsAccHi, a_lo + 32 + 8 * kk, bdesc, p.idesc, acc);
                }
                umma_commit(empty(s));   // ring slot free once these MMAs have read it
                umma_commit(free_a(a));  // and the A-stage
            }
            umma_commit(done);
            if (!mbar_wait_bounded(done, 0)) atomicOr(p.err, 1);
        }
    } else {
        const int grp = warp / kTsGroupWarps;  // this warp's K-blocks: i = grp, grp + 2, ...
        const int wg = warp % kTsGroupWarps;
        const int q = wg & 3;   // TMEM lanes / byte columns 32 q .. 32 q + 31
        const int h = wg >> 2;  // rows 32 h .. 32 h + 31 of each K-block
        const int li = lane & 3, lj = lane >> 2;
        const int bc = 32 * q + lane;  // this lane's byte column after the transpose
        const int wc = 8 * q + lj;     // the 32-bit word column this lane loads
        const uint32_t lane_base = static_cast<uint32_t>(32 * q) << 16;
        // columns beyond the tile's bytes (last tile) read column 0's constants:
        // their A rows only reach accumulator rows that are never stored
        const int col = tile_b0 + (bc < tile_cols ? bc : 0);
        bool ok = true;
        ColumnConstants cc{};
        if (grp < n_kb) cc = load_constants(p, (kb_begin + grp) * kBK + 32 * h, col);
        for (int i = grp; i < n_kb; i += 2) {
            const int s = i % kTsRing, as = i % kTsAStages;
            const ColumnConstants cur = cc;
            if (i + 2 < n_kb) cc = load_constants(p, (kb_begin + i + 2) * kBK + 32 * h, col);  // next block's, early
            // warp-uniform waits: the tcgen05.st below is .sync.aligned
            bool got = mbar_wait_bounded(full_w(s), (i / kTsRing) & 1);
            if (i >= kTsAStages) got = got && mbar_wait_bounded(free_a(as), ((i / kTsAStages) - 1) & 1);
            if (!__all_sync(0xffffffffu, got)) {
                if (lane == 0) atomicOr(p.err, 1);
                ok = false;
                break;
            }
            tc_fence_after();  // the MMAs that read this A-stage before have completed
            const unsigned char* raw = gbase + s * kTsStageBytes;
            const uint32_t s2_lo = bf2_splat(cur.s_lo), s2_hi = bf2_splat(cur.s_hi);
            const uint32_t zb_lo = bf2_splat(128.0f + static_cast<float>(cur.z_lo));
            const uint32_t zb_hi = bf2_splat(128.0f + static_cast<float>(cur.z_hi));
            uint32_t lo[16], hi[16];
#pragma unroll
            for (int a = 0; a < 4; ++a) {
                uint32_t t[2];
#pragma unroll
                for (int b = 0; b < 2; ++b) {
                    const int r = 32 * h + 8 * a + b + 2 * li;  // (r & 7) == b + 2 li
                    const uint32_t w = *reinterpret_cast<const uint32_t*>(
                        raw + r * kTileBytes + ((((wc >> 2) ^ (b + 2 * li)) << 4) | ((wc & 3) << 2)));
                    t[b] = transpose4x4(w, li);  // byte column bc, rows 32h + 8a + b + {0, 2, 4, 6}
                }
#pragma unroll
                for (int pp = 0; pp < 4; ++pp) {
                    // rows 8a + 2pp (low half of the word) and 8a + 2pp + 1 (high half)
                    const uint32_t pr =
                        prmt(t[0], t[1], static_cast<uint32_t>(pp | (pp << 4) | ((4 + pp) << 8) | ((4 + pp) << 12)));
                    const uint32_t ql = lop3_and_or(pr, 0x000F000Fu, 0x43004300u);
                    const uint32_t qh = lop3_and_or(pr >> 4, 0x000F000Fu, 0x43004300u);
                    lo[4 * a + pp] = bf2_sub_mul(ql, zb_lo, s2_lo);
                    hi[4 * a + pp] = bf2_sub_mul(qh, zb_hi, s2_hi);
                }
            }
            const uint32_t a_col = tmem + lane_base + kTsACol + 64 * as + 16 * h;
            tmem_st16(a_col, lo);
            tmem_st16(a_col + 32, hi);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(full_a(as));
        }
        if (warp < kWorkers) gemm_epilogue<4>(p, tmem, kTsAccHi, done, ok, tile_b0, tok0, &s_last);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
    }
}

// ---------------------------------------------------------------------------
// MatMul.multiplyByQuantizedTransposed (MatMul.kt:954-981) on tcgen05, INT4
// (INT8 below), m >= 16: dx[m x K] (+)= dy[m x N] . dequant(W)^T.  D[128 x nt] = A[128 x N] .
// B[nt x N]^T with A = dequantized weight rows (one row per output row k of
// dx, contraction over the N columns) and B = dy in bf16 (one row per token).
// A CTA owns 128 rows k0 .. k0 + 127; a stage is one TMA box of those rows x 64
// packed bytes (bytes n0 .. n0 + 63): its low nibbles are columns n0 .. n0 + 63
// and its high nibbles columns R + n0 .. (split-half packing, R = N / 2), two
// contraction blocks of 64 that accumulate into one TMEM accumulator against
// the two matching 64-column tiles of dy.  Dequantizing warp w takes rows
// 16 w .. + 15, lane l row 16 w + l / 2 and bytes 32 (l % 2) .. + 31: a PRMT
// puts two adjacent bytes in the halves of a word, a LOP3 ORs each nibble into
// the mantissa of bf16 128.0 (exact), (128 + q) - (128 + zero) is exact, and
// one bf16 multiply by the column's scale rounds it -- the forward GEMM's
// arithmetic, here with a scale and zero point per column of the pair.  The
// epilogue, split-K partials and reduction are the one-accumulator (INT8)
// path of the forward GEMM: output "columns" are rows k of dx.
// INT8 (BITS = 8): a stage's 64 bytes are columns n0 .. n0 + 63 (one
// contraction block, one dy tile, one A tile); the signed byte becomes q
// exactly through the fp32 mantissa and one fp32 multiply by the column's
// scale (QuantizedTensor.kt:201) is rounded to bf16, as in the forward GEMM.
constexpr int kTRows = 128;              // output rows per CTA (the MMA's M)
constexpr int kTMaxNT = 128;             // tokens per CTA (the MMA's N)
constexpr int kTRawBytes = kTRows * 64;  // 8 KiB: 128 rows x 64 packed bytes
constexpr int kTXBytes = kTMaxNT * 64 * 2;  // 16 KiB: a 64-column bf16 tile of dy
constexpr int kTABytes = kTRows * 64 * 2;   // 16 KiB: a 64-column bf16 A tile
constexpr int kTStageBytes = kTRawBytes + 2 * kTXBytes + 2 * kTABytes;  // 72 KiB
constexpr int kTMaxGroups = 4;           // groups a 128-row tile can touch (group sizes 32, 64, multiples of 128)
// per group: scales low [64] | scales high [64] | zeros low [64] | zeros high [64]
constexpr int kTGroupBytes = 2 * 64 * 4 + 2 * 64;
constexpr int kTScaleStageBytes = kTMaxGroups * kTGroupBytes;
constexpr int kTBarBytes = 256;
// A stage holds the dy tiles of this launch's nt tokens only (nt x 128 bytes each,
// a multiple of 2 KiB), so at nt <= 48 the ring has room for a fourth stage.
__host__ __device__ constexpr int t_stage_bytes(int nt) { return kTRawBytes + 2 * nt * 64 * 2 + 2 * kTABytes; }
constexpr size_t t_smem_bytes(int stages, int nt) {
    return 1024 + static_cast<size_t>(stages) * (t_stage_bytes(nt) + kTScaleStageBytes) + kTBarBytes;
}
constexpr int kTMaxNT4 = 48;  // the largest nt with four stages
static_assert(kTStageBytes == t_stage_bytes(kTMaxNT) && kTRawBytes % 1024 == 0 && kTXBytes % 1024 == 0 &&
              t_stage_bytes(16) % 1024 == 0, "1024-byte tiles");
// + 1 KiB of static shared memory
static_assert(t_smem_bytes(kStages, kTMaxNT) + 1024 <= 232448 && t_smem_bytes(4, kTMaxNT4) + 1024 <= 232448,
              "shared memory per CTA");
static_assert(8 * (4 * 4 + 1) + 4 <= kTBarBytes, "barrier area");

template <int BITS, int STAGES>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_t_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_dy,
                  GemmParams p) {
    constexpr bool kInt4 = BITS == 4;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    __shared__ int s_last;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int k0 = blockIdx.x * kTRows;  // first output row (row of W, column of dx)
    const int tok0 = blockIdx.y * p.nt;
    const int ncols = p.K;               // the weight's columns N (the contraction; p.N is dx's row length)
    const int half = kInt4 ? ncols / 2 : ncols;  // INT4: columns per nibble half (N % 128 == 0); bytes per row
    const int kb_total = half / 64;
    const int kb_begin = static_cast<int>(static_cast<int64_t>(blockIdx.z) * kb_total / gridDim.z);
    const int kb_end = static_cast<int>(static_cast<int64_t>(blockIdx.z + 1) * kb_total / gridDim.z);
    const int n_kb = kb_end - kb_begin;
    const int g_first = min(k0 / p.gs, p.G - 1);
    const int g_last = min((k0 + kTRows - 1) / p.gs, p.G - 1);

    const int xbytes = p.nt * 64 * 2;  // one dy tile: nt rows x 64 bf16
    const int stage_bytes = kTRawBytes + 2 * xbytes + 2 * kTABytes;
    const uint32_t raw_s = smem_u32(smem_raw);
    const uint32_t base = (raw_s + 1023u) & ~1023u;
    unsigned char* gbase = smem_raw + (base - raw_s);
    const uint32_t scl = base + STAGES * stage_bytes;  // group slots [stage][group]
    const uint32_t bars = scl + STAGES * kTScaleStageBytes;
    auto full_w = [&](int s) { return bars + 8 * s; };
    auto full_x = [&](int s) { return bars + 8 * (STAGES + s); };
    auto full_a = [&](int s) { return bars + 8 * (2 * STAGES + s); };
    auto empty = [&](int s) { return bars + 8 * (3 * STAGES + s); };
    const uint32_t done = bars + 8 * (4 * STAGES);
    uint32_t* tmem_slot =
        reinterpret_cast<uint32_t*>(gbase + STAGES * (stage_bytes + kTScaleStageBytes) + 8 * (4 * STAGES + 1));

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full_w(s), 1);
            mbar_init(full_x(s), 1);
            mbar_init(full_a(s), kWorkers);
            mbar_init(empty(s), 1);
        }
        mbar_init(done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(p.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    dev::pdl_launch_dependents();
    if (warp == kProducerWarp) {
        if (lane == 0) {
            const uint32_t xtx = static_cast<uint32_t>((kInt4 ? 2 : 1) * p.nt * 64 * 2);
            const uint32_t gtx = static_cast<uint32_t>((g_last - g_first + 1) * (kInt4 ? kTGroupBytes : 64 * 4));
            // the packed bytes and the group constants of block i -> full_w(i % NS)
            auto issue_w = [&](int i) {
                const int s = i % STAGES;
                const int n0 = (kb_begin + i) * 64;
                mbar_expect_tx(full_w(s), kTRawBytes + gtx);
                tma_load_2d(base + s * stage_bytes, &tmap_w, n0, k0, full_w(s));
                for (int g = g_first; g <= g_last; ++g) {
                    const uint32_t dst = scl + s * kTScaleStageBytes + (g - g_first) * kTGroupBytes;
                    const int64_t go = static_cast<int64_t>(g) * ncols;
                    bulk_load(dst, p.scales + go + n0, 64 * 4, full_w(s));
                    if (kInt4) {
                        bulk_load(dst + 256, p.scales + go + half + n0, 64 * 4, full_w(s));
                        bulk_load(dst + 512, p.zeros + go + n0, 64, full_w(s));
                        bulk_load(dst + 576, p.zeros + go + half + n0, 64, full_w(s));
                    }
                }
            };
            // the two bf16 tiles of dy (columns n0.., R + n0..) of block i -> full_x(i % NS)
            auto issue_x = [&](int i) {
                const int s = i % STAGES;
                const int n0 = (kb_begin + i) * 64;
                const uint32_t xs = base + s * stage_bytes + kTRawBytes;
                mbar_expect_tx(full_x(s), xtx);
                tma_load_2d(xs, &tmap_dy, n0, tok0, full_x(s));
                if (kInt4) tma_load_2d(xs + xbytes, &tmap_dy, half + n0, tok0, full_x(s));
            };
            // weights of the first stages before the wait (no kernel of the chain writes
            // them), dy only after it: dy is the previous kernel's output
            const int pre = min(n_kb, STAGES);
            for (int i = 0; i < pre; ++i) issue_w(i);
            dev::pdl_wait();
            for (int i = 0; i < pre; ++i) issue_x(i);
            int issued = pre;
            for (int i = pre; i < n_kb; ++i) {
                const int s = i % STAGES;
                if (!mbar_wait_bounded(empty(s), ((i / STAGES) - 1) & 1)) {
                    atomicOr(p.err, 1);
                    break;
                }
                issue_w(i);
                issue_x(i);
                ++issued;
            }
            // the last copies issued into each slot have landed before the CTA may exit
            for (int i = max(0, issued - STAGES); i < issued; ++i) {
                if (!mbar_wait_bounded(full_w(i % STAGES), (i / STAGES) & 1)) break;
                if (!mbar_wait_bounded(full_x(i % STAGES), (i / STAGES) & 1)) break;
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            for (int i = 0; i < n_kb; ++i) {
                const int s = i % STAGES;
                const uint32_t par = (i / STAGES) & 1;
                if (!mbar_wait_bounded(full_x(s), par) || !mbar_wait_bounded(full_a(s), par)) {
                    atomicOr(p.err, 1);
                    break;
                }
                tc_fence_after();
                const uint32_t xlo = base + s * stage_bytes + kTRawBytes, xhi = xlo + xbytes;
                const uint32_t alo = xhi + xbytes, ahi = alo + kTABytes;
#pragma unroll
                for (int kk = 0; kk < 64 / 16; ++kk) {
                    const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
                    umma_bf16(tmem, umma_desc_sw128(alo + kk * 32), umma_desc_sw128(xlo + kk * 32), p.idesc, acc);
                    if (kInt4)
                        umma_bf16(tmem, umma_desc_sw128(ahi + kk * 32), umma_desc_sw128(xhi + kk * 32), p.idesc, 1u);
                }
                umma_commit(empty(s));  // the stage is free once these MMAs have read it
            }
            umma_commit(done);
            if (!mbar_wait_bounded(done, 0)) atomicOr(p.err, 1);  // no MMA in flight past this point
        }
    } else {
        bool ok = true;
        const int r = 16 * warp + (lane >> 1);  // INT8: row of the tile
        const int hh = lane & 1;                // INT8: bytes 32 hh .. + 31 of the row
        const int gsl = min((k0 + r) / p.gs, p.G - 1) - g_first;  // the row's group slot
        const int c4 = threadIdx.x & 15, rg = threadIdx.x >> 4;  // INT4: bytes 4 c4 .., rows 8 rg ..
        const int gsl4 = min((k0 + 8 * rg) / p.gs, p.G - 1) - g_first;
        for (int i = 0; i < n_kb; ++i) {
            const int s = i % STAGES;
            if (!mbar_wait_bounded(full_w(s), (i / STAGES) & 1)) {
                if (lane == 0) atomicOr(p.err, 1);
                ok = false;
                break;
            }
            const unsigned char* st = gbase + s * stage_bytes;
            if constexpr (kInt4) {
                // thread: bytes 4 c4 .. + 3 (columns n0 + 4 c4 .. + 3 low, R + n0 + .. high)
                // of rows 8 rg .. 8 rg + 7, which share one group: the scales and zero
                // points are converted once per stage, not per row.  Half-warps take
                // their rows in opposite parity order (row loads conflict-free).
                const unsigned char* slot =
                    gbase + STAGES * stage_bytes + s * kTScaleStageBytes + gsl4 * kTGroupBytes;
                const float4 sl = *reinterpret_cast<const float4*>(slot + 16 * c4);
                const float4 sh = *reinterpret_cast<const float4*>(slot + 256 + 16 * c4);
                const uint32_t zl = *reinterpret_cast<const uint32_t*>(slot + 512 + 4 * c4);
                const uint32_t zh = *reinterpret_cast<const uint32_t*>(slot + 576 + 4 * c4);
                const uint32_t sl0 = pack_bf16(sl.x, sl.y), sl1 = pack_bf16(sl.z, sl.w);
                const uint32_t sh0 = pack_bf16(sh.x, sh.y), sh1 = pack_bf16(sh.z, sh.w);
                // zero points as bf16 128 + z, two columns per word
                const uint32_t zl0 = lop3_and_or(prmt(zl, 0u, 0x4140u), 0x000F000Fu, 0x43004300u);
                const uint32_t zl1 = lop3_and_or(prmt(zl, 0u, 0x4342u), 0x000F000Fu, 0x43004300u);
                const uint32_t zh0 = lop3_and_or(prmt(zh, 0u, 0x4140u), 0x000F000Fu, 0x43004300u);
                const uint32_t zh1 = lop3_and_or(prmt(zh, 0u, 0x4342u), 0x000F000Fu, 0x43004300u);
                unsigned char* alo = gbase + s * stage_bytes + kTRawBytes + 2 * xbytes;
                unsigned char* ahi = alo + kTABytes;
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    const int rr = 8 * rg + (jj ^ (rg & 1));
                    const uint32_t w = *reinterpret_cast<const uint32_t*>(st + rr * 64 + 4 * c4);
                    // bytes (0, 1) and (2, 3) in the halves of a word; each nibble ORed into
                    // bf16 128.0 is 128 + q exactly, minus 128 + zero exactly, times the scale
                    const uint32_t p0 = prmt(w, 0u, 0x4140u), p1 = prmt(w, 0u, 0x4342u);
                    const uint32_t lo0 = bf2_sub_mul(lop3_and_or(p0, 0x000F000Fu, 0x43004300u), zl0, sl0);
                    const uint32_t lo1 = bf2_sub_mul(lop3_and_or(p1, 0x000F000Fu, 0x43004300u), zl1, sl1);
                    const uint32_t hi0 = bf2_sub_mul(lop3_and_or(p0 >> 4, 0x000F000Fu, 0x43004300u), zh0, sh0);
                    const uint32_t hi1 = bf2_sub_mul(lop3_and_or(p1 >> 4, 0x000F000Fu, 0x43004300u), zh1, sh1);
                    // bf16 columns 4 c4 .. + 3 of row rr: 8 bytes of 16-byte chunk c4 / 2, 128-byte swizzle
                    const uint32_t off =
                        static_cast<uint32_t>(rr * 128 + (((c4 >> 1) ^ (rr & 7)) << 4) + 8 * (c4 & 1));
                    *reinterpret_cast<uint2*>(alo + off) = make_uint2(lo0, lo1);
                    *reinterpret_cast<uint2*>(ahi + off) = make_uint2(hi0, hi1);
                }
            } else {
                // bytes 32 hh .. + 31 of row r: columns n0 + 32 hh + j, each
                // 2^23 + (q + 128) in an fp32 mantissa minus 2^23 + 128 (exactly q),
                // times the column's scale in fp32, rounded to bf16
                const uint4 wa = *reinterpret_cast<const uint4*>(st + r * 64 + 32 * hh);
                const uint4 wb = *reinterpret_cast<const uint4*>(st + r * 64 + 32 * hh + 16);
                const unsigned char* slot = gbase + STAGES * stage_bytes + s * kTScaleStageBytes + gsl * kTGroupBytes;
                const float* sc = reinterpret_cast<const float*>(slot) + 32 * hh;
                const uint32_t wv[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
                uint32_t lo[16];
#pragma unroll
                for (int q = 0; q < 8; ++q) {
#pragma unroll
                    for (int h2 = 0; h2 < 2; ++h2) {
                        const int j = 4 * q + 2 * h2;
                        // byte j (j + 1) of the lane's 32 into the low byte of 0x4B000000
                        const uint32_t b0 = prmt(wv[q], 0x4Bu, static_cast<uint32_t>(2 * h2) | 0x4550u);
                        const uint32_t b1 = prmt(wv[q], 0x4Bu, static_cast<uint32_t>(2 * h2 + 1) | 0x4550u);
                        const float q0 = __uint_as_float(b0 ^ 0x80u) - 8388736.0f;
                        const float q1 = __uint_as_float(b1 ^ 0x80u) - 8388736.0f;
                        const float2 s2 = *reinterpret_cast<const float2*>(sc + j);
                        lo[2 * q + h2] = pack_bf16(__fmul_rn(s2.x, q0), __fmul_rn(s2.y, q1));
                    }
                }
                unsigned char* alo = gbase + s * stage_bytes + kTRawBytes + 2 * xbytes;
#pragma unroll
                for (int c = 0; c < 4; ++c) {  // 16-byte chunk 4 hh + c of row r, 128-byte swizzle
                    const uint32_t off = static_cast<uint32_t>(r * 128 + (((4 * hh + c) ^ (r & 7)) << 4));
                    *reinterpret_cast<uint4*>(alo + off) =
                        make_uint4(lo[4 * c], lo[4 * c + 1], lo[4 * c + 2], lo[4 * c + 3]);
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic stores -> MMA reads
            __syncwarp();
            if (lane == 0) mbar_arrive(full_a(s));
        }
        // output "columns" are rows k0 .. k0 + 127 of dx (the one-accumulator path)
        gemm_epilogue<8>(p, tmem, 0, done, ok, k0, tok0, &s_last);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(p.tmem_cols)
                     : "memory");
    }
}

// Split-K partial tiles [tile][split][nt][columns] summed in split order, then
// c = (accumulate ? c : 0) + alpha * sum + bias (+ LoRA term): the arithmetic,
// in the same order, of the last-CTA reduction in gemm_tc_kernel, spread over
// the whole GPU (thread: 4 adjacent columns of one token of one tile).
template <int BITS>
__global__ void __launch_bounds__(256) split_reduce_kernel(GemmParams p, int tiles_x, int tiles_y, int S) {
    constexpr int kCT = BITS == 4 ? 2 * kTileBytes : kTileBytes;
    constexpr int kQuads = kCT / 4;
    dev::pdl_launch_dependents();
    dev::pdl_wait();  // the partials are the previous kernel's output
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    if (BITS == 4 && p.swiglu) {
        // thread: 4 adjacent bytes of one token of one tile, their gate (low
        // nibble) and up (high nibble) columns (SwiGLU.forwardInto,
        // Tensor.kt:231-237; the arithmetic of kt_silu_mul_rows)
        const int64_t total_b = static_cast<int64_t>(tiles_x) * tiles_y * p.nt * (kTileBytes / 4);
        for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total_b; i += stride) {
            const int q4 = static_cast<int>(i % (kTileBytes / 4)) * 4;
            const int64_t rest = i / (kTileBytes / 4);
            const int t = static_cast<int>(rest % p.nt);
            const int64_t tile_id = rest / p.nt;
            const int bx = static_cast<int>(tile_id % tiles_x);
            const int tok = static_cast<int>(tile_id / tiles_x) * p.nt + t;
            const float* parts = p.partials + tile_id * S * (static_cast<int64_t>(p.nt) * kCT);
            float4 g4 = make_float4(0.f, 0.f, 0.f, 0.f), u4 = g4;
#pragma unroll 4
            for (int sp = 0; sp < S; ++sp) {
                const float* row = parts + (static_cast<int64_t>(sp) * p.nt + t) * kCT;
                const float4 a = __ldcg(reinterpret_cast<const float4*>(row + q4));
                const float4 b = __ldcg(reinterpret_cast<const float4*>(row + kTileBytes + q4));
                g4.x += a.x; g4.y += a.y; g4.z += a.z; g4.w += a.w;
                u4.x += b.x; u4.y += b.y; u4.z += b.z; u4.w += b.w;
            }
            const float gv[4] = {g4.x, g4.y, g4.z, g4.w}, uv[4] = {u4.x, u4.y, u4.z, u4.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int cb = bx * kTileBytes + q4 + j;
                if (cb >= p.R || tok >= p.M) continue;
                float g = fmaf(p.alpha, gv[j], 0.0f), u = fmaf(p.alpha, uv[j], 0.0f);
                if (p.bias != nullptr) {
                    g += p.bias[cb];
                    u += p.bias[p.R + cb];
                }
                if (p.lora.p != nullptr) {
                    g += lora_term(p.lora, tok, cb, p.N);
                    u += lora_term(p.lora, tok, p.R + cb, p.N);
                }
                p.y[static_cast<int64_t>(tok) * p.R + cb] = g / (1.0f + expf(-g)) * u;
            }
        }
        return;
    }
    const int64_t total = static_cast<int64_t>(tiles_x) * tiles_y * p.nt * kQuads;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int q4 = static_cast<int>(i % kQuads) * 4;
        const int64_t rest = i / kQuads;
        const int t = static_cast<int>(rest % p.nt);
        const int64_t tile_id = rest / p.nt;
        const int bx = static_cast<int>(tile_id % tiles_x);
        const int tok = static_cast<int>(tile_id / tiles_x) * p.nt + t;
        const float* parts = p.partials + tile_id * S * (static_cast<int64_t>(p.nt) * kCT);
        float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
        for (int sp = 0; sp < S; ++sp) {
            const float4 u =
                __ldcg(reinterpret_cast<const float4*>(parts + (static_cast<int64_t>(sp) * p.nt + t) * kCT + q4));
            a0.x += u.x; a0.y += u.y; a0.z += u.z; a0.w += u.w;
        }
        const float v[4] = {a0.x, a0.y, a0.z, a0.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int col = q4 + j;
            const int cb = bx * kTileBytes + (col & 127);
            const int oc = (BITS == 4 && col >= 128) ? p.R + cb : cb;
            if (cb >= p.R || oc >= p.N || tok >= p.M) continue;
            float* out = p.y + static_cast<int64_t>(tok) * p.N + oc;
            float r = fmaf(p.alpha, v[j], p.accumulate ? *out : 0.0f);
            if (p.bias != nullptr) r += p.bias[oc];
            if (p.lora.p != nullptr) r += lora_term(p.lora, tok, oc, p.N);
            *out = r;
        }
    }
}

// x (fp32 [M x K]) -> bf16, 8 elements per thread (K % 8 == 0).
__global__ void x_to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ xb, int64_t n8) {
    dev::pdl_launch_dependents();
    dev::pdl_wait();  // x is the previous kernel's output
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i >= n8) return;
    const float4 a = __ldg(reinterpret_cast<const float4*>(x) + 2 * i);
    const float4 b = __ldg(reinterpret_cast<const float4*>(x) + 2 * i + 1);
    uint4 o;
    o.x = pack_bf16(a.x, a.y);
    o.y = pack_bf16(a.z, a.w);
    o.z = pack_bf16(b.x, b.y);
    o.w = pack_bf16(b.z, b.w);
    reinterpret_cast<uint4*>(xb)[i] = o;
}

// RMSNorm.forwardInto (RMSNorm.kt:71-90) of each x row, then bf16: one block
// per row (K % 8 == 0), x * (1 / sqrt(mean(x^2) + eps)) * w rounded once.
__global__ void __launch_bounds__(256) x_to_bf16_norm_kernel(const float* __restrict__ x,
                                                             const float* __restrict__ w, float eps,
                                                             __nv_bfloat16* __restrict__ xb, int K) {
    dev::pdl_launch_dependents();
    dev::pdl_wait();  // x is the previous kernel's output
    __shared__ float red[8];
    const float* xr = x + static_cast<int64_t>(blockIdx.x) * K;
    float ss = 0.0f;
    for (int i = 4 * threadIdx.x; i < K; i += 4 * 256) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(xr + i));
        ss = fmaf(v.x, v.x, ss);
        ss = fmaf(v.y, v.y, ss);
        ss = fmaf(v.z, v.z, ss);
        ss = fmaf(v.w, v.w, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float r = 1.0f / sqrtf(tot / static_cast<float>(K) + eps);
    uint4* out = reinterpret_cast<uint4*>(xb + static_cast<int64_t>(blockIdx.x) * K);
    for (int i = 8 * threadIdx.x; i < K; i += 8 * 256) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(xr + i));
        const float4 b = __ldg(reinterpret_cast<const float4*>(xr + i + 4));
        const float4 wa = __ldg(reinterpret_cast<const float4*>(w + i));
        const float4 wb = __ldg(reinterpret_cast<const float4*>(w + i + 4));
        uint4 o;
        o.x = pack_bf16(a.x * r * wa.x, a.y * r * wa.y);
        o.y = pack_bf16(a.z * r * wa.z, a.w * r * wa.w);
        o.z = pack_bf16(b.x * r * wb.x, b.y * r * wb.y);
        o.w = pack_bf16(b.z * r * wb.z, b.w * r * wb.w);
        out[i / 8] = o;
    }
}

// INT4 weights with the 32-row swizzled TMA descriptor take gemm_ts_kernel up
// to m = 128 (one token tile); above, gemm_tc_kernel's 256-token tiles
// dequantize each weight tile half as often (measured faster at m = 512).
// KT_GEMM_TS=0 keeps every m on gemm_tc_kernel, for comparison.
// Largest m the TMEM-A kernel takes, in token tiles of at most kTsMaxNT
// (KT_GEMM_TS_MAX; default kTsMaxNT: one token tile).
int ts_max_m() {
    static const int v = [] {
        const char* e = std::getenv("KT_GEMM_TS_MAX");
        return e ? std::max(0, std::atoi(e)) : kTsMaxNT;
    }();
    return v;
}
bool use_ts(const QView& w, int m) {
    static const bool on = [] {
        const char* v = std::getenv("KT_GEMM_TS");
        return v == nullptr || std::atoi(v) != 0;
    }();
    return on && w.bits == 4 && w.tmap_mma != nullptr && m <= std::max(kTsMaxNT, ts_max_m());
}

// Tokens per CTA (the MMA's N): m rounded up to 16, at most 256 (128 on the
// TMEM-A kernel).
int nt_for(const QView& w, int m) {
    return std::min(use_ts(w, m) ? kTsMaxNT : kMaxNT, (m + 15) / 16 * 16);
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

// K-splits: up to one CTA per SM, at most kMaxSplits splits of at least
// kMinSplitBlocks K-blocks each (overridable for tuning).
// Measured on B200 with the split reduction on its own kernel: at least 2
// blocks and at most 16 splits was the fastest setting over decode (m 16-64)
// and prefill (m 512) shapes; 8 blocks per split left small weights on a
// handful of SMs (2x slower at m 16-64).
int kMinSplitBlocks = [] { const char* v = std::getenv("KT_GEMM_MIN_SPLIT_BLOCKS"); return v ? std::max(1, std::atoi(v)) : 2; }();
int kMaxSplits = [] { const char* v = std::getenv("KT_GEMM_MAX_SPLITS"); return v ? std::max(1, std::atoi(v)) : 16; }();
int splits_for(const QView& w, int m, int sm_count) {
    const int tiles = (w.bytes_per_row + kTileBytes - 1) / kTileBytes;
    const int ttiles = (m + nt_for(w, m) - 1) / nt_for(w, m);
    const int kb_total = (w.rows + kBK - 1) / kBK;
    int s = std::max(1, sm_count / (tiles * ttiles));
    s = std::min({s, std::max(1, kb_total / kMinSplitBlocks), kMaxSplits});
    if (static_cast<int64_t>(tiles) * ttiles > kTicketCapEach) s = 1;
    return std::min(s, 65535);
}

size_t x_bytes(const QView& w, int m) { return align256(static_cast<size_t>(m) * w.rows * 2); }

// Split-K partials of at least this many token rows x splits per tile are
// summed by split_reduce_kernel instead of the tile's last CTA.  Measured on
// B200, the separate kernel was as fast or faster at every m >= 16 (the last
// CTA of a tile reads S partial tiles alone: 2 MB at m = 512, S = 8), so by
// default it takes every split; a larger value keeps small partials on the
// last-CTA path.
int kReduceKernelMin = [] { const char* v = std::getenv("KT_GEMM_REDUCE_MIN"); return v ? std::max(1, std::atoi(v)) : 16; }();

// cudaLaunchKernelEx with programmatic dependent launch allowed.
template <typename... Params, typename... Args>
cudaError_t launch_chained(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                           Args... args) {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = grid;
    lc.blockDim = block;
    lc.dynamicSmemBytes = smem;
    lc.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    return cudaLaunchKernelEx(&lc, kernel, static_cast<Params>(args)...);
}

}  // namespace

bool gemm_tc_supported(const QView& w, int32_t m, const float* a) {
    if ((w.bits != 4 && w.bits != 8) || m < 9 || w.tmap_raw64 == nullptr) return false;
    if (a != nullptr && reinterpret_cast<uintptr_t>(a) % 16 != 0) return false;
    return w.rows % 8 == 0 && w.group_size % 32 == 0 && w.columns % 32 == 0;
}

bool gemm_swiglu_fused(const QView& w, int32_t m, int sm_count) {
    if (!gemm_tc_supported(w, m, nullptr) || w.bits != 4 || w.columns != 2 * w.bytes_per_row) return false;
    const int S = splits_for(w, m, sm_count);
    return S > 1 && nt_for(w, m) * S >= kReduceKernelMin;
}

size_t gemm_tc_workspace_bytes(const QView& w, int32_t m, int sm_count) {
    const int S = splits_for(w, m, sm_count);
    size_t bytes = kWorkspaceReservedBytes + x_bytes(w, m);
    if (S > 1) {
        const size_t tiles = (w.bytes_per_row + kTileBytes - 1) / kTileBytes;
        const size_t ttiles = (m + nt_for(w, m) - 1) / nt_for(w, m);
        bytes += tiles * ttiles * S * static_cast<size_t>(nt_for(w, m)) * 256 * sizeof(float);
    }
    return bytes;
}

cudaError_t launch_gemm_tc(const QView& w, const MatmulArgs& a, int sm_count, cudaStream_t s, void* workspace,
                           size_t workspace_bytes) {
    if (workspace == nullptr || workspace_bytes < gemm_tc_workspace_bytes(w, a.m, sm_count))
        return cudaErrorInvalidValue;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    __nv_bfloat16* xb = reinterpret_cast<__nv_bfloat16*>(ws + kWorkspaceReservedBytes);
    if (a.swiglu && !gemm_swiglu_fused(w, a.m, sm_count)) return cudaErrorInvalidValue;
    const int64_t n8 = static_cast<int64_t>(a.m) * w.rows / 8;
    cudaError_t e = a.norm_weight != nullptr
                        ? launch_chained(x_to_bf16_norm_kernel, dim3(static_cast<unsigned>(a.m)), dim3(256), 0, s,
                                         a.a, a.norm_weight, a.norm_eps, xb, w.rows)
                        : launch_chained(x_to_bf16_kernel, dim3(static_cast<unsigned>((n8 + 255) / 256)), dim3(256),
                                         0, s, a.a, xb, n8);
    if (e != cudaSuccess) return e;

    GemmParams p{};
    p.scales = w.scales;
    p.zeros = w.zeros;
    p.y = a.c;
    p.bias = a.bias;
    p.err = a.err;
    p.M = a.m;
    p.K = w.rows;
    p.N = w.columns;
    p.R = w.bytes_per_row;
    p.gs = w.group_size;
    p.G = w.groups;
    p.nt = nt_for(w, a.m);
    p.nt_cols = p.nt;
    int cols = 32;
    while (cols < (w.bits == 4 ? 2 : 1) * p.nt) cols *= 2;
    p.tmem_cols = cols;
    // kind::f16: D f32 (bits 4-5 = 1), A bf16 (7-9 = 1), B bf16 (10-12 = 1),
    // both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28.
    p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(p.nt >> 3) << 17) |
              (static_cast<uint32_t>(128 >> 4) << 24);
    p.alpha = a.alpha;
    p.accumulate = a.accumulate;
    p.lora = a.lora;
    const int S = splits_for(w, a.m, sm_count);
    p.tickets = reinterpret_cast<int32_t*>(ws + kGemmTicketOffset);
    p.partials = reinterpret_cast<float*>(ws + kWorkspaceReservedBytes + x_bytes(w, a.m));
    p.reduce_kernel = S > 1 && p.nt * S >= kReduceKernelMin ? 1 : 0;
    p.swiglu = a.swiglu;

    alignas(64) CUtensorMap tmap_x;
    if (!encode_tmap_2d(&tmap_x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, xb, static_cast<uint64_t>(w.rows),
                        static_cast<uint64_t>(a.m), static_cast<uint64_t>(w.rows) * 2, kBK,
                        static_cast<uint32_t>(p.nt), CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    const bool ts = use_ts(w, a.m);
    if (ts) p.nt_cols = kTsAccHi;
    auto kernel = ts ? gemm_ts_kernel : w.bits == 4 ? gemm_tc_kernel<4> : gemm_tc_kernel<8>;
    const size_t smem = ts ? kTsSmemBytes : kSmemBytes;
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const dim3 grid((w.bytes_per_row + kTileBytes - 1) / kTileBytes, (a.m + p.nt - 1) / p.nt, S);
    e = launch_chained(kernel, grid, dim3(ts ? kTsThreads : kThreads), smem, s, ts ? *w.tmap_mma : *w.tmap_raw64,
                       tmap_x, p);
    if (e != cudaSuccess || !p.reduce_kernel) return e;
    const int64_t quads = static_cast<int64_t>(grid.x) * grid.y * p.nt * (p.swiglu ? 32 : w.bits == 4 ? 64 : 32);
    const int blocks = static_cast<int>(std::min<int64_t>((quads + 255) / 256, static_cast<int64_t>(sm_count) * 8));
    return launch_chained(w.bits == 4 ? split_reduce_kernel<4> : split_reduce_kernel<8>, dim3(blocks), dim3(256), 0,
                          s, p, static_cast<int>(grid.x), static_cast<int>(grid.y), S);
}

// ---- the transposed product on tcgen05 (gemm_t_kernel)

bool gemm_t_supported(const QView& w, int32_t m, const float* dy) {
    if (m < 16 || w.rows < 1) return false;
    if (!(w.bits == 4 && w.columns % 128 == 0) && !(w.bits == 8 && w.columns % 64 == 0)) return false;
    if (!(w.group_size == 32 || w.group_size == 64 || w.group_size % 128 == 0)) return false;
    return dy == nullptr || reinterpret_cast<uintptr_t>(dy) % 16 == 0;
}

namespace {
int t_nt(int m) { return std::min(kTMaxNT, (m + 15) / 16 * 16); }
int t_splits(const QView& w, int m, int sm_count) {
    const int tiles = ((w.rows + kTRows - 1) / kTRows) * ((m + t_nt(m) - 1) / t_nt(m));
    const int kb_total = w.columns / (w.bits == 4 ? 128 : 64);  // stages of 64 packed bytes
    int s = std::max(1, sm_count / tiles);
    s = std::min({s, std::max(1, kb_total / kMinSplitBlocks), kMaxSplits});
    if (tiles > kTicketCapEach) s = 1;
    return s;
}
}  // namespace

size_t gemm_t_workspace_bytes(const QView& w, int32_t m, int sm_count) {
    const int S = t_splits(w, m, sm_count);
    size_t bytes = kWorkspaceReservedBytes + align256(static_cast<size_t>(m) * w.columns * 2);
    if (S > 1) {
        const size_t tiles = static_cast<size_t>((w.rows + kTRows - 1) / kTRows) * ((m + t_nt(m) - 1) / t_nt(m));
        bytes += tiles * S * static_cast<size_t>(t_nt(m)) * kTRows * sizeof(float);
    }
    return bytes;
}

cudaError_t launch_gemm_t(const QView& w, const float* dy, float* dx, int32_t m, int32_t accumulate, int32_t* err,
                          int sm_count, cudaStream_t s, void* workspace, size_t workspace_bytes) {
    if (!gemm_t_supported(w, m, dy) || workspace == nullptr ||
        workspace_bytes < gemm_t_workspace_bytes(w, m, sm_count))
        return cudaErrorInvalidValue;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    __nv_bfloat16* dyb = reinterpret_cast<__nv_bfloat16*>(ws + kWorkspaceReservedBytes);
    const int64_t n8 = static_cast<int64_t>(m) * w.columns / 8;
    cudaError_t e = launch_chained(x_to_bf16_kernel, dim3(static_cast<unsigned>((n8 + 255) / 256)), dim3(256), 0, s,
                                   dy, dyb, n8);
    if (e != cudaSuccess) return e;
    GemmParams p{};
    p.scales = w.scales;
    p.zeros = w.zeros;
    p.y = dx;
    p.err = err;
    p.M = m;
    p.K = w.columns;  // the contraction (the weight's columns)
    p.N = w.rows;     // dx's row length: output "columns" are the weight's rows
    p.R = w.rows;
    p.gs = w.group_size;
    p.G = w.groups;
    p.nt = t_nt(m);
    p.nt_cols = p.nt;
    int cols = 32;
    while (cols < p.nt) cols *= 2;
    p.tmem_cols = cols;
    // kind::f16: D f32, A and B bf16, both K-major, N >> 3 at bits 17-22, M >> 4 at bits 24-28
    p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(p.nt >> 3) << 17) |
              (static_cast<uint32_t>(kTRows >> 4) << 24);
    p.alpha = 1.0f;
    p.accumulate = accumulate;
    const int S = t_splits(w, m, sm_count);
    p.tickets = reinterpret_cast<int32_t*>(ws + kGemmTicketOffset);
    p.partials = reinterpret_cast<float*>(ws + kWorkspaceReservedBytes + align256(static_cast<size_t>(m) * w.columns * 2));
    p.reduce_kernel = S > 1 && p.nt * S >= kReduceKernelMin ? 1 : 0;
    alignas(64) CUtensorMap tmap_w, tmap_dy;
    // packed rows as bytes: boxes of 64 bytes x 128 rows, no swizzle (rows read linearly)
    if (!encode_tmap_2d(&tmap_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w.q, static_cast<uint64_t>(w.bytes_per_row),
                        static_cast<uint64_t>(w.rows), static_cast<uint64_t>(w.bytes_per_row), 64, kTRows,
                        CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_tmap_2d(&tmap_dy, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, dyb, static_cast<uint64_t>(w.columns),
                        static_cast<uint64_t>(m), static_cast<uint64_t>(w.columns) * 2, 64, static_cast<uint32_t>(p.nt),
                        CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;
    const bool four = p.nt <= kTMaxNT4;
    auto kernel = w.bits == 4 ? (four ? gemm_t_kernel<4, 4> : gemm_t_kernel<4, kStages>)
                              : (four ? gemm_t_kernel<8, 4> : gemm_t_kernel<8, kStages>);
    const size_t smem = t_smem_bytes(four ? 4 : kStages, p.nt);
    e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    const dim3 grid((w.rows + kTRows - 1) / kTRows, (m + p.nt - 1) / p.nt, S);
    e = launch_chained(kernel, grid, dim3(kThreads), smem, s, tmap_w, tmap_dy, p);
    if (e != cudaSuccess || !p.reduce_kernel) return e;
    const int64_t quads = static_cast<int64_t>(grid.x) * grid.y * p.nt * 32;
    const int blocks = static_cast<int>(std::min<int64_t>((quads + 255) / 256, static_cast<int64_t>(sm_count) * 8));
    return launch_chained(split_reduce_kernel<8>, dim3(blocks), dim3(256), 0, s, p, static_cast<int>(grid.x),
                          static_cast<int>(grid.y), S);
}

}  // namespace kt
