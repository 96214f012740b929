// kt_gemv_mma.cu -- INT4 decode GEMV (m <= 8) with tensor-core products:
// MatMul.multiplyQuantized (Engine/kotensor/src/main/kotlin/MatMul.kt:460-536,
// :599-828) for m = 1..8.
//
// Why tensor cores for a memory-bound GEMV.  B200's HBM streams ~13e12 INT4
// weights/s while its CUDA cores issue ~3.7e13 lane instructions/s; an fp32
// FMA kernel needs >= 2.4 instructions per weight (unpack + FMA) and measured
// 3.4, so it is issue-bound well below the HBM roofline.  Here the products
// run on mma.sync.m16n8k16 (fp16 inputs, fp32 accumulate) and the CUDA cores
// only turn nibbles into fp16 operands: 6 instructions per 256 weights.
//
// Exactness.  The A operand holds the raw nibbles as exact fp16 values with
// no offset: two bytes of two rows are interleaved with PRMT and one AND masks
// each nibble into the low mantissa bits of a zero exponent, the fp16
// subnormal q * 2^-24 (low nibble) or 16 q * 2^-24 (high nibble).  The B
// operand holds x split into two fp16 terms, hi = fp16(x') and lo = fp16(x' -
// hi), with x' = x * 2^s and 2^s a power of two per (slice, token) that puts
// the slice's max|x| in [2^14, 2^15): a 22-bit significand, exact products,
// fp32 accumulation of sum q x' alone.  (An earlier encoding OR-ed the nibble
// into 1024.0h, exact as well, but then the accumulator carried 1024 sum x'
// beside sum q x' and lost ~8 bits to it.)  Each group's accumulator C is
// combined as in the reference (combineGroup, MatMul.kt:804-828):
//     y[j] += scale[g,j] * (2^(24-s) C - zero[g,j] * sum_l x_l)      (low)
//     y[j] += scale[g,j] * (2^(20-s) C - zero[g,j] * sum_l x_l)      (high)
// with sum_l x_l the group's sum of (hi + lo) * 2^-s, i.e. of what the tensor
// cores saw.
//
// Tiling.  A CTA owns 128 packed bytes of every row (INT4: 128 low-nibble and
// 128 high-nibble columns).  Its 16 warps form 8 pairs; each pair owns a
// contiguous K-slice (a multiple of 32 rows) and its two warps the two 64-byte
// halves of the tile row.  A thread-block cluster of CK CTAs along K splits K
// further.  In an m16n8k16 tile, A row g (g = lane/4) is the low nibble of one
// byte and row g+8 the high nibble of the same byte; lane t = lane%4 holds
// k-slots 2t, 2t+1, 2t+8, 2t+9, i.e. those rows of the 16-row step, so a
// thread reads one 8-byte chunk of four rows and feeds 8 MMAs from it.  B
// column n = 2q + part (part 0 = hi, 1 = lo) carries token q % M (tokens are
// replicated when M < 4), so C columns 2t, 2t+1 of lane (g, t) are token t % M.
//
// Activations.  Once per slice the pair loads its rows of x, finds the power
// of two per token, and writes the fp16 terms (padded rows, conflict-free B
// loads) and the 32-row chunk sums of x to shared memory; the weight ring is
// already filling meanwhile.
//
// Streaming.  Each pair owns a ring of kStages stages of 32 rows x 128 bytes,
// filled by one lane with one 2-D TMA copy per stage (128-byte swizzle) plus,
// on the first stage of each group, 1-D bulk copies of that group's scales and
// zero points into a ring of group slots.  A "full" mbarrier per stage tracks
// the copies and an "empty" mbarrier per stage the release by both warps; every
// wait is bounded (globaltimer) and a timeout sets the context's error word and
// drains the copies still in flight before the CTA exits.  The kernel is
// launched with programmatic stream serialization: the weight prefetch overlaps
// the previous kernel, griddepcontrol.wait orders the reads of x and the writes
// of y after it.
//
// Token groups.  One CTA carries at most 4 tokens (the 8 B columns); m = 5..8
// runs as one launch with two groups of CTAs, tokens [0, 4) and [4, m), each
// streaming the weight.  The group is the fastest-varying part of blockIdx.x,
// so the two CTAs of a (tile, split) are scheduled together and the second
// read of the tile mostly hits L2.  A group short of 4 tokens stages zeros for
// the missing ones and writes no row for them.
//
// Reduction order (deterministic, no atomics, no global scratch): group
// partials in registers per thread in row order; the 8 slices of a CTA through
// shared memory in slice order; the CK CTAs of a cluster through distributed
// shared memory in rank order.
#include <cuda_fp16.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>

#include "kt_internal.h"

namespace kt {
namespace {

constexpr int kPairs = 4;               // K-slices per CTA; two warps (column halves) per slice
constexpr int kWarps = 2 * kPairs;
constexpr int kThreads = kWarps * 32;
constexpr int kStep = 16;               // rows per MMA step
constexpr int kRowsPerStage = 32;       // rows per TMA stage (two MMA steps)
constexpr int kTileBytes = 128;         // packed bytes per CTA tile row
constexpr int kStages = 4;              // stages per slice ring (also group slots)
constexpr int kXsRows = 1024;           // token-rows of x a slice stages in shared memory
constexpr uint64_t kWaitLimitNs = 2000000000ull;

constexpr int kStageBytes = kRowsPerStage * kTileBytes;               // 4096
constexpr int kScaleSlotBytes = 2 * kTileBytes * 4 + 2 * kTileBytes;  // 1280
constexpr int kRingBytes = kStages * kStageBytes;                     // per slice
constexpr int kSlotRingBytes = kStages * kScaleSlotBytes;             // per slice
constexpr int kRedBytes = kWarps * 16 * 32 * 4;                       // reuses the rings
constexpr int kMainBytes = kPairs * kRingBytes;
constexpr int kPartBytes = 4 * 2 * kTileBytes * 4;
// Rows of one slice for M tokens (a multiple of 64).
template <int M>
__host__ __device__ constexpr int max_slice_rows() { return kXsRows / M / 64 * 64; }
// staged x per slice: [token][part][stride] fp16; the 8-half pad puts the 8
// (token, part) rows a warp reads at once in different banks
template <int M>
__host__ __device__ constexpr int xs_stride() { return max_slice_rows<M>() + 8; }
template <int M>
__host__ __device__ constexpr int xs_bytes() { return M * 2 * xs_stride<M>() * 2; }
constexpr int kXsBytes = 4224;  // the largest xs_bytes<M>() over M = 1..4
constexpr int kChunkBytes = kXsRows / kRowsPerStage * 4;  // chunk sums [chunk][token]
constexpr int kXmaxBytes = 2 * 4 * 4;                                 // [warp of the pair][token]
constexpr int kXsPairBytes = kXsBytes + kChunkBytes + kXmaxBytes;
constexpr size_t kSmemBytes = static_cast<size_t>(kMainBytes) + kPairs * kSlotRingBytes + kPartBytes +
                              kPairs * kXsPairBytes + kPairs * kStages * 16;
static_assert(kRedBytes <= kMainBytes, "reduction buffer must fit in the rings");
static_assert(kRowsPerStage == 32, "the TMA box of QView::tmap_mma is 32 rows");
static_assert(xs_bytes<1>() <= kXsBytes && xs_bytes<2>() <= kXsBytes && xs_bytes<3>() <= kXsBytes &&
                  xs_bytes<4>() == kXsBytes, "x staging area");
static_assert(kXsPairBytes % 16 == 0, "slice staging areas stay 16-byte aligned");
static_assert(2 * (kSmemBytes + 1024) <= 233472, "two CTAs per SM");

struct MmaParams {
    const float* scales;
    const uint8_t* zeros;
    const float* x;
    float* y;
    const float* bias;
    int32_t* err;
    int32_t K, N, R, gs;
    float alpha;
    int32_t accumulate;
    LoraEpilogue lora;
    // split-K (gridDim.y > 1): per-CTA partial tiles and per-tile arrival
    // counters (zero on entry, left zero on exit)
    float* partials;       // [tiles][groups][splits][M][256]
    int32_t* tickets;      // [tiles][groups]
    int32_t m_total;       // rows of the call (token group z holds rows [4z, min(4z + M, m_total)))
    const float* norm_w;   // RMSNorm of every x row before the product (NULL: off)
    float norm_eps;
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
// 2-D TMA tile load into this CTA's shared memory (no multicast).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
// 1-D bulk copy global -> this CTA's shared memory (no multicast).
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ int atomic_add_acq_rel(int32_t* p, int v) {
    int old;
    asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// The 8 MMAs of one 16-row step from the four 8-byte row chunks w[0..3]
// (rows 2t, 2t+1, 2t+8, 2t+9); MMA i = 4k + j <-> byte 4k + j of the chunk.
// A holds the fp16 subnormals q * 2^-24 (low nibbles) and 16 q * 2^-24 (high
// nibbles); the 2^24 and the 16x are removed in the group epilogue.
__device__ __forceinline__ void mma_step(float (&c)[8][4], const uint2 (&w)[4], uint32_t b0, uint32_t b1) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const uint32_t w0 = (&w[0].x)[k], w1 = (&w[1].x)[k], w2 = (&w[2].x)[k], w3 = (&w[3].x)[k];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t sel = static_cast<uint32_t>(j | ((4 + j) << 8));
            const uint32_t p01 = prmt(w0, w1, sel);  // byte j of rows 2t and 2t+1 at bits 0-7 / 16-23
            const uint32_t p23 = prmt(w2, w3, sel);
            uint32_t a[4];
            a[0] = p01 & 0x000F000Fu;
            a[1] = p01 & 0x00F000F0u;
            a[2] = p23 & 0x000F000Fu;
            a[3] = p23 & 0x00F000F0u;
            mma_16816(c[4 * k + j], a, b0, b1);
        }
    }
}

__device__ __forceinline__ void pair_barrier(int pair) {
    asm volatile("bar.sync %0, 64;" ::"r"(1 + pair) : "memory");
}

// Shared memory: rings[8 slices][NS][32][128] (later red[16][16][32]) |
// slots[8][NS][1280] | part[4][256] | x staging[8][kXsPairBytes] | mbarriers[8][2][NS].
template <int M>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_mma_kernel(const __grid_constant__ CUtensorMap tmap, MmaParams p) {
    extern __shared__ __align__(1024) unsigned char smem[];
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int pair = warp >> 1;  // K-slice of the CTA
    const int hw = warp & 1;     // column half of the 128-byte tile row
    const int g = lane >> 2;     // MMA row group
    const int t = lane & 3;      // MMA k quad: rows 2t, 2t+1, 2t+8, 2t+9; token t of C
    const int gb = 8 * hw + g;   // this lane's 8-byte chunk of the tile row
    const int groups = (p.m_total + 3) / 4;                 // token groups (1 unless M == 4 and m > 4)
    const int tile_b0 = static_cast<int>(blockIdx.x) / groups * kTileBytes;
    const int tile_cols = min(kTileBytes, p.R - tile_b0);  // packed bytes of this tile inside the row
    const int half = p.R;
    const int row0 = 4 * (static_cast<int>(blockIdx.x) % groups);  // first row (token) of this CTA's group
    const int mv = min(M, p.m_total - row0);                // tokens of the group that exist

    // K-slices: the K/32 stages spread evenly over splits x kPairs slices
    // (the host keeps every slice within max_slice_rows<M>())
    const int n_slices = gridDim.y * kPairs;
    const int slice = blockIdx.y * kPairs + pair;
    const int k_stages = p.K / kRowsPerStage;
    const int s_begin = static_cast<int>(static_cast<int64_t>(slice) * k_stages / n_slices);
    const int s_end = static_cast<int>(static_cast<int64_t>(slice + 1) * k_stages / n_slices);
    const int r_begin = s_begin * kRowsPerStage;
    const int r_end = s_end * kRowsPerStage;
    const int n_stages = s_end - s_begin;

    unsigned char* ring = smem + pair * kRingBytes;
    unsigned char* slots = smem + kMainBytes + pair * kSlotRingBytes;
    float* part = reinterpret_cast<float*>(smem + kMainBytes + kPairs * kSlotRingBytes);
    unsigned char* xstage = smem + kMainBytes + kPairs * kSlotRingBytes + kPartBytes + pair * kXsPairBytes;
    __half* xs = reinterpret_cast<__half*>(xstage);                      // [token][part][kXsStride]
    float* chunk_sum = reinterpret_cast<float*>(xstage + kXsBytes);       // [chunk][M]
    float* xmax = reinterpret_cast<float*>(xstage + kXsBytes + kChunkBytes);  // [2][4]
    // per slice: "full" mbarriers (TMA completion) then "empty" mbarriers (both warps released the slot)
    const uint32_t bars =
        smem_u32(smem + kMainBytes + kPairs * kSlotRingBytes + kPartBytes + kPairs * kXsPairBytes) +
        pair * kStages * 16;
    const uint32_t empty = bars + kStages * 8;
    const uint32_t ring_s = smem_u32(ring);
    const uint32_t slots_s = smem_u32(slots);
    const int g_first = r_begin / p.gs;
    const bool producer = hw == 0 && lane == 0;

    if (producer) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(bars + 8 * s, 1);
            mbar_init(empty + 8 * s, 2);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    // Stage st: rows [r_begin + 32 st, +32) into ring slot st % NS; a stage that
    // starts a group (or the slice) also brings the group's scales and zero
    // points into group slot (group - g_first) % NS.
    // Producer state: the next stage's first row, the next group to fetch and
    // the row where it starts (the slice's first stage always fetches).
    int p_row = r_begin, p_gi = g_first, p_gstart = r_begin, p_issued = 0;
    // Issued by the whole warp 0 of the pair, stages in order: lane 0 arms the
    // stage's mbarrier and copies the weights, lanes 1-4 copy a new group's
    // low / high scales and zero points (complete_tx before the arming
    // arrive cannot complete the phase: the arrive is still pending).
    const uint32_t sbytes = static_cast<uint32_t>(tile_cols) * 10;  // 2 x fp32 scales + 2 x u8 zeros
    const uint32_t lane_off = lane <= 2 ? (lane - 1) * kTileBytes * 4 : kTileBytes * (5 + lane);
    const uint32_t lane_bytes = lane <= 2 ? tile_cols * 4 : tile_cols;
    const unsigned char* lane_src =
        lane <= 2 ? reinterpret_cast<const unsigned char*>(p.scales + tile_b0 + (lane == 2 ? half : 0))
                  : p.zeros + tile_b0 + (lane == 4 ? half : 0);
    const int lane_esize = lane <= 2 ? 4 : 1;
    auto issue = [&](int st) {
        const int slot = st & (kStages - 1);
        const uint32_t bar = bars + 8 * slot;
        const bool group_start = p_row == p_gstart;
        if (lane == 0) {
            mbar_expect_tx(bar, kStageBytes + (group_start ? sbytes : 0));
            tma_load_2d(ring_s + slot * kStageBytes, &tmap, tile_b0, p_row, bar);
        }
        if (group_start) {
            if (lane >= 1 && lane <= 4) {
                const uint32_t dst = slots_s + ((p_gi - g_first) & (kStages - 1)) * kScaleSlotBytes + lane_off;
                bulk_load(dst, lane_src + static_cast<int64_t>(p_gi) * p.N * lane_esize, lane_bytes, bar);
            }
            ++p_gi;
            p_gstart = p_gi * p.gs;
        }
        p_row += kRowsPerStage;
        ++p_issued;
    };
    if (hw == 0) {
        for (int s = 0; s < kStages && s < n_stages; ++s) issue(s);  // the whole ring, before the wait
    }
    pdl_launch_dependents();
    pdl_wait();  // x and y below may belong to the previous kernel

    // RMSNorm prologue (p.norm_w; RMSNorm.forwardInto, RMSNorm.kt:71-90): every
    // CTA sums the squares of its tokens' whole rows (the same order in every
    // CTA, so all of them get the same scale) and stages x * scale * w.
    float nrm[M];
#pragma unroll
    for (int m = 0; m < M; ++m) nrm[m] = 1.0f;
    if (p.norm_w != nullptr) {
        __shared__ float s_nred[kWarps][4];
        float ss[M];
#pragma unroll
        for (int m = 0; m < M; ++m) {
            ss[m] = 0.0f;
            if (m >= mv) continue;
            const float* xr = p.x + static_cast<int64_t>(row0 + m) * p.K;
#pragma unroll 4
            for (int i = 4 * tid; i < p.K; i += 4 * kThreads) {
                const float4 v4 = __ldg(reinterpret_cast<const float4*>(xr + i));
                ss[m] = fmaf(v4.x, v4.x, ss[m]);
                ss[m] = fmaf(v4.y, v4.y, ss[m]);
                ss[m] = fmaf(v4.z, v4.z, ss[m]);
                ss[m] = fmaf(v4.w, v4.w, ss[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss[m] += __shfl_xor_sync(0xffffffffu, ss[m], o);
            if (lane == 0) s_nred[warp][m] = ss[m];
        }
        __syncthreads();
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float tot = 0.0f;
#pragma unroll
            for (int w2 = 0; w2 < kWarps; ++w2) tot += s_nred[w2][m];
            nrm[m] = 1.0f / sqrtf(tot / static_cast<float>(p.K) + p.norm_eps);
        }
    }

    // Stage this slice's rows of x: thread pt of the pair holds rows pt + 64 j.
    const int pt = hw * 32 + lane;
    const int n_rows = r_end - r_begin;
    constexpr int kPer = max_slice_rows<M>() / 64;
    constexpr int kXsStride = xs_stride<M>();
    float xv[M][kPer];
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const float* xm = p.x + static_cast<int64_t>(row0 + m) * p.K + r_begin;
        float mx = 0.0f;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int r = pt + 64 * j;
            xv[m][j] = r < n_rows && m < mv ? __ldg(xm + r) : 0.0f;
            if (p.norm_w != nullptr && r < n_rows) xv[m][j] = xv[m][j] * nrm[m] * __ldg(p.norm_w + r_begin + r);
            mx = fmaxf(mx, fabsf(xv[m][j]));
            if (64 * (j + 1) >= n_rows) break;  // pair-uniform
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        if (lane == 0) xmax[hw * 4 + m] = mx;
    }
    pair_barrier(pair);  // mbarrier init and the two warps' maxima
    float unscale[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const float mx = fmaxf(xmax[m], xmax[4 + m]);
        int sh = 14 - (mx > 0.0f ? ilogbf(mx) : 0);
        sh = max(-126, min(126, sh));
        const float sc = ldexpf(1.0f, sh);
        unscale[m] = ldexpf(1.0f, -sh);
        __half* hi = xs + (2 * m) * kXsStride;
        __half* lo = hi + kXsStride;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            if (64 * j >= n_rows) break;  // pair-uniform
            const int r = pt + 64 * j;
            const float v = xv[m][j] * sc;
            const __half h = __float2half_rn(v);
            const __half l = __float2half_rn(v - __half2float(h));
            if (r < n_rows) {
                hi[r] = h;
                lo[r] = l;
            }
            // chunk 2j + hw: the 32 rows this warp holds, summed in butterfly order
            float s = __half2float(h) + __half2float(l);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            if (lane == 0 && 64 * j + 32 * hw < n_rows) chunk_sum[(2 * j + hw) * M + m] = s * unscale[m];
        }
    }
    pair_barrier(pair);  // staged x visible to both warps of the pair

    // B column n = 2 q + part (q = g/2, part = g%2: 0 = hi, 1 = lo) carries
    // token q % M: with M < 4 each token is replicated into kRep column pairs,
    // so the C columns 2t, 2t+1 of every lane t hold token t % M and the kRep
    // lanes of a token split the group epilogue's columns between them.
    // (M == 3 leaves q = 3 / lane t = 3 unused: B is 0 there.)
    constexpr int kRep = M == 1 ? 4 : (M == 2 ? 2 : 1);
    const int q = g >> 1;
    const int btok = q % M;
    const bool b_active = q < kRep * M;
    const __half* xb = xs + (2 * btok + (g & 1)) * kXsStride;
    const int ttok = t % M;
    const bool t_active = t < kRep * M;
    const int sub = t / M;  // which share of the columns this lane finishes
    float un_t = unscale[0];
#pragma unroll
    for (int m = 1; m < M; ++m)
        if (ttok == m) un_t = unscale[m];
    // This lane's four rows inside a step and their swizzled 8-byte offsets:
    // 16-byte chunk gb/2 of row r sits at chunk (gb/2) ^ (r & 7).
    int roff[4], soff[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        roff[i] = 2 * t + (i & 1) + 8 * (i >> 1);
        soff[i] = roff[i] * kTileBytes + (((gb >> 1) ^ (roff[i] & 7)) << 4) + 8 * (gb & 1);
    }

    // token t % M, bytes [sub*NB, (sub+1)*NB) of the chunk: [0,NB) low-nibble
    // columns, [NB,2NB) high-nibble columns
    constexpr int kNB = 8 / kRep;
    float y[2 * kNB];
#pragma unroll
    for (int j = 0; j < 2 * kNB; ++j) y[j] = 0.0f;
    float c[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i][0] = c[i][1] = c[i][2] = c[i][3] = 0.0f;

    float rs = 0.0f;  // this token's sum of x over the group's rows in this slice
    bool ok = true;
    int done = 0;     // stages whose copies this lane saw complete
    int gi = g_first;
    int group_end = min((gi + 1) * p.gs, r_end);
    const bool one_stage_groups = p.gs == kRowsPerStage;
    for (int st = 0; st < n_stages; ++st) {
        const int slot = st & (kStages - 1);
        if (ok) {
            if (mbar_wait_bounded(bars + 8 * slot, (st / kStages) & 1)) {
                done = st + 1;
            } else {
                ok = false;
                atomicOr(p.err, 1);
            }
            ok = __all_sync(0xffffffffu, ok);  // the warp stops waiting together
        }
        if (hw == 0 && st > 0 && st + kStages - 1 < n_stages) {
            // stage st + NS - 1 goes into the slot of stage st - 1 once both
            // warps have released that stage (lane 0 waits for the warp)
            const int prev = st - 1;
            int go = 0;
            if (lane == 0 && ok) go = mbar_wait_bounded(empty + 8 * (prev & (kStages - 1)), (prev / kStages) & 1) ? 1 : 2;
            go = __shfl_sync(0xffffffffu, go, 0);
            if (go == 2) {
                ok = false;
                if (lane == 0) atomicOr(p.err, 1);
            } else if (go == 1) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue(st + kStages - 1);
            }
        }
        const unsigned char* stage = ring + slot * kStageBytes;
#pragma unroll
        for (int ks = 0; ks < kRowsPerStage / kStep; ++ks) {
            const int row0 = st * kRowsPerStage + ks * kStep;  // inside the slice
            // rows 2t, 2t+1 and 2t+8, 2t+9 are adjacent fp16 pairs: two 4-byte loads
            uint32_t b0 = *reinterpret_cast<const uint32_t*>(xb + row0 + roff[0]);
            uint32_t b1 = *reinterpret_cast<const uint32_t*>(xb + row0 + roff[2]);
            if constexpr (M == 3) {
                if (!b_active) b0 = b1 = 0u;
            }
            uint2 w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                w[i] = *reinterpret_cast<const uint2*>(stage + ks * kStep * kTileBytes + soff[i]);
            mma_step(c, w, b0, b1);
        }
        // Release the stage once every lane of this warp has read it; with groups
        // of one stage only after the group epilogue below, which reads the
        // group's scale slot -- the slot the refill of stage st + NS reuses.
        if (!one_stage_groups) {
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + 8 * slot);
        }
        rs += chunk_sum[st * M + ttok];
        if (r_begin + (st + 1) * kRowsPerStage >= group_end) {
            // Group epilogue for token t:
            //   low:  y += scale * (2^(24-s) C - zero rowSum)
            //   high: y += scale * (2^(20-s) C - zero rowSum)
            // Columns beyond the tile's bytes hold stale slot data; their
            // outputs are never written.
            if (t_active) {
                // this lane's share: bytes [i0, i0 + NB) of its 8-byte chunk
                const int i0 = sub * kNB;
                float cs[kNB][4];
#pragma unroll
                for (int e = 0; e < kNB; ++e)
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        float v = c[e][k];
#pragma unroll
                        for (int s = 1; s < kRep; ++s)
                            if (sub == s) v = c[s * kNB + e][k];
                        cs[e][k] = v;
                    }
                const unsigned char* sl = slots + ((gi - g_first) & (kStages - 1)) * kScaleSlotBytes;
                const float* s_lo = reinterpret_cast<const float*>(sl) + 8 * gb + i0;
                const float* s_hi = reinterpret_cast<const float*>(sl + kTileBytes * 4) + 8 * gb + i0;
                const uint8_t* z_lo = sl + kTileBytes * 8 + 8 * gb + i0;
                const uint8_t* z_hi = sl + kTileBytes * 9 + 8 * gb + i0;
                const float un_lo = un_t * 16777216.0f, un_hi = un_t * 1048576.0f;  // 2^24, 2^20 (exact)
#pragma unroll
                for (int e = 0; e < kNB; ++e) {
                    const float zlf = static_cast<float>(z_lo[e]), zhf = static_cast<float>(z_hi[e]);
                    y[e] = fmaf(s_lo[e], fmaf(cs[e][0] + cs[e][1], un_lo, -zlf * rs), y[e]);
                    y[kNB + e] = fmaf(s_hi[e], fmaf(cs[e][2] + cs[e][3], un_hi, -zhf * rs), y[kNB + e]);
                }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) c[i][0] = c[i][1] = c[i][2] = c[i][3] = 0.0f;
            rs = 0.0f;
            ++gi;
            group_end = min((gi + 1) * p.gs, r_end);
        }
        if (one_stage_groups) {
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + 8 * slot);
        }
    }
    // After a timeout: wait (bounded) for this slice's copies still in flight
    // before the rings are reused and before the CTA's shared memory is released.
    if (producer) {
        for (int s = done; s < p_issued; ++s) {
            if (!mbar_wait_bounded(bars + 8 * (s & (kStages - 1)), (s / kStages) & 1)) break;
        }
    }

    // (1) slices of the CTA in order; red[w][e][lane] reuses the rings.
    __syncthreads();
    float* red = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int e = 0; e < 2 * kNB; ++e) red[(warp * 2 * kNB + e) * 32 + lane] = y[e];
    __syncthreads();
    constexpr int CT = 2 * kTileBytes;  // 256 columns per tile: [0,128) low, [128,256) high
    for (int idx = tid; idx < M * CT; idx += kThreads) {
        const int m = idx / CT, col = idx % CT;
        const int hi = col >= kTileBytes;
        const int cb = hi ? col - kTileBytes : col;  // byte of the tile row
        const int cgb = cb >> 3, i = cb & 7;
        const int e = (hi ? kNB : 0) + i % kNB;
        const int ln = 4 * (cgb & 7) + m + M * (i / kNB);
        const int hw_c = cgb >> 3;
        float v = 0.0f;
#pragma unroll
        for (int pr = 0; pr < kPairs; ++pr) v += red[((2 * pr + hw_c) * 2 * kNB + e) * 32 + ln];
        part[idx] = v;
    }
    __syncthreads();  // part[] complete
    auto emit = [&](int idx, float v) {
        const int m = idx / CT, col = idx % CT;
        const int byte = tile_b0 + (col < kTileBytes ? col : col - kTileBytes);
        const int out_col = col < kTileBytes ? byte : half + byte;
        if (m < mv && byte < p.R && out_col < p.N) {
            float* out = p.y + static_cast<int64_t>(row0 + m) * p.N + out_col;
            float r = fmaf(p.alpha, v, p.accumulate ? *out : 0.0f);
            if (p.bias != nullptr) r += p.bias[out_col];
            if (p.lora.p != nullptr) r += lora_term(p.lora, row0 + m, out_col, p.N);
            *out = r;
        }
    };
    const int S = gridDim.y;
    if (S == 1) {
        for (int idx = tid; idx < M * CT; idx += kThreads) emit(idx, part[idx]);
        return;
    }
    // (2) split-K: every CTA of the tile publishes its partial tile; the last
    // to arrive sums all of them in split order and writes y.
    // The CTA barrier orders every thread's partial stores before thread 0's
    // acq_rel atomic (fence cumulativity), which publishes them at GPU scope
    // and, in the last CTA, acquires the other CTAs' partials for the whole
    // CTA through the second barrier.
    __shared__ int s_last;
    const int ticket = blockIdx.x;  // (tile, group)
    float* tile_parts = p.partials + static_cast<int64_t>(ticket) * S * (M * CT);
    float* mine = tile_parts + static_cast<int64_t>(blockIdx.y) * (M * CT);
    for (int idx = tid; idx < M * CT; idx += kThreads) __stcg(mine + idx, part[idx]);
    __syncthreads();
    if (tid == 0) s_last = atomic_add_acq_rel(p.tickets + ticket, 1) == S - 1;
    __syncthreads();
    if (!s_last) return;
    for (int idx = tid; idx < M * CT; idx += kThreads) {
        // issue the loads of up to 8 splits before summing them in split order
        float v = 0.0f;
        for (int s0 = 0; s0 < S; s0 += 8) {
            float t[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                t[j] = s0 + j < S ? __ldcg(tile_parts + static_cast<int64_t>(s0 + j) * (M * CT) + idx) : 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (s0 + j < S) v += t[j];
        }
        emit(idx, v);
    }
    if (tid == 0) p.tickets[ticket] = 0;  // ready for the next launch on this workspace
}

struct MmaOverrides {
    std::atomic<int> splits;
};
MmaOverrides& mma_overrides() {
    static MmaOverrides o{{[] {
        const char* v = std::getenv("KT_MMA_SPLITS");
        return v ? std::atoi(v) : 0;
    }()}};
    return o;
}

// CTAs of this kernel one SM holds (cached per device).
int blocks_per_sm() {
    constexpr int kMaxDevices = 64;
    static std::atomic<int> cache[kMaxDevices] = {};  // host threads may race here
    int dev = 0;
    cudaGetDevice(&dev);
    std::atomic<int>* slot = dev >= 0 && dev < kMaxDevices ? &cache[dev] : nullptr;
    if (slot != nullptr) {
        const int c = slot->load(std::memory_order_acquire);
        if (c != 0) return c;
    }
    int n = 0;
    auto kernel = gemv_mma_kernel<1>;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes)) !=
            cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kThreads, kSmemBytes) != cudaSuccess)
        n = 1;
    cudaGetLastError();
    n = std::max(n, 1);
    if (slot != nullptr) slot->store(n, std::memory_order_release);
    return n;
}

int tiles_of(int R) { return (R + kTileBytes - 1) / kTileBytes; }

// Workspace layout: the arrival counters sit at a fixed offset in the
// reserved front (so no launch's partial tiles ever land where another launch
// keeps its counters) | partial tiles after the reserved front.
constexpr int kTicketCap = kTicketCapEach;
constexpr size_t kTicketBytes = kWorkspaceReservedBytes;

// CTA groups along grid z (4 tokens each) and tokens per CTA of a call with m rows.
int groups_of(int m) { return (m + 3) / 4; }
int m_per_cta(int m) { return std::min(m, 4); }

int max_slice_rows_of(int m) {
    switch (m) {
        case 1: return max_slice_rows<1>();
        case 2: return max_slice_rows<2>();
        case 3: return max_slice_rows<3>();
        default: return max_slice_rows<4>();
    }
}

// Fewest K-splits that keep every slice within max_slice_rows.
int min_splits(int K, int m) {
    const int per = kPairs * max_slice_rows_of(m);
    return (K + per - 1) / per;
}

// K-splits per column tile: enough CTAs (over every token group) to fill every
// SM slot in one wave (at least one stage per slice), at most kMaxSplits (the
// tile's last CTA reads every split's partial tile: 37 splits of a 4-token tile
// are 150 KB), never fewer than min_splits.
constexpr int kMaxSplits = 16;
int choose_splits(int R, int K, int m, int sm_count) {
    const int tiles = tiles_of(R) * groups_of(m);
    const int slots = blocks_per_sm() * sm_count;
    const int k_stages = K / kRowsPerStage;
    int s = std::min(kMaxSplits, std::max(1, slots / tiles));
    s = std::min(s, std::max(1, k_stages / kPairs));
    const int o = mma_overrides().splits.load(std::memory_order_relaxed);
    if (o >= 1) s = o;
    s = std::max(s, min_splits(K, m));
    return tiles > kTicketCap ? min_splits(K, m) : s;
}

template <int M>
cudaError_t launch_m(const QView& w, const MmaParams& p, int splits, int groups, cudaStream_t s) {
    auto kernel = gemv_mma_kernel<M>;
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(tiles_of(p.R) * groups, splits, 1);
    lc.blockDim = dim3(kThreads, 1, 1);
    lc.dynamicSmemBytes = kSmemBytes;
    lc.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    return cudaLaunchKernelEx(&lc, kernel, *w.tmap_mma, p);
}

}  // namespace

void set_mma_tuning(int k_splits) { mma_overrides().splits.store(k_splits, std::memory_order_relaxed); }

bool gemv_mma_supported(const QView& w, int32_t m, const float* a) {
    (void)a;
    if (w.bits != 4 || m < 1 || m > kGemvMmaMaxM || w.tmap_mma == nullptr) return false;
    return w.columns % 32 == 0 && w.rows % kRowsPerStage == 0 && w.group_size % kRowsPerStage == 0 &&
           min_splits(w.rows, m) <= 65535 &&
           (min_splits(w.rows, m) == 1 || tiles_of(w.bytes_per_row) * groups_of(m) <= kTicketCap);
}

size_t gemv_mma_workspace_bytes(const QView& w, int32_t m, int sm_count) {
    const int splits = choose_splits(w.bytes_per_row, w.rows, m, sm_count);
    if (splits <= 1) return 0;
    const size_t tiles = static_cast<size_t>(tiles_of(w.bytes_per_row)) * groups_of(m);
    return kTicketBytes + tiles * splits * static_cast<size_t>(m_per_cta(m)) * 2 * kTileBytes * sizeof(float);
}

cudaError_t launch_gemv_mma(const QView& w, const MatmulArgs& a, int sm_count, cudaStream_t s, void* workspace,
                            size_t workspace_bytes) {
    MmaParams p{};
    p.scales = w.scales;
    p.zeros = w.zeros;
    p.x = a.a;
    p.y = a.c;
    p.bias = a.bias;
    p.err = a.err;
    p.K = w.rows;
    p.N = w.columns;
    p.R = w.bytes_per_row;
    p.gs = w.group_size;
    p.alpha = a.alpha;
    p.accumulate = a.accumulate;
    p.lora = a.lora;
    p.m_total = a.m;
    p.norm_w = a.norm_weight;
    p.norm_eps = a.norm_eps;
    const int splits = choose_splits(p.R, p.K, a.m, sm_count);
    const int groups = groups_of(a.m);
    if (splits > 1) {
        if (workspace == nullptr || workspace_bytes < gemv_mma_workspace_bytes(w, a.m, sm_count))
            return cudaErrorInvalidValue;
        p.tickets = reinterpret_cast<int32_t*>(static_cast<unsigned char*>(workspace) + kGemvTicketOffset);
        p.partials = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + kTicketBytes);
    }
    if (a.m < 1 || a.m > kGemvMmaMaxM) return cudaErrorInvalidValue;
    switch (m_per_cta(a.m)) {
        case 1: return launch_m<1>(w, p, splits, groups, s);
        case 2: return launch_m<2>(w, p, splits, groups, s);
        case 3: return launch_m<3>(w, p, splits, groups, s);
        default: return launch_m<4>(w, p, splits, groups, s);
    }
}

}  // namespace kt
