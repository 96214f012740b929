// kt_gemv_mma.cu -- INT4 decode GEMV (m <= 4) with tensor-core products:
// MatMul.multiplyQuantized (Engine/kotensor/src/main/kotlin/MatMul.kt:460-536,
// :599-828) for m = 1..4.
//
// Why tensor cores for a memory-bound GEMV.  B200's HBM streams ~13e12 INT4
// weights/s while its CUDA cores issue ~3.7e13 lane instructions/s; an fp32
// FMA kernel needs >= 2.4 instructions per weight (unpack + FMA) and measured
// 3.4, so it is issue-bound well below the HBM roofline.  Here the products
// run on mma.sync.m16n8k16 (fp16 inputs, fp32 accumulate) and the CUDA cores
// only turn nibbles into fp16 operands: 10 instructions per 8 weights.
//
// Exactness.  The A operand holds the raw nibbles q as fp16 integers 0..15
// (exact): two bytes of two rows are interleaved with PRMT, LOP3 masks each
// nibble into the mantissa of 1024.0h (0x6400), and one f16x2 op removes the
// 1024 (and the 16x of the high nibble) exactly.  The B operand holds x split
// into two fp16 terms, hi = fp16(x') and lo = fp16(x' - hi), with
// x' = x * 2^s scaled by a power of two per (warp slice, row of x) so hi is in
// [2^14, 2^15) for the largest |x| -- a 22-bit significand, products exact,
// fp32 accumulation.  Each group's accumulator is then combined as in the
// reference (combineGroup, MatMul.kt:804-828):
//     y[j] += scale[g,j] * (2^-s * (C_hi + C_lo) - zero[g,j] * sum_l x_l)
// with sum_l x_l accumulated in fp32 from the unscaled x.
//
// Tiling.  A CTA owns 128 packed bytes of every row (INT4: 128 low-nibble
// columns and 128 high-nibble columns) and 8 warps split K into contiguous
// slices (multiples of 16 rows); a thread-block cluster of CK CTAs along K
// splits it further.  In an m16n8k16 tile, A row g (g = lane/4) is the low
// nibble of one byte and row g+8 the high nibble of the same byte; lane
// t = lane%4 holds k-slots 2t, 2t+1, 2t+8, 2t+9, i.e. those rows of the
// 16-row step, so a thread reads one 16-byte chunk of four rows and feeds 16
// MMAs from it (with the 128-byte swizzle, the 8 lanes of each shared-load
// phase hit 8 different bank groups).  B column n = 2*token + part
// (part 0 = hi, 1 = lo), so C columns 2t, 2t+1 of lane (g, t) are token t.
//
// Streaming.  Each warp owns a ring of kStages stages of 32 rows x 128 bytes,
// filled by lane 0 with one 2-D TMA copy per stage (128-byte swizzle) plus, on
// the first stage of each group, 1-D bulk copies of that group's scales and
// zero points into a per-warp ring of group slots.  Completion is tracked by one mbarrier per
// stage; every wait is bounded (globaltimer) and a timeout sets the context's
// error word.  The kernel is launched with programmatic stream serialization:
// the weight prefetch overlaps the previous kernel, griddepcontrol.wait orders
// the reads of x and the writes of y after it.
//
// Reduction order (deterministic, no atomics, no global scratch): group
// partials in registers per thread in row order; the 8 warps of a CTA through
// shared memory in warp order; the CK CTAs of a cluster through distributed
// shared memory in rank order.
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>

#include "kt_internal.h"

namespace cg = cooperative_groups;

namespace kt {
namespace {

constexpr int kPairs = 8;               // K-slices per CTA; two warps (column halves) per slice
constexpr int kWarps = 2 * kPairs;
constexpr int kThreads = kWarps * 32;
constexpr int kStep = 16;               // rows per MMA step
constexpr int kRowsPerStage = 32;       // rows per TMA stage (two MMA steps)
constexpr int kTileBytes = 128;         // packed bytes per CTA tile row
constexpr int kStages = 4;              // stages per slice ring (also group slots)
constexpr int kMaxSliceGroups = 128;
constexpr uint64_t kWaitLimitNs = 2000000000ull;

constexpr int kStageBytes = kRowsPerStage * kTileBytes;               // 4096
constexpr int kScaleSlotBytes = 2 * kTileBytes * 4 + 2 * kTileBytes;  // 1280
constexpr int kRingBytes = kStages * kStageBytes;                     // per slice
constexpr int kSlotRingBytes = kStages * kScaleSlotBytes;             // per slice
constexpr int kRsBytes = kMaxSliceGroups * 4 * 4;                     // per slice: rowsums [group][token]
constexpr int kRedBytes = kWarps * 16 * 32 * 4;                       // reuses the rings
constexpr int kMainBytes = kPairs * kRingBytes;
constexpr int kPartBytes = 4 * 2 * kTileBytes * 4;
constexpr size_t kSmemBytes = static_cast<size_t>(kMainBytes) + kPairs * kSlotRingBytes + kPairs * kRsBytes +
                              kPartBytes + kPairs * kStages * 16;
static_assert(kRedBytes <= kMainBytes, "reduction buffer must fit in the rings");
static_assert(kRowsPerStage == 32, "the TMA box of QView::tmap_mma is 32 rows");


struct MmaParams {
    const float* scales;
    const uint8_t* zeros;
    const float* x;
    float* y;
    const float* bias;
    int32_t* err;
    int32_t K, N, R, gs;
    int32_t slice_rows;    // multiple of kRowsPerStage
    uint32_t h1024;        // 0x64006400: f16x2 {1024, 1024}
    float alpha;
    int32_t accumulate;
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
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

template <uint32_t MASK>
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "n"(MASK), "r"(c));
    return d;
}
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
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}



// A fragments of the 16 MMAs of one 16-row step from the four 16-byte row
// chunks w[0..3] (rows 2t, 2t+1, 2t+8, 2t+9), MMA i = 4k + j <-> byte 4k + j.
// Two-term fp16 split of (v0, v1): the hi pair fp16(v) or the lo pair fp16(v - hi).
__device__ __forceinline__ uint32_t split_part(float v0, float v1, bool lo) {
    const __half2 h = __floats2half2_rn(v0, v1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(v0 - hf.x, v1 - hf.y);
    const __half2 r = lo ? l : h;
    return *reinterpret_cast<const uint32_t*>(&r);
}

// The 8 MMAs of one 16-row step from the four 8-byte row chunks w[0..3]
// (rows 2t, 2t+1, 2t+8, 2t+9); MMA i = 4k + j <-> byte 4k + j of the chunk.
// A holds {1024 + q} (low nibbles) and {1024 + 16 q} (high nibbles), exact in
// fp16; the 1024 offset and the 16x are removed in the group epilogue.
__device__ __forceinline__ void mma_step(float (&c)[8][4], const uint2 (&w)[4], uint32_t b0, uint32_t b1,
                                         uint32_t h1024) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
        const uint32_t w0 = (&w[0].x)[k], w1 = (&w[1].x)[k], w2 = (&w[2].x)[k], w3 = (&w[3].x)[k];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t sel = static_cast<uint32_t>(j | ((4 + j) << 8));
            const uint32_t p01 = prmt(w0, w1, sel);  // byte j of rows 2t and 2t+1 at bits 0-7 / 16-23
            const uint32_t p23 = prmt(w2, w3, sel);
            uint32_t a[4];
            a[0] = lop3_and_or<0x000F000Fu>(p01, h1024);
            a[1] = lop3_and_or<0x00F000F0u>(p01, h1024);
            a[2] = lop3_and_or<0x000F000Fu>(p23, h1024);
            a[3] = lop3_and_or<0x00F000F0u>(p23, h1024);
            mma_16816(c[4 * k + j], a, b0, b1);
        }
    }
}

__device__ __forceinline__ void pair_barrier(int pair) {
    asm volatile("bar.sync %0, 64;" ::"r"(1 + pair) : "memory");
}

// Shared memory: rings[8 slices][NS][32][128] (later red[16][16][32]) |
// slots[8][NS][1280] | rowsum[8][128][4] | part[4][256] | mbarriers[8][NS].
template <int M>
__global__ void __launch_bounds__(kThreads, 1)
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
    const int tile_b0 = blockIdx.x * kTileBytes;
    const int tile_cols = min(kTileBytes, p.R - tile_b0);  // packed bytes of this tile inside the row
    const int half = p.R;

    const int slice = blockIdx.y * kPairs + pair;
    const int r_begin = min(slice * p.slice_rows, p.K);
    const int r_end = min(r_begin + p.slice_rows, p.K);
    const int n_stages = (r_end - r_begin) / kRowsPerStage;  // K and slices are multiples of kRowsPerStage

    unsigned char* ring = smem + pair * kRingBytes;
    unsigned char* slots = smem + kMainBytes + pair * kSlotRingBytes;
    float* rs_s = reinterpret_cast<float*>(smem + kMainBytes + kPairs * kSlotRingBytes) + pair * kMaxSliceGroups * 4;
    float* part = reinterpret_cast<float*>(smem + kMainBytes + kPairs * kSlotRingBytes + kPairs * kRsBytes);
    // per slice: "full" mbarriers (TMA completion) then "empty" mbarriers (both warps released the slot)
    const uint32_t bars = smem_u32(smem + kMainBytes + kPairs * kSlotRingBytes + kPairs * kRsBytes + kPartBytes) +
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
    // Stage st: rows [r_begin + 32 st, +32) into ring slot st % NS; a stage that
    // starts a group (or the slice) also brings the group's scales and zero
    // points into group slot (group - g_first) % NS.
    // Producer state: the next stage's first row, the next group to fetch and
    // the row where it starts (the slice's first stage always fetches).
    int p_row = r_begin, p_gi = g_first, p_gstart = r_begin;
    auto issue = [&](int st) {  // producer only, stages in order
        const int slot = st & (kStages - 1);
        const uint32_t bar = bars + 8 * slot;
        const bool group_start = p_row == p_gstart;
        const uint32_t sbytes = static_cast<uint32_t>(tile_cols) * 10;  // 2 x fp32 scales + 2 x u8 zeros
        mbar_expect_tx(bar, kStageBytes + (group_start ? sbytes : 0));
        tma_load_2d(ring_s + slot * kStageBytes, &tmap, tile_b0, p_row, bar);
        if (group_start) {
            const uint32_t dst = slots_s + ((p_gi - g_first) & (kStages - 1)) * kScaleSlotBytes;
            const int64_t go = static_cast<int64_t>(p_gi) * p.N;
            bulk_load(dst, p.scales + go + tile_b0, tile_cols * 4, bar);
            bulk_load(dst + kTileBytes * 4, p.scales + go + half + tile_b0, tile_cols * 4, bar);
            bulk_load(dst + kTileBytes * 8, p.zeros + go + tile_b0, tile_cols, bar);
            bulk_load(dst + kTileBytes * 9, p.zeros + go + half + tile_b0, tile_cols, bar);
            ++p_gi;
            p_gstart = p_gi * p.gs;
        }
        p_row += kRowsPerStage;
    };
    if (producer) {
        for (int s = 0; s < kStages - 1 && s < n_stages; ++s) issue(s);
    }
    pdl_launch_dependents();
    pdl_wait();  // x and y below may belong to the previous kernel

    // Slice prologue (both warps of the pair compute the scales; warp 0 of the
    // pair writes the group row sums of exactly what the tensor cores see:
    // hi + lo of x * 2^s, in fixed lane and shuffle order).
    float xscale[M], xunscale[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const float* xm = p.x + static_cast<int64_t>(m) * p.K;
        float mx = 0.0f;
        for (int r = r_begin + lane; r < r_end; r += 32) mx = fmaxf(mx, fabsf(__ldg(xm + r)));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        int sh = 14 - (mx > 0.0f ? ilogbf(mx) : 0);
        sh = max(-126, min(126, sh));
        xscale[m] = ldexpf(1.0f, sh);
        xunscale[m] = ldexpf(1.0f, -sh);
        if (hw == 0) {
            for (int gi = g_first; gi * p.gs < r_end; ++gi) {
                const int a0 = max(gi * p.gs, r_begin), a1 = min((gi + 1) * p.gs, r_end);
                float s = 0.0f;
                for (int r = a0 + lane; r < a1; r += 32) {
                    const float v = __ldg(xm + r) * xscale[m];
                    const float h = __half2float(__float2half_rn(v));
                    s += h + __half2float(__float2half_rn(v - h));
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                if (lane == 0) rs_s[(gi - g_first) * 4 + m] = s * xunscale[m];
            }
        }
    }
    pair_barrier(pair);  // mbarrier init and row sums visible to both warps of the pair

    // This lane's B column: token g/2, part g%2 (0 = hi, 1 = lo); tokens >= M
    // read token 0 and scale it by 0.
    const int btok = g >> 1;
    const bool bpart_lo = g & 1;
    const float* xb = p.x + static_cast<int64_t>(btok < M ? btok : 0) * p.K;
    float bscale = 0.0f, un_t = 1.0f;
#pragma unroll
    for (int m = 0; m < M; ++m) {
        if (m == btok) bscale = xscale[m];
        if (m == t) un_t = xunscale[m];
    }
    // This lane's four rows inside a step and their swizzled 8-byte offsets:
    // 16-byte chunk gb/2 of row r sits at chunk (gb/2) ^ (r & 7).
    int roff[4], soff[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        roff[i] = 2 * t + (i & 1) + 8 * (i >> 1);
        soff[i] = roff[i] * kTileBytes + (((gb >> 1) ^ (roff[i] & 7)) << 4) + 8 * (gb & 1);
    }

    float y[16];  // token t: [0,8) low-nibble columns 8 gb + i, [8,16) high-nibble columns
#pragma unroll
    for (int j = 0; j < 16; ++j) y[j] = 0.0f;
    float c[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i][0] = c[i][1] = c[i][2] = c[i][3] = 0.0f;

    const uint32_t h1024 = p.h1024;
    bool ok = true;
    int gi = g_first;
    int group_end = min((gi + 1) * p.gs, r_end);
    for (int st = 0; st < n_stages; ++st) {
        const int slot = st & (kStages - 1);
        if (ok && !mbar_wait_bounded(bars + 8 * slot, (st / kStages) & 1)) {
            ok = false;
            if (lane == 0) atomicOr(p.err, 1);
        }
        if (producer && ok && st + kStages - 1 < n_stages) {
            // stage st + NS - 1 goes into the slot of stage st - 1 (unused when
            // st == 0) once both warps have released that stage
            const int prev = st - 1;
            if (st > 0 && !mbar_wait_bounded(empty + 8 * (prev & (kStages - 1)), (prev / kStages) & 1)) {
                ok = false;
                atomicOr(p.err, 1);
            } else {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue(st + kStages - 1);
            }
        }
        const unsigned char* stage = ring + slot * kStageBytes;
#pragma unroll
        for (int ks = 0; ks < kRowsPerStage / kStep; ++ks) {
            const int row0 = r_begin + st * kRowsPerStage + ks * kStep;
            // rows 2t, 2t+1 and 2t+8, 2t+9 are adjacent pairs: two 8-byte loads
            const float2 xa = __ldg(reinterpret_cast<const float2*>(xb + row0 + roff[0]));
            const float2 xc = __ldg(reinterpret_cast<const float2*>(xb + row0 + roff[2]));
            const uint32_t b0 = split_part(xa.x * bscale, xa.y * bscale, bpart_lo);
            const uint32_t b1 = split_part(xc.x * bscale, xc.y * bscale, bpart_lo);
            uint2 w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                w[i] = *reinterpret_cast<const uint2*>(stage + ks * kStep * kTileBytes + soff[i]);
            mma_step(c, w, b0, b1, h1024);
        }
        __syncwarp();  // every lane of this warp has read the stage
        if (lane == 0) mbar_arrive(empty + 8 * slot);
        if (r_begin + (st + 1) * kRowsPerStage >= group_end) {
            // Group epilogue for token t:
            //   low:  y += scale * (2^-s C - (1024 + zero) rowSum)
            //   high: y += scale * (2^-s C / 16 - (64 + zero) rowSum)
            // Columns beyond the tile's bytes hold stale slot data; their
            // outputs are never written.
            if (t < M) {
                const unsigned char* sl = slots + ((gi - g_first) & (kStages - 1)) * kScaleSlotBytes;
                const float4* s_lo = reinterpret_cast<const float4*>(sl) + 2 * gb;
                const float4* s_hi = reinterpret_cast<const float4*>(sl + kTileBytes * 4) + 2 * gb;
                const uint2 z_lo = *reinterpret_cast<const uint2*>(sl + kTileBytes * 8 + 8 * gb);
                const uint2 z_hi = *reinterpret_cast<const uint2*>(sl + kTileBytes * 9 + 8 * gb);
                const float rs = rs_s[(gi - g_first) * 4 + t];
                const float un16 = un_t * 0.0625f;
#pragma unroll
                for (int q = 0; q < 2; ++q) {
                    const float4 sl4 = s_lo[q], sh4 = s_hi[q];
                    const uint32_t zl = (&z_lo.x)[q], zh = (&z_hi.x)[q];
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const int i = 4 * q + b;
                        // byte b -> float via the 2^23 pattern: [b, 0, 0, 0x4B] - 2^23
                        const uint32_t sel = static_cast<uint32_t>(b | (4 << 4) | (4 << 8) | (7 << 12));
                        const float zlf = __uint_as_float(prmt(zl, 0x4B000000u, sel)) - 8388608.0f;
                        const float zhf = __uint_as_float(prmt(zh, 0x4B000000u, sel)) - 8388608.0f;
                        y[i] = fmaf((&sl4.x)[b], fmaf(c[i][0] + c[i][1], un_t, -(1024.0f + zlf) * rs), y[i]);
                        y[8 + i] = fmaf((&sh4.x)[b], fmaf(c[i][2] + c[i][3], un16, -(64.0f + zhf) * rs), y[8 + i]);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) c[i][0] = c[i][1] = c[i][2] = c[i][3] = 0.0f;
            ++gi;
            group_end = min((gi + 1) * p.gs, r_end);
        }
    }

    // (1) slices of the CTA in order; red[w][e][lane] reuses the rings.
    __syncthreads();
    float* red = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int e = 0; e < 16; ++e) red[(warp * 16 + e) * 32 + lane] = y[e];
    __syncthreads();
    constexpr int CT = 2 * kTileBytes;  // 256 columns per tile: [0,128) low, [128,256) high
    for (int idx = tid; idx < M * CT; idx += kThreads) {
        const int m = idx / CT, col = idx % CT;
        const int hi = col >= kTileBytes;
        const int cb = hi ? col - kTileBytes : col;  // byte of the tile row
        const int cgb = cb >> 3, i = cb & 7;
        const int e = (hi ? 8 : 0) + i;
        const int ln = 4 * (cgb & 7) + m;
        const int hw_c = cgb >> 3;
        float v = 0.0f;
#pragma unroll
        for (int pr = 0; pr < kPairs; ++pr) v += red[((2 * pr + hw_c) * 16 + e) * 32 + ln];
        part[idx] = v;
    }
    // (2) CTAs of the cluster along K in rank order; rank r finishes columns [r*CT/CK, (r+1)*CT/CK).
    cg::cluster_group cluster = cg::this_cluster();
    const int CK = gridDim.y;
    if (CK > 1) cluster.sync(); else __syncthreads();
    const int rank = CK > 1 ? static_cast<int>(cluster.block_rank()) : 0;
    const int j0 = rank * CT / CK, j1 = (rank + 1) * CT / CK;
    const int span = j1 - j0;
    for (int idx = tid; idx < M * span; idx += kThreads) {
        const int m = idx / span;
        const int col = j0 + idx % span;
        float v;
        if (CK > 1) {
            v = 0.0f;
            for (int q = 0; q < CK; ++q) v += cluster.map_shared_rank(part, q)[m * CT + col];
        } else {
            v = part[m * CT + col];
        }
        const int byte = tile_b0 + (col < kTileBytes ? col : col - kTileBytes);
        const int out_col = col < kTileBytes ? byte : half + byte;
        if (byte < p.R && out_col < p.N) {
            float* out = p.y + static_cast<int64_t>(m) * p.N + out_col;
            float r = fmaf(p.alpha, v, p.accumulate ? *out : 0.0f);
            if (p.bias != nullptr) r += p.bias[out_col];
            *out = r;
        }
    }
    if (CK > 1) cluster.sync();  // keep this CTA's shared memory alive until every rank has read it
}

struct MmaOverrides {
    int ck;
};
MmaOverrides& mma_overrides() {
    static MmaOverrides o{[] {
        const char* v = std::getenv("KT_MMA_CK");
        return v ? std::atoi(v) : 0;
    }()};
    return o;
}

// One CTA per SM: the largest cluster along K (<= 16) that keeps the grid in one
// wave and >= 64 rows per warp.
// Clusters of `ck` CTAs of this kernel that the device holds at once (cached;
// clusters must fit in one GPC, so this is not sm_count / ck).
int max_active_clusters(int ck) {
    static int cache[17] = {0};
    if (cache[ck] != 0) return cache[ck];
    auto kernel = gemv_mma_kernel<1>;
    int n = 0;
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes)) ==
            cudaSuccess &&
        (ck <= 8 || cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) == cudaSuccess)) {
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3(1, ck, 1);
        lc.blockDim = dim3(kThreads, 1, 1);
        lc.dynamicSmemBytes = kSmemBytes;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = ck;
        attr[0].val.clusterDim.z = 1;
        lc.attrs = attr;
        lc.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, kernel, &lc) != cudaSuccess) n = 0;
    }
    cudaGetLastError();  // a refused query only rules this cluster size out
    cache[ck] = n > 0 ? n : -1;
    return cache[ck];
}

// The largest cluster along K whose whole grid is co-resident in one wave and
// that leaves >= 32 rows per slice.
int choose_ck(int R, int K, int sm_count) {
    const int tiles = (R + kTileBytes - 1) / kTileBytes;
    int best = 1;
    for (int ck = 1; ck <= 16; ++ck) {
        if (tiles * ck > sm_count) break;
        if (K / (kPairs * ck) < 32) break;
        if (tiles <= max_active_clusters(ck)) best = ck;
    }
    return best;
}

int slice_rows_for(int K, int ck) {
    const int slices = kPairs * ck;
    const int per = (K + slices - 1) / slices;
    return (per + kRowsPerStage - 1) / kRowsPerStage * kRowsPerStage;
}

template <int M>
cudaError_t launch_m(const QView& w, const MmaParams& p, int ck, cudaStream_t s) {
    auto kernel = gemv_mma_kernel<M>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    if (ck > 8) {
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
    }
    MmaParams q = p;
    q.slice_rows = slice_rows_for(p.K, ck);
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((p.R + kTileBytes - 1) / kTileBytes, ck, 1);
    lc.blockDim = dim3(kThreads, 1, 1);
    lc.dynamicSmemBytes = kSmemBytes;
    lc.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = ck;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 2;
    return cudaLaunchKernelEx(&lc, kernel, *w.tmap_mma, q);
}

}  // namespace

void set_mma_tuning(int cluster_k) { mma_overrides().ck = cluster_k; }

bool gemv_mma_supported(const QView& w, int32_t m, const float* a) {
    if (w.bits != 4 || m < 1 || m > kGemvMmaMaxM || w.tmap_mma == nullptr) return false;
    if (w.columns % 32 != 0 || w.rows % kRowsPerStage != 0 || w.group_size % kRowsPerStage != 0) return false;
    if (reinterpret_cast<uintptr_t>(a) % 8 != 0) return false;  // paired 8-byte loads of x
    // Every warp slice must keep its group row sums in shared memory, at the
    // latest with the largest cluster (16 CTAs x 8 slices).
    return slice_rows_for(w.rows, 16) / w.group_size + 2 <= kMaxSliceGroups;
}

cudaError_t launch_gemv_mma(const QView& w, const MatmulArgs& a, int sm_count, cudaStream_t s) {
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
    p.h1024 = 0x64006400u;
    p.alpha = a.alpha;
    p.accumulate = a.accumulate;
    int ck = choose_ck(p.R, p.K, sm_count);
    const int o = mma_overrides().ck;
    if (o >= 1 && o <= 16) ck = o;
    // Each warp slice must fit kMaxSliceGroups group row sums.
    while (ck < 16 && slice_rows_for(p.K, ck) / p.gs + 2 > kMaxSliceGroups) ++ck;
    switch (a.m) {
        case 1: return launch_m<1>(w, p, ck, s);
        case 2: return launch_m<2>(w, p, ck, s);
        case 3: return launch_m<3>(w, p, ck, s);
        case 4: return launch_m<4>(w, p, ck, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace kt
