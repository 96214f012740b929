// kt_gemv_chain.cu -- a chain of m = 1 quantized GEMVs in one persistent
// launch: the decode step's consecutive projections (an FFN's up / gate|up
// product and its down product, fed the first one's output), each
// MatMul.multiplyQuantized (Engine/kotensor/src/main/kotlin/MatMul.kt:460-536,
// :599-828) at m = 1, with QuantizedLinear's bias (QuantizedLinear.kt:18-25),
// the RMSNorm of the input (RMSNorm.kt:71-90) and SwiGLU's silu(gate) * up
// (SwiGLU.kt:19-25) available per step as in kt_gemv_imma.cu.
//
// Why one launch.  A separate m = 1 GEMV launch streams its weight at HBM
// speed but pays ~4 us of fixed phases (waiting for the previous kernel,
// staging x, the CTA and split-K reductions) during which little is in
// flight.  Here every CTA of a persistent, co-resident grid walks the steps in
// order and owns at most one (column tile, K-split) item per step; as soon as
// its item of step i has consumed its last weight stage, its producer lanes
// start copying the weights of its item of step i + 1 into the ring (weights
// do not depend on x), so the copies run on during the reductions of step i
// and the wait for step i's output.  A step whose input is an earlier step's
// output waits for that step's finished-tile counter (release / acquire,
// bounded) before staging x.
//
// The arithmetic of an item is gemv_imma_kernel's, bit for bit: integer
// mma.sync.m16n8k32 on the raw nibbles (INT4, u8 x s8) or bytes (INT8, s8 x
// s8), x scaled per warp by a power of two to a 22-bit integer split into three
// signed bytes, the reference's per-group combine scale * (D - zero * SX),
// split-K partials summed in split order by the tile's last CTA.
//
// Shared memory: rings[4 pairs][NS][32][128] | scale slots[4][NS][1280] |
// x staging[4][..] | reduction[8][8][32] | mbarriers.  The rings are never
// reused for the reduction, so the next item's copies may land during it.
#include <algorithm>
#include <atomic>
#include <cstdlib>

#include "kt_device.cuh"
#include "kt_internal.h"

namespace kt {
namespace {

using namespace dev;

constexpr int kPairs = 4;
constexpr int kWarps = 2 * kPairs;
constexpr int kThreads = kWarps * 32;
constexpr int kRowsPerStage = 32;       // TMA box height (QView::tmap_mma)
constexpr int kBlockRows = 8;           // weight rows per MMA
constexpr int kTileBytes = 128;
constexpr int kStages = 4;
constexpr int kMaxSliceRows = 1024;     // rows of x one slice stages
constexpr int kMaxSplits = 16;

constexpr int kStageBytes = kRowsPerStage * kTileBytes;               // 4096
constexpr int kScaleSlotBytes = 2 * kTileBytes * 4 + 2 * kTileBytes;  // 1280: s_lo, s_hi, z_lo, z_hi
constexpr int kRingBytes = kStages * kStageBytes;
constexpr int kSlotRingBytes = kStages * kScaleSlotBytes;
constexpr int kMainBytes = kPairs * kRingBytes;
constexpr int kXsBytes = kMaxSliceRows * 4;                           // [row]{xh, xm, xl, 0}
constexpr int kSxBytes = kMaxSliceRows / kBlockRows * 4;              // [block] sum of X
constexpr int kXsPairBytes = kXsBytes + kSxBytes;
constexpr int kRedBytes = kWarps * 8 * 32 * 4;
constexpr size_t kSmemBytes = static_cast<size_t>(kMainBytes) + kPairs * kSlotRingBytes +
                              kPairs * kXsPairBytes + kRedBytes + kPairs * kStages * 16;
static_assert(kXsPairBytes % 16 == 0, "slice staging areas stay 16-byte aligned");
static_assert(2 * (kSmemBytes + 1024 + 256) <= 233472, "two CTAs per SM (dynamic, reserved and static)");

template <int BITS>
constexpr int ct_of() { return BITS == 4 ? 2 * kTileBytes : kTileBytes; }

struct ChainJob {
    const float* scales;
    const uint8_t* zeros;
    const float* x;
    float* y;
    const float* bias;
    const float* norm_w;  // RMSNorm of x before the product (NULL: off)
    float norm_eps;
    float alpha;
    int32_t K, N, R, gs, bits;
    int32_t accumulate;
    int32_t swiglu;       // y[byte] = silu(gate column byte) * (up column half + byte)
    int32_t input;        // the step whose output x is (-1: x is ready at launch)
    int32_t tiles, splits;
    float* partials;      // split-K: [tiles][splits][256]
    int32_t* tickets;     // [tiles], zero on entry and on exit
};

struct ChainParams {
    CUtensorMap tmap[kChainMaxSteps];
    ChainJob job[kChainMaxSteps];
    int32_t n_jobs;
    int32_t* done;  // [kChainMaxSteps] finished tiles per step, then the grid's exit counter
    int32_t* err;
};

__device__ __forceinline__ void imma_16832(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                           uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void imma_16832_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void pair_barrier(int pair) {
    asm volatile("bar.sync %0, 64;" ::"r"(1 + pair) : "memory");
}

// This pair's K-slice of item (step j, CTA b): rows [r_begin, r_end).
struct Slice {
    int tile_b0, tile_cols, r_begin, r_end, n_stages, g_first;
};
__device__ __forceinline__ bool item_of(const ChainJob& J, int b, int pair, Slice& s) {
    if (b >= J.tiles * J.splits) return false;
    const int tile = b / J.splits, split = b - tile * J.splits;
    const int n_slices = J.splits * kPairs;
    const int slice = split * kPairs + pair;
    const int k_stages = J.K / kRowsPerStage;
    const int s_begin = static_cast<int>(static_cast<int64_t>(slice) * k_stages / n_slices);
    const int s_end = static_cast<int>(static_cast<int64_t>(slice + 1) * k_stages / n_slices);
    s.tile_b0 = tile * kTileBytes;
    s.tile_cols = min(kTileBytes, J.R - s.tile_b0);
    s.r_begin = s_begin * kRowsPerStage;
    s.r_end = s_end * kRowsPerStage;
    s.n_stages = s_end - s_begin;
    s.g_first = s.r_begin / J.gs;
    return true;
}

// The producer side of one pair (lanes 0-4 of the pair's warp 0): the weight
// stages of the pair's slice of one item, in order, into the ring, and each
// group's scales and zero points into the group-slot ring.  Stage and group
// numbers are global over the items this pair has streamed, so the ring's
// mbarrier phases run on from one item to the next.
struct Producer {
    const CUtensorMap* tmap;
    const ChainJob* J;
    Slice sl;
    int local;     // next local stage to issue
    int p_row, p_gi, p_gstart;
    uint32_t gstage;  // global number of that stage
    uint32_t ggroup;  // global number of the next group to open
    bool active;
};

__device__ __forceinline__ void producer_issue_one(Producer& P, int lane, uint32_t bars, uint32_t ring_s,
                                                   uint32_t slots_s) {
    const ChainJob& J = *P.J;
    const int slot = static_cast<int>(P.gstage & (kStages - 1));
    const uint32_t bar = bars + 8 * slot;
    const bool group_start = P.p_row == P.p_gstart;
    const int esz4 = J.bits == 4;
    const uint32_t sbytes = static_cast<uint32_t>(P.sl.tile_cols) * (esz4 ? 10 : 4);
    if (lane == 0) {
        mbar_expect_tx(bar, kStageBytes + (group_start ? sbytes : 0));
        tma_load_2d(ring_s + slot * kStageBytes, P.tmap, P.sl.tile_b0, P.p_row, bar);
    }
    if (group_start) {
        const int n_copy_lanes = esz4 ? 4 : 1;
        if (lane >= 1 && lane <= n_copy_lanes) {
            // INT4: s_lo, s_hi, z_lo, z_hi; INT8: the tile's scales
            const uint32_t lane_off = lane <= 2 ? (lane - 1) * kTileBytes * 4 : kTileBytes * (5 + lane);
            const uint32_t lane_bytes = lane <= 2 ? P.sl.tile_cols * 4 : P.sl.tile_cols;
            const int half = J.R;
            const unsigned char* lane_src =
                lane <= 2 ? reinterpret_cast<const unsigned char*>(J.scales + P.sl.tile_b0 + (lane == 2 ? half : 0))
                          : J.zeros + P.sl.tile_b0 + (lane == 4 ? half : 0);
            const int lane_esize = lane <= 2 ? 4 : 1;
            const uint32_t dst = slots_s + (P.ggroup & (kStages - 1)) * kScaleSlotBytes + lane_off;
            bulk_load(dst, lane_src + static_cast<int64_t>(P.p_gi) * J.N * lane_esize, lane_bytes, bar);
        }
        ++P.p_gi;
        P.p_gstart = P.p_gi * J.gs;
        ++P.ggroup;
    }
    P.p_row += kRowsPerStage;
    ++P.local;
    ++P.gstage;
}

// Issues the next stage if its slot is free: waits (bounded) for the release
// of the stage NS before it; false on a timeout.
__device__ __forceinline__ bool producer_step(Producer& P, int lane, uint32_t bars, uint32_t empty, uint32_t ring_s,
                                              uint32_t slots_s) {
    if (!P.active || P.local >= P.sl.n_stages) return true;
    int go = 1;
    if (P.gstage >= kStages) {
        const uint32_t prev = P.gstage - kStages;
        if (lane == 0) go = mbar_wait_bounded(empty + 8 * (prev & (kStages - 1)), (prev / kStages) & 1) ? 1 : 0;
        go = __shfl_sync(0xffffffffu, go, 0);
    }
    if (!go) return false;
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    producer_issue_one(P, lane, bars, ring_s, slots_s);
    return true;
}


// Sets P to stream the pair's slice of item (step j, CTA b); inactive when the
// CTA has no item in step j.
__device__ __forceinline__ void producer_start(Producer& P, const ChainParams& p, int j, int b, int pair) {
    P.active = j < p.n_jobs && item_of(p.job[j], b, pair, P.sl);
    if (!P.active) return;
    P.tmap = &p.tmap[j];
    P.J = &p.job[j];
    P.local = 0;
    P.p_row = P.sl.r_begin;
    P.p_gi = P.sl.g_first;
    P.p_gstart = P.sl.r_begin;
}

// The next step after j in which CTA b has an item (p.n_jobs: none).
__device__ __forceinline__ int next_step(const ChainParams& p, int j, int b) {
    for (int k = j + 1; k < p.n_jobs; ++k)
        if (b < p.job[k].tiles * p.job[k].splits) return k;
    return p.n_jobs;
}

// One item: (step j, CTA b).  `ok` is CTA-uniform on entry and on exit; a
// bounded wait that runs out clears it and sets the error word.
template <int BITS>
__device__ __forceinline__ void run_item(const ChainParams& p, int j, int b, int j_next, Producer& P,
                                         unsigned char* smem, int& ok, uint32_t& c_stage, uint32_t& c_group) {
    constexpr int kCT = ct_of<BITS>();
    constexpr int kJ = BITS == 4 ? 4 : 2;
    const ChainJob& J = p.job[j];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, pair = warp >> 1, hw = warp & 1;
    const int g = lane >> 2, t = lane & 3;
    const int half = J.R;
    Slice sl;
    item_of(J, b, pair, sl);
    const int tile = b / J.splits, split = b - tile * J.splits;
    unsigned char* ring = smem + pair * kRingBytes;
    unsigned char* slots = smem + kMainBytes + pair * kSlotRingBytes;
    unsigned char* xstage = smem + kMainBytes + kPairs * kSlotRingBytes + pair * kXsPairBytes;
    float* red = reinterpret_cast<float*>(smem + kMainBytes + kPairs * kSlotRingBytes + kPairs * kXsPairBytes);
    uint8_t* xs = xstage;
    int32_t* sxb = reinterpret_cast<int32_t*>(xstage + kXsBytes);
    const uint32_t bars = smem_u32(smem + kMainBytes + kPairs * kSlotRingBytes + kPairs * kXsPairBytes + kRedBytes) +
                          pair * kStages * 16;
    const uint32_t empty = bars + kStages * 8;
    const uint32_t ring_s = smem_u32(ring);
    const uint32_t slots_s = smem_u32(slots);
    const bool producer = hw == 0;
    __shared__ int s_flag;
    __shared__ float s_nred[kWarps];
    float* s_swig = red;  // [2 * kTileBytes], once the CTA reduction has read red

    // ---- the input: an earlier step's output is complete once all its tiles are
    if (J.input >= 0) {
        if (tid == 0) {
            const int32_t need = p.job[J.input].tiles;
            const int32_t* cnt = p.done + J.input;
            bool ready = ld_acquire(cnt) >= need;
            if (!ready && ok) {
                const uint64_t t0 = globaltimer();
                while (!(ready = ld_acquire(cnt) >= need)) {
                    if (globaltimer() - t0 > kWaitLimitNs) break;
                }
            }
            if (!ready && ok) atomicOr(p.err, 1);
            s_flag = ready ? ok : 0;
        }
        __syncthreads();
        ok = s_flag;
    }

    // ---- RMSNorm prologue and x staging (gemv_imma_kernel's, with loads through
    // L2: x may have been written by other CTAs of this launch)
    float nrm = 1.0f;
    if (J.norm_w != nullptr) {
        float ss = 0.0f;
#pragma unroll 4
        for (int i = 4 * tid; i < J.K; i += 4 * kThreads) {
            const float4 v4 = __ldcg(reinterpret_cast<const float4*>(J.x + i));
            ss = fmaf(v4.x, v4.x, ss);
            ss = fmaf(v4.y, v4.y, ss);
            ss = fmaf(v4.z, v4.z, ss);
            ss = fmaf(v4.w, v4.w, ss);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) s_nred[warp] = ss;
        __syncthreads();
        float tot = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < kWarps; ++w2) tot += s_nred[w2];
        nrm = 1.0f / sqrtf(tot / static_cast<float>(J.K) + J.norm_eps);
    }
    const int n_f4 = (sl.r_end - sl.r_begin) / 8;
    float4 xv[4];
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int f = lane + 32 * i;
        const int row = 8 * (2 * (f >> 1) + hw) + 4 * (f & 1);
        xv[i] = f < n_f4 ? __ldcg(reinterpret_cast<const float4*>(J.x + sl.r_begin + row))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
        if (J.norm_w != nullptr && f < n_f4) {
            const float4 w4 = __ldg(reinterpret_cast<const float4*>(J.norm_w + sl.r_begin + row));
            xv[i] = make_float4(xv[i].x * nrm * w4.x, xv[i].y * nrm * w4.y, xv[i].z * nrm * w4.z,
                                xv[i].w * nrm * w4.w);
        }
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(xv[i].x), fabsf(xv[i].y)), fmaxf(fabsf(xv[i].z), fabsf(xv[i].w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    int sh = mx > 0.0f ? 21 - ilogbf(mx) : 0;
    sh = max(-126, min(126, sh));
    const float sc = ldexpf(1.0f, sh);
    const float unscale = ldexpf(1.0f, -sh);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int f = lane + 32 * i;
        const int row = 8 * (2 * (f >> 1) + hw) + 4 * (f & 1);
        const float v[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
        int X[4];
        uint32_t packed[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            X[k] = __float2int_rn(v[k] * sc);
            const int xh = (X[k] + 32896) >> 16;
            const int rem = X[k] - (xh << 16);
            const int xm = (rem + 128) >> 8;
            const int xl = rem - (xm << 8);
            packed[k] = (static_cast<uint32_t>(xh) & 0xFFu) | ((static_cast<uint32_t>(xm) & 0xFFu) << 8) |
                        ((static_cast<uint32_t>(xl) & 0xFFu) << 16);
        }
        const int s4 = X[0] + X[1] + X[2] + X[3];
        const int s8 = s4 + __shfl_xor_sync(0xffffffffu, s4, 1);
        if (f < n_f4) {
            *reinterpret_cast<uint4*>(xs + 4 * row) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            if ((f & 1) == 0) sxb[row / kBlockRows] = s8;
        }
    }
    __syncwarp();

    // ---- main loop (gemv_imma_kernel's)
    const uint32_t part_byte = static_cast<uint32_t>(g >> 2);
    const uint32_t pos = static_cast<uint32_t>(g & 3);
    const uint32_t sel_hm = (0x4444u & ~(0xFu << (4 * pos))) | (part_byte << (4 * pos));
    const uint32_t sel_l = g < 4 ? (0x4444u & ~(0xFu << (4 * pos))) | (2u << (4 * pos)) : 0x4444u;
    const int off0 = (2 * t) * kTileBytes + ((g ^ (2 * t)) << 4);
    const int off1 = (2 * t + 1) * kTileBytes + ((g ^ (2 * t + 1)) << 4);
    const int u = t & 1;
    const bool low_owner = t < 2;
    float y[2 * kJ];
#pragma unroll
    for (int q = 0; q < 2 * kJ; ++q) y[q] = 0.0f;
    int c[kJ][4];
    int e[kJ][4];
#pragma unroll
    for (int jj = 0; jj < kJ; ++jj)
        c[jj][0] = c[jj][1] = c[jj][2] = c[jj][3] = e[jj][0] = e[jj][1] = e[jj][2] = e[jj][3] = 0;
    long long sx = 0;
    int gi = sl.g_first;
    int group_end = min((gi + 1) * J.gs, sl.r_end);
    for (int st = 0; st < sl.n_stages; ++st) {
        const uint32_t gst = c_stage + static_cast<uint32_t>(st);
        const int slot = static_cast<int>(gst & (kStages - 1));
        if (ok && !mbar_wait_bounded(bars + 8 * slot, (gst / kStages) & 1)) {
            ok = 0;
            atomicOr(p.err, 1);
        }
        ok = __all_sync(0xffffffffu, ok);
        // stage st + NS - 1 into the slot stage st - 1 used, once both warps released it
        if (producer && ok && st > 0 && P.local == st + kStages - 1 &&
            !producer_step(P, lane, bars, empty, ring_s, slots_s)) {
            ok = 0;
            if (lane == 0) atomicOr(p.err, 1);
        }
        if (ok) {
            const unsigned char* stage = ring + slot * kStageBytes;
#pragma unroll
            for (int bb = 0; bb < 2; ++bb) {
                const int blk = 2 * bb + hw;
                const int brow = st * kRowsPerStage + blk * kBlockRows;
                const uint2 xw = *reinterpret_cast<const uint2*>(xs + 4 * (brow + 2 * t));
                const uint32_t b0 = prmt(xw.x, 0u, sel_hm), b1 = prmt(xw.y, 0u, sel_hm);
                const uint32_t l0 = prmt(xw.x, 0u, sel_l), l1 = prmt(xw.y, 0u, sel_l);
                const uint4 w0 = *reinterpret_cast<const uint4*>(stage + blk * kBlockRows * kTileBytes + off0);
                const uint4 w1 = *reinterpret_cast<const uint4*>(stage + blk * kBlockRows * kTileBytes + off1);
                sx += sxb[brow / kBlockRows];
                if constexpr (BITS == 4) {
                    const uint32_t a[4][4] = {
                        {w0.x & 0x0F0F0F0Fu, w0.x & 0xF0F0F0F0u, w1.x & 0x0F0F0F0Fu, w1.x & 0xF0F0F0F0u},
                        {w0.y & 0x0F0F0F0Fu, w0.y & 0xF0F0F0F0u, w1.y & 0x0F0F0F0Fu, w1.y & 0xF0F0F0F0u},
                        {w0.z & 0x0F0F0F0Fu, w0.z & 0xF0F0F0F0u, w1.z & 0x0F0F0F0Fu, w1.z & 0xF0F0F0F0u},
                        {w0.w & 0x0F0F0F0Fu, w0.w & 0xF0F0F0F0u, w1.w & 0x0F0F0F0Fu, w1.w & 0xF0F0F0F0u}};
#pragma unroll
                    for (int jj = 0; jj < kJ; ++jj) {
                        imma_16832(c[jj], a[jj][0], a[jj][1], a[jj][2], a[jj][3], b0, b1);
                        imma_16832(e[jj], a[jj][0], a[jj][1], a[jj][2], a[jj][3], l0, l1);
                    }
                } else {
                    imma_16832_s8(c[0], w0.x, w0.y, w1.x, w1.y, b0, b1);
                    imma_16832_s8(e[0], w0.x, w0.y, w1.x, w1.y, l0, l1);
                    imma_16832_s8(c[kJ - 1], w0.z, w0.w, w1.z, w1.w, b0, b1);
                    imma_16832_s8(e[kJ - 1], w0.z, w0.w, w1.z, w1.w, l0, l1);
                }
            }
            if (sl.r_begin + (st + 1) * kRowsPerStage >= group_end) {
                const unsigned char* gsl = slots + (c_group & (kStages - 1)) * kScaleSlotBytes;
                const float* s_arr = reinterpret_cast<const float*>(gsl + (low_owner ? 0 : kTileBytes * 4));
                const uint8_t* z_arr = gsl + kTileBytes * (low_owner ? 8 : 9);
                const float sxf = static_cast<float>(sx);
#pragma unroll
                for (int jj = 0; jj < kJ; ++jj) {
                    const int send0 = low_owner ? c[jj][2] : c[jj][0];
                    const int send1 = low_owner ? c[jj][3] : c[jj][1];
                    const int recv0 = __shfl_xor_sync(0xffffffffu, send0, 2);
                    const int recv1 = __shfl_xor_sync(0xffffffffu, send1, 2);
                    const int lrecv0 = __shfl_xor_sync(0xffffffffu, e[jj][2], 2);
                    const int lrecv1 = __shfl_xor_sync(0xffffffffu, e[jj][3], 2);
                    const float dh0 = static_cast<float>(low_owner ? c[jj][0] : recv0);
                    const float dm0 = static_cast<float>(low_owner ? recv0 : c[jj][2]);
                    const float dl0 = static_cast<float>(low_owner ? e[jj][0] : lrecv0);
                    const float dh1 = static_cast<float>(low_owner ? c[jj][1] : recv1);
                    const float dm1 = static_cast<float>(low_owner ? recv1 : c[jj][3]);
                    const float dl1 = static_cast<float>(low_owner ? e[jj][1] : lrecv1);
                    const float d0 = fmaf(dh0, 65536.0f, fmaf(dm0, 256.0f, dl0));
                    const float d1 = fmaf(dh1, 65536.0f, fmaf(dm1, 256.0f, dl1));
                    if constexpr (BITS == 4) {
                        const int bq = 16 * g + 4 * jj + 2 * u;
                        const float2 s2 = *reinterpret_cast<const float2*>(s_arr + bq);
                        const uint32_t z2 = *reinterpret_cast<const uint16_t*>(z_arr + bq);
                        const float k16 = low_owner ? 1.0f : 0.0625f;
                        y[2 * jj] = fmaf(s2.x, fmaf(d0, k16, -static_cast<float>(z2 & 0xFFu) * sxf), y[2 * jj]);
                        y[2 * jj + 1] =
                            fmaf(s2.y, fmaf(d1, k16, -static_cast<float>(z2 >> 8) * sxf), y[2 * jj + 1]);
                    } else {
                        const int bq = 16 * g + 8 * jj + (low_owner ? 0 : 4) + 2 * u;
                        const float2 s2 = *reinterpret_cast<const float2*>(reinterpret_cast<const float*>(gsl) + bq);
                        y[2 * jj] = fmaf(s2.x, d0, y[2 * jj]);
                        y[2 * jj + 1] = fmaf(s2.y, d1, y[2 * jj + 1]);
                    }
                }
#pragma unroll
                for (int jj = 0; jj < kJ; ++jj)
                    c[jj][0] = c[jj][1] = c[jj][2] = c[jj][3] = e[jj][0] = e[jj][1] = e[jj][2] = e[jj][3] = 0;
                sx = 0;
                ++gi;
                ++c_group;
                group_end = min((gi + 1) * J.gs, sl.r_end);
            }
        }
        // release the stage, and a group slot read just above, to the producer
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + 8 * slot);
    }
    c_stage += static_cast<uint32_t>(sl.n_stages);

    // ---- the CTA's next item: its first stages stream in during what follows
    if (producer && ok) {
        producer_start(P, p, j_next, b, pair);
        for (int s = 0; s < kStages && P.active && ok; ++s) {
            if (!producer_step(P, lane, bars, empty, ring_s, slots_s)) {
                ok = 0;
                if (lane == 0) atomicOr(p.err, 1);
            }
        }
    }

    // ---- (1) warps of the CTA in order
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 2 * kJ; ++q) red[(warp * 8 + q) * 32 + lane] = y[q] * unscale;
    ok = __syncthreads_and(ok);
    if (!ok) return;
    float v = 0.0f;
    if (tid < kCT) {
        const int bq = tid & (kTileBytes - 1);
        const int gg = bq >> 4, jw = (bq >> 2) & 3, sg = bq & 3;
        const int hi = BITS == 4 ? tid >> 7 : jw & 1;
        const int jx = BITS == 4 ? jw : jw >> 1;
        const int ln = 4 * gg + 2 * hi + (sg >> 1);
        const int q = 2 * jx + (sg & 1);
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += red[(w * 8 + q) * 32 + ln];
    }
    const int tile_b0 = sl.tile_b0;
    auto emit = [&](int col, float val) {
        const int byte = tile_b0 + (col & (kTileBytes - 1));
        const int out_col = BITS == 4 && col >= kTileBytes ? half + byte : byte;
        if (col < kCT && byte < J.R && out_col < J.N) {
            float* out = J.y + out_col;
            float r = fmaf(J.alpha, val, J.accumulate ? __ldcg(out) : 0.0f);
            if (J.bias != nullptr) r += J.bias[out_col];
            *out = r;
        }
    };
    auto swiglu_out = [&](int bq, float gv, float uv) {
        gv = fmaf(J.alpha, gv, 0.0f);  // emit()'s arithmetic, as in gemv_imma_kernel
        uv = fmaf(J.alpha, uv, 0.0f);
        if (J.bias != nullptr) {
            gv += J.bias[bq];
            uv += J.bias[half + bq];
        }
        J.y[bq] = gv / (1.0f + expf(-gv)) * uv;
    };
    auto finish_tile = [&](float val) {
        if (J.swiglu) {
            __syncthreads();  // every thread is done reading red
            s_swig[tid] = val;
            __syncthreads();
            const int byte = tile_b0 + tid;
            if (tid < kTileBytes && byte < J.R) swiglu_out(byte, s_swig[tid], s_swig[tid + kTileBytes]);
        } else {
            emit(tid, val);
        }
        // the tile is done: every thread's stores before thread 0's release
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            red_release_add(p.done + j, 1);
        }
    };
    const int S = J.splits;
    if (S == 1) {
        finish_tile(v);
        return;
    }
    // (2) split-K through global memory: the tile's last CTA sums the partials in split order
    float* tile_parts = J.partials + static_cast<int64_t>(tile) * S * kCT;
    if (tid < kCT) __stcg(tile_parts + static_cast<int64_t>(split) * kCT + tid, v);
    __syncthreads();
    if (tid == 0) s_flag = atomic_add_acq_rel(J.tickets + tile, 1) == S - 1;
    __syncthreads();
    if (!s_flag) return;
    float sum = 0.0f;
    for (int s0 = 0; s0 < S; s0 += 16) {
        float tv[16];
#pragma unroll
        for (int q = 0; q < 16; ++q)
            tv[q] = s0 + q == split ? v
                    : s0 + q < S && tid < kCT ? __ldcg(tile_parts + static_cast<int64_t>(s0 + q) * kCT + tid) : 0.0f;
#pragma unroll
        for (int q = 0; q < 16; ++q)
            if (s0 + q < S) sum += tv[q];
    }
    if (tid == 0) J.tickets[tile] = 0;  // ready for the next launch on this workspace
    finish_tile(sum);
}

__global__ void __launch_bounds__(kThreads, 2) gemv_chain_kernel(const __grid_constant__ ChainParams p) {
    extern __shared__ __align__(1024) unsigned char smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, pair = warp >> 1, hw = warp & 1;
    const int b = blockIdx.x;
    const uint32_t bars = smem_u32(smem + kMainBytes + kPairs * kSlotRingBytes + kPairs * kXsPairBytes + kRedBytes) +
                          pair * kStages * 16;
    const uint32_t empty = bars + kStages * 8;
    if (hw == 0 && lane == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(bars + 8 * s, 1);
            mbar_init(empty + 8 * s, 2);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    pdl_launch_dependents();
    pdl_wait();  // the first step's x and every output may belong to the previous kernel

    Producer P;
    P.gstage = 0;
    P.ggroup = 0;
    uint32_t c_stage = 0, c_group = 0;
    int ok = 1;
    int j = next_step(p, -1, b);
    if (hw == 0) {
        producer_start(P, p, j, b, pair);
        for (int s = 0; s < kStages && P.active; ++s)
            producer_step(P, lane, bars, empty, smem_u32(smem + pair * kRingBytes),
                          smem_u32(smem + kMainBytes + pair * kSlotRingBytes));
    }
    while (j < p.n_jobs && ok) {
        const int jn = next_step(p, j, b);
        if (p.job[j].bits == 4) run_item<4>(p, j, b, jn, P, smem, ok, c_stage, c_group);
        else run_item<8>(p, j, b, jn, P, smem, ok, c_stage, c_group);
        j = jn;
    }
    // copies still in flight (after a timeout) land before the CTA exits: at
    // most the last NS stages this pair issued
    if (hw == 0 && lane == 0) {
        for (uint32_t s = P.gstage > kStages ? P.gstage - kStages : 0; s < P.gstage; ++s)
            if (!mbar_wait_bounded(bars + 8 * (s & (kStages - 1)), (s / kStages) & 1)) break;
    }
    // the grid's last CTA to leave zeroes the step counters for the next launch
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(p.done + kChainMaxSteps, 1) == static_cast<int>(gridDim.x) - 1) {
            for (int k = 0; k < kChainMaxSteps; ++k) p.done[k] = 0;
            p.done[kChainMaxSteps] = 0;
            __threadfence();
        }
    }
}


int tiles_of(int R) { return (R + kTileBytes - 1) / kTileBytes; }

int min_splits(int K) {
    const int per = kPairs * kMaxSliceRows;
    return (K + per - 1) / per;
}

// CTAs of the chain kernel one SM holds (cached per device); the grid never
// exceeds this times the SM count, so every CTA of a launch can be resident
// at once once earlier kernels have drained (the steps wait on one another).
int chain_blocks_per_sm() {
    constexpr int kMaxDevices = 64;
    static std::atomic<int> cache[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    std::atomic<int>* slot = dev >= 0 && dev < kMaxDevices ? &cache[dev] : nullptr;
    if (slot != nullptr) {
        const int c = slot->load(std::memory_order_acquire);
        if (c != 0) return c;
    }
    int n = 0;
    if (cudaFuncSetAttribute(gemv_chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemBytes)) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_chain_kernel, kThreads, kSmemBytes) != cudaSuccess)
        n = 0;
    cudaGetLastError();
    if (n > 0 && slot != nullptr) slot->store(n, std::memory_order_release);
    return n;
}

// K-splits of a step: fill the grid's CTAs with its tiles, at most kMaxSplits,
// at least one stage per slice, slices of at most kMaxSliceRows rows.
int chain_splits(const QView& w, int grid) {
    const int tiles = tiles_of(w.bytes_per_row);
    const int k_stages = w.rows / kRowsPerStage;
    int s = std::min(kMaxSplits, std::max(1, grid / tiles));
    s = std::min(s, std::max(1, k_stages / kPairs));
    return std::max(s, min_splits(w.rows));
}

}  // namespace

bool gemv_chain_step_supported(const QView& w, const float* a, bool swiglu, int sm_count) {
    if (!gemv_imma_supported(w, 1, a)) return false;
    if (swiglu && (w.bits != 4 || w.columns != 2 * w.bytes_per_row)) return false;
    const int grid = chain_blocks_per_sm() * sm_count;
    const int tiles = tiles_of(w.bytes_per_row);
    const int s = chain_splits(w, grid);
    return grid > 0 && static_cast<int64_t>(tiles) * s <= grid && s <= kMaxSplits &&
           w.rows / kRowsPerStage >= s * kPairs;
}

size_t gemv_chain_workspace_bytes(const ChainStep* steps, int n, int sm_count) {
    const int grid = chain_blocks_per_sm() * sm_count;
    size_t bytes = kWorkspaceReservedBytes;
    for (int i = 0; i < n; ++i) {
        const int s = chain_splits(steps[i].w, grid);
        if (s > 1)
            bytes += static_cast<size_t>(tiles_of(steps[i].w.bytes_per_row)) * s *
                     (steps[i].w.bits == 4 ? ct_of<4>() : ct_of<8>()) * sizeof(float);
    }
    return bytes;
}

cudaError_t launch_gemv_chain(const ChainStep* steps, int n, int sm_count, cudaStream_t s, void* workspace,
                              size_t workspace_bytes, int32_t* err) {
    if (n < 1 || n > kChainMaxSteps) return cudaErrorInvalidValue;
    const int grid = chain_blocks_per_sm() * sm_count;
    if (grid <= 0) return cudaErrorInvalidConfiguration;
    if (workspace == nullptr || workspace_bytes < gemv_chain_workspace_bytes(steps, n, sm_count))
        return cudaErrorInvalidValue;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    ChainParams p{};
    p.n_jobs = n;
    p.done = reinterpret_cast<int32_t*>(ws + kChainCounterOffset);
    p.err = err;
    int32_t* tickets = p.done + kChainMaxSteps + 1;
    size_t part_off = kWorkspaceReservedBytes;
    int used_tickets = 0;
    int max_items = 1;
    for (int i = 0; i < n; ++i) {
        const ChainStep& c = steps[i];
        if (!gemv_chain_step_supported(c.w, c.a, c.swiglu != 0, sm_count)) return cudaErrorInvalidValue;
        ChainJob& J = p.job[i];
        p.tmap[i] = *c.w.tmap_mma;
        J.scales = c.w.scales;
        J.zeros = c.w.zeros;
        J.x = c.a;
        J.y = c.c;
        J.bias = c.bias;
        J.norm_w = c.norm_weight;
        J.norm_eps = c.norm_eps;
        J.alpha = c.alpha;
        J.K = c.w.rows;
        J.N = c.w.columns;
        J.R = c.w.bytes_per_row;
        J.gs = c.w.group_size;
        J.bits = c.w.bits;
        J.accumulate = c.accumulate;
        J.swiglu = c.swiglu;
        J.input = c.input;
        J.tiles = tiles_of(J.R);
        J.splits = chain_splits(c.w, grid);
        max_items = std::max(max_items, J.tiles * J.splits);
        if (J.splits > 1) {
            if (used_tickets + J.tiles > kChainTicketCap) return cudaErrorInvalidValue;
            J.tickets = tickets + used_tickets;
            used_tickets += J.tiles;
            J.partials = reinterpret_cast<float*>(ws + part_off);
            part_off += static_cast<size_t>(J.tiles) * J.splits * (J.bits == 4 ? ct_of<4>() : ct_of<8>()) * sizeof(float);
        }
    }
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(std::min(grid, max_items), 1, 1);
    lc.blockDim = dim3(kThreads, 1, 1);
    lc.dynamicSmemBytes = kSmemBytes;
    lc.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    return cudaLaunchKernelEx(&lc, gemv_chain_kernel, p);
}

}  // namespace kt
