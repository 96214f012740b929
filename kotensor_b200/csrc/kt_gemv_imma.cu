// kt_gemv_imma.cu -- INT4 / INT8 decode GEMV for one token (m = 1) on integer
// tensor-core products: MatMul.multiplyQuantized (Engine/kotensor/src/main/
// kotlin/MatMul.kt:460-536, :599-828) for m = 1, the decode step's shape.
//
// Operands.  mma.sync.m16n8k32 u8 x s8 -> s32.  The reduction index k of one
// MMA is split as k = 4 rho + sigma: rho (0..7) is one of 8 weight rows,
// sigma (0..3) a byte position inside a 32-bit word of that row.  MMA row g
// (0..7) is one word column of the tile row and row g + 8 the same word's high
// nibbles, so every A register is a weight word as it lies in shared memory,
// masked: w & 0x0F0F0F0F (low nibbles, q) or w & 0xF0F0F0F0 (high nibbles,
// 16 q).  No byte shuffling: two AND per word per row.  Two MMAs share those A
// registers.  In the first, B row 4 rho + sigma, column n carries activation
// part n / 4 (0 = high, 1 = middle byte) of row rho when sigma == n % 4 and 0
// otherwise, so D[g][n] is the dot product of the rows with column "byte n % 4
// of word g" -- 32 columns x 8 rows x 2 nibbles, every output lane useful; in
// the second, columns 0-3 carry the low byte the same way (columns 4-7 zero).
//
// Exactness.  x is scaled by a power of two 2^sh per warp (max|x 2^sh| in
// [2^21, 2^22)), rounded to an integer X (22-bit magnitude, the precision of
// an fp32 mantissa relative to the warp's largest |x|) and split
// X = 65536 xh + 256 xm + xl into signed bytes; the products are exact
// integers in s32.  Per group (combineGroup, MatMul.kt:804-828), with SX the
// group's sum of X over this warp's rows and D = 65536 D_h + 256 D_m + D_l:
//     low nibble:  y += scale * (D - zero * SX)
//     high nibble: y += scale * (D / 16 - zero * SX)
// and y is multiplied by 2^-sh once at the end.  The products are exact, so
// the only roundings are x's 22-bit quantization relative to the warp's max|x|
// and fp32 accumulation -- fp32 class for any spread of magnitudes inside a
// warp's rows up to 2^22 (outlier channels included).
//
// INT8 weights (BITS = 8) run the same pipeline on signed bytes (s8 x s8
// MMAs): A rows g and g + 8 are words 4g + 2jj and 4g + 2jj + 1 of the lane's
// 16-byte chunk (two MMA pairs per chunk instead of four), a tile is 128
// output columns, and the group combine has no zero point (out += scale * D).
//
// Tiling and streaming are those of the fp16 kernel (kt_gemv_mma.cu): a CTA
// owns 128 packed bytes of every row (256 output columns); 4 pairs of warps
// own consecutive K-slices; each pair streams its slice through a ring of
// 32-row x 128-byte TMA stages (128-byte swizzle) plus bulk copies of each
// group's scales and zero points, with bounded mbarrier waits; inside a stage
// warp 0 of the pair takes 8-row blocks 0 and 2, warp 1 blocks 1 and 3.  K is
// split over CTAs when the column tiles alone cannot fill the GPU; the last
// CTA of a tile sums the split partials in split order (deterministic).
#include <algorithm>
#include <atomic>
#include <initializer_list>
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
constexpr int kMaxSplits = 16;          // K-splits per column tile (a cluster of at most 16 CTAs)

constexpr int kStageBytes = kRowsPerStage * kTileBytes;               // 4096
constexpr int kScaleSlotBytes = 2 * kTileBytes * 4 + 2 * kTileBytes;  // 1280: s_lo, s_hi, z_lo, z_hi
constexpr int kRingBytes = kStages * kStageBytes;
constexpr int kSlotRingBytes = kStages * kScaleSlotBytes;
constexpr int kMainBytes = kPairs * kRingBytes;
// output columns per tile: 256 (INT4, two nibbles per byte) or 128 (INT8)
template <int BITS>
constexpr int ct_of() { return BITS == 4 ? 2 * kTileBytes : kTileBytes; }
constexpr int kRedBytes = kWarps * 8 * 32 * 4;                        // reuses the rings
constexpr int kXsBytes = kMaxSliceRows * 4;                           // [row]{xh, xm, xl, 0}
constexpr int kSxBytes = kMaxSliceRows / kBlockRows * 4;              // [block] sum of X
constexpr int kXsPairBytes = kXsBytes + kSxBytes;
constexpr size_t kSmemBytes = static_cast<size_t>(kMainBytes) + kPairs * kSlotRingBytes +
                              kPairs * kXsPairBytes + kPairs * kStages * 16;
static_assert(kRedBytes <= kMainBytes, "reduction buffer must fit in the rings");
static_assert(kXsPairBytes % 16 == 0, "slice staging areas stay 16-byte aligned");
static_assert(2 * (kSmemBytes + 1024) <= 233472, "two CTAs per SM");

struct ImmaParams {
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
    int32_t swiglu;    // y[byte] = silu(gate column byte) * (up column half + byte) instead of both columns
    const float* norm_w;  // RMSNorm of x before the product (NULL: off)
    float norm_eps;
    int32_t cluster;   // split-K inside a cluster (1) or through partials in global memory (0)
    float* partials;   // split-K: [tiles][splits][256]
    int32_t* tickets;  // [tiles], zero on entry and on exit
    TpExchange tp;     // row-parallel exchange fused into the epilogue (nranks 0: none)
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

// Shared memory: rings[4 slices][NS][32][128] (later red[8][8][32]) |
// slots[4][NS][1280] | x staging[4][kXsPairBytes] | mbarriers[4][2][NS].
template <int BITS>
__global__ void __launch_bounds__(kThreads, 2)
    gemv_imma_kernel(const __grid_constant__ CUtensorMap tmap, ImmaParams p) {
    constexpr int kCT = ct_of<BITS>();
    constexpr int kJ = BITS == 4 ? 4 : 2;  // MMA pairs per 8-row block and warp
    extern __shared__ __align__(1024) unsigned char smem[];
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int pair = warp >> 1;
    const int hw = warp & 1;
    const int g = lane >> 2;  // word column of the tile row (A rows g, g + 8); B column n = g
    const int t = lane & 3;   // rows 2t, 2t+1 of an 8-row block; C columns 2t, 2t+1
    const int tile_b0 = blockIdx.x * kTileBytes;
    const int tile_cols = min(kTileBytes, p.R - tile_b0);
    const int half = p.R;

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
    unsigned char* xstage = smem + kMainBytes + kPairs * kSlotRingBytes + pair * kXsPairBytes;
    uint8_t* xs = xstage;                                                   // [row]{xh, xm, xl, 0}
    int32_t* sxb = reinterpret_cast<int32_t*>(xstage + kXsBytes);           // [block] sum of X
    const uint32_t bars =
        smem_u32(smem + kMainBytes + kPairs * kSlotRingBytes + kPairs * kXsPairBytes) +
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
    // starts a group also brings the group's scales and zero points into group
    // slot (group - g_first) % NS (lanes 1-4 of warp 0; the arming arrive of
    // lane 0 is still pending, so their complete_tx cannot finish the phase).
    int p_row = r_begin, p_gi = g_first, p_gstart = r_begin, p_issued = 0;
    // INT4: lanes 1-4 copy the low / high nibble columns' scales and zero
    // points (s_lo, s_hi, z_lo, z_hi); INT8: lane 1 copies the tile's scales
    const uint32_t sbytes = static_cast<uint32_t>(tile_cols) * (BITS == 4 ? 10 : 4);
    const int n_copy_lanes = BITS == 4 ? 4 : 1;
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
            if (lane >= 1 && lane <= n_copy_lanes) {
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
    pair_barrier(pair);  // the mbarriers are initialised before warp 1 waits on them
    pdl_launch_dependents();
    pdl_wait();  // x and y below may belong to the previous kernel

    // ---- stage x for this warp's rows, the 8-row blocks hw, hw + 2, ... of the
    // slice: float4 f of the warp is rows 8 (2 (f / 2) + hw) + 4 (f % 2) .. + 3.
    // Each warp picks its own power of two 2^sh (max|x 2^sh| in [2^21, 2^22)),
    // so |X| < 2^22; X = 65536 xh + 256 xm + xl with xh = (X + 32896) >> 16 in
    // [-64, 64], the remainder in [-32896, 32639] and so xm = (rem + 128) >> 8
    // and xl = rem - 256 xm in [-128, 127]; the warp's results are unscaled
    // before the warps are summed.
    // RMSNorm prologue (p.norm_w): every CTA sums the squares of the whole row
    // of x (the same order in every CTA, so every CTA gets the same scale) and
    // stages x * scale * w for its rows (RMSNorm.kt:71-90).
    float nrm = 1.0f;
    if (p.norm_w != nullptr) {
        __shared__ float s_nred[kWarps];
        float ss = 0.0f;
#pragma unroll 4
        for (int i = 4 * tid; i < p.K; i += 4 * kThreads) {
            const float4 v4 = __ldg(reinterpret_cast<const float4*>(p.x + i));
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
        nrm = 1.0f / sqrtf(tot / static_cast<float>(p.K) + p.norm_eps);
    }
    const int n_rows = r_end - r_begin;
    const int n_f4 = n_rows / 8;  // <= 128: four per lane
    float4 xv[4];
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int f = lane + 32 * i;
        const int row = 8 * (2 * (f >> 1) + hw) + 4 * (f & 1);
        xv[i] = f < n_f4 ? __ldg(reinterpret_cast<const float4*>(p.x + r_begin + row)) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (p.norm_w != nullptr && f < n_f4) {
            const float4 w4 = __ldg(reinterpret_cast<const float4*>(p.norm_w + r_begin + row));
            xv[i] = make_float4(xv[i].x * nrm * w4.x, xv[i].y * nrm * w4.y, xv[i].z * nrm * w4.z, xv[i].w * nrm * w4.w);
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
        uint32_t packed[4];  // {xh, xm, xl, 0} of rows row .. row + 3
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
        const int s8 = s4 + __shfl_xor_sync(0xffffffffu, s4, 1);  // the block's 8 rows (lanes f, f ^ 1)
        if (f < n_f4) {
            *reinterpret_cast<uint4*>(xs + 4 * row) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
            if ((f & 1) == 0) sxb[row / kBlockRows] = s8;
        }
    }
    __syncwarp();  // staged x visible to the warp (each warp reads only its own rows)

    // B fragments: in the first MMA column n = g carries part g / 4 (0 = xh,
    // 1 = xm) in byte g % 4, in the second columns g < 4 carry xl in byte g.
    // From the words {xh, xm, xl, 0} of rows 2t and 2t + 1 of a block: b0 = that
    // part of row 2t in byte g % 4, b1 the same of row 2t + 1 (selector nibbles
    // >= 4 pick the zero operand).
    const uint32_t part_byte = static_cast<uint32_t>(g >> 2);
    const uint32_t pos = static_cast<uint32_t>(g & 3);
    const uint32_t sel_hm = (0x4444u & ~(0xFu << (4 * pos))) | (part_byte << (4 * pos));
    const uint32_t sel_l = g < 4 ? (0x4444u & ~(0xFu << (4 * pos))) | (2u << (4 * pos)) : 0x4444u;
    // this lane's 16-byte chunk (words 4g .. 4g+3) of rows 2t and 2t+1 of a block, swizzled
    // (16-byte chunk c of row r sits at chunk c ^ (r & 7)); blocks start on multiples of 8 rows
    const int off0 = (2 * t) * kTileBytes + ((g ^ (2 * t)) << 4);
    const int off1 = (2 * t + 1) * kTileBytes + ((g ^ (2 * t + 1)) << 4);

    // Epilogue columns of this lane: words 4g + j (j = 0..3), bytes 2u, 2u + 1 of
    // each (u = t & 1); low nibbles for t < 2, high nibbles for t >= 2.
    const int u = t & 1;
    const bool low_owner = t < 2;
    float y[2 * kJ];
#pragma unroll
    for (int e = 0; e < 2 * kJ; ++e) y[e] = 0.0f;
    int c[kJ][4];  // {xh, xm} parts
    int e[kJ][4];  // xl part (columns 0-3)
#pragma unroll
    for (int j = 0; j < kJ; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = e[j][0] = e[j][1] = e[j][2] = e[j][3] = 0;
    long long sx = 0;  // this warp's sum of X over the group's rows so far (|X| < 2^22: 64-bit for any group size)
    bool ok = true;
    int done = 0;
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
            ok = __all_sync(0xffffffffu, ok);
        }
        if (hw == 0 && st > 0 && st + kStages - 1 < n_stages) {
            // stage st + NS - 1 into the slot of stage st - 1 once both warps released it
            const int prev = st - 1;
            int go = 0;
            if (lane == 0 && ok)
                go = mbar_wait_bounded(empty + 8 * (prev & (kStages - 1)), (prev / kStages) & 1) ? 1 : 2;
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
        for (int bb = 0; bb < 2; ++bb) {
            const int blk = 2 * bb + hw;                  // 8-row block of the stage
            const int brow = st * kRowsPerStage + blk * kBlockRows;  // inside the slice
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
                for (int j = 0; j < kJ; ++j) {
                    imma_16832(c[j], a[j][0], a[j][1], a[j][2], a[j][3], b0, b1);
                    imma_16832(e[j], a[j][0], a[j][1], a[j][2], a[j][3], l0, l1);
                }
            } else {  // A rows g, g + 8: words 4g + 2jj, 4g + 2jj + 1 of rows 2t (a0, a1) and 2t + 1 (a2, a3)
                imma_16832_s8(c[0], w0.x, w0.y, w1.x, w1.y, b0, b1);
                imma_16832_s8(e[0], w0.x, w0.y, w1.x, w1.y, l0, l1);
                imma_16832_s8(c[kJ - 1], w0.z, w0.w, w1.z, w1.w, b0, b1);
                imma_16832_s8(e[kJ - 1], w0.z, w0.w, w1.z, w1.w, l0, l1);
            }
        }
        // Release the stage once every lane of this warp has read it; with groups
        // of one stage only after the group epilogue below, which reads the
        // group's scale slot -- the slot the refill of stage st + NS - 1 reuses.
        if (!one_stage_groups) {
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + 8 * slot);
        }
        if (r_begin + (st + 1) * kRowsPerStage >= group_end) {
            // Group epilogue.  C of lane (g, t): c[j][0..1] = D[g][2t..2t+1] (low
            // nibbles, byte 2u + 0/1, part t / 2: xh or xm), c[j][2..3] the high
            // nibbles; lanes t and t ^ 2 hold the two parts of the same bytes.
            // e[j] of lanes t < 2 holds the xl part of those bytes (low nibbles in
            // e[j][0..1], high in e[j][2..3]); lanes t >= 2 own the high nibbles
            // and take theirs from lane t ^ 2.
            const unsigned char* sl = slots + ((gi - g_first) & (kStages - 1)) * kScaleSlotBytes;
            const float* s_arr = reinterpret_cast<const float*>(sl + (low_owner ? 0 : kTileBytes * 4));
            const uint8_t* z_arr = sl + kTileBytes * (low_owner ? 8 : 9);
            const float sxf = static_cast<float>(sx);
#pragma unroll
            for (int j = 0; j < kJ; ++j) {
                const int send0 = low_owner ? c[j][2] : c[j][0];
                const int send1 = low_owner ? c[j][3] : c[j][1];
                const int recv0 = __shfl_xor_sync(0xffffffffu, send0, 2);
                const int recv1 = __shfl_xor_sync(0xffffffffu, send1, 2);
                const int lrecv0 = __shfl_xor_sync(0xffffffffu, e[j][2], 2);
                const int lrecv1 = __shfl_xor_sync(0xffffffffu, e[j][3], 2);
                // D = 65536 D_h + 256 D_m + D_l in fp32 (no int32 overflow for any group size)
                const float dh0 = static_cast<float>(low_owner ? c[j][0] : recv0);
                const float dm0 = static_cast<float>(low_owner ? recv0 : c[j][2]);
                const float dl0 = static_cast<float>(low_owner ? e[j][0] : lrecv0);
                const float dh1 = static_cast<float>(low_owner ? c[j][1] : recv1);
                const float dm1 = static_cast<float>(low_owner ? recv1 : c[j][3]);
                const float dl1 = static_cast<float>(low_owner ? e[j][1] : lrecv1);
                const float d0 = fmaf(dh0, 65536.0f, fmaf(dm0, 256.0f, dl0));
                const float d1 = fmaf(dh1, 65536.0f, fmaf(dm1, 256.0f, dl1));
                if constexpr (BITS == 4) {
                    const int b = 16 * g + 4 * j + 2 * u;  // byte of the tile row
                    const float2 s2 = *reinterpret_cast<const float2*>(s_arr + b);
                    const uint32_t z2 = *reinterpret_cast<const uint16_t*>(z_arr + b);
                    const float k16 = low_owner ? 1.0f : 0.0625f;
                    y[2 * j] = fmaf(s2.x, fmaf(d0, k16, -static_cast<float>(z2 & 0xFFu) * sxf), y[2 * j]);
                    y[2 * j + 1] = fmaf(s2.y, fmaf(d1, k16, -static_cast<float>(z2 >> 8) * sxf), y[2 * j + 1]);
                } else {  // word 4g + 2j (rows g, lanes t < 2) or 4g + 2j + 1 (rows g + 8), bytes 2u, 2u + 1
                    const int b = 16 * g + 8 * j + (low_owner ? 0 : 4) + 2 * u;
                    const float2 s2 = *reinterpret_cast<const float2*>(reinterpret_cast<const float*>(sl) + b);
                    y[2 * j] = fmaf(s2.x, d0, y[2 * j]);
                    y[2 * j + 1] = fmaf(s2.y, d1, y[2 * j + 1]);
                }
            }
#pragma unroll
            for (int j = 0; j < kJ; ++j) c[j][0] = c[j][1] = c[j][2] = c[j][3] = e[j][0] = e[j][1] = e[j][2] = e[j][3] = 0;
            sx = 0;
            ++gi;
            group_end = min((gi + 1) * p.gs, r_end);
        }
        if (one_stage_groups) {
            __syncwarp();
            if (lane == 0) mbar_arrive(empty + 8 * slot);
        }
    }
    // After a timeout: wait (bounded) for this slice's copies still in flight
    // before the rings are reused and the CTA's shared memory is released.
    if (producer) {
        for (int s = done; s < p_issued; ++s) {
            if (!mbar_wait_bounded(bars + 8 * (s & (kStages - 1)), (s / kStages) & 1)) break;
        }
    }

    // (1) warps of the CTA in order; red[w][e][lane] reuses the rings.
    __shared__ int s_last;
    __syncthreads();
    float* red = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int e = 0; e < 2 * kJ; ++e) red[(warp * 8 + e) * 32 + lane] = y[e] * unscale;
    __syncthreads();
    // column col = tid (< kCT): byte b = col % 128 of the tile row; INT4: high
    // nibble if col >= 128, lane half hi = the nibble, j = the word of the
    // chunk; INT8: the word jw of the chunk is j = jw / 2, lane half hi = jw % 2.
    // Its lane (g, t) and register e as assigned above.
    float v = 0.0f;
    if (tid < kCT) {
        const int b = tid & (kTileBytes - 1);
        const int gg = b >> 4, jw = (b >> 2) & 3, sg = b & 3;
        const int hi = BITS == 4 ? tid >> 7 : jw & 1;
        const int j = BITS == 4 ? jw : jw >> 1;
        const int ln = 4 * gg + 2 * hi + (sg >> 1);
        const int e = 2 * j + (sg & 1);
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += red[(w * 8 + e) * 32 + ln];
    }
    // output column of tile column col (INT4: low nibbles then high nibbles)
    auto out_col_of = [&](int col) {
        const int byte = tile_b0 + (col & (kTileBytes - 1));
        return BITS == 4 && col >= kTileBytes ? half + byte : byte;
    };
    auto emit = [&](int col, float val) {
        const int byte = tile_b0 + (col & (kTileBytes - 1));
        const int out_col = out_col_of(col);
        if (col < kCT && byte < p.R && out_col < p.N) {
            float* out = p.y + out_col;
            float r = fmaf(p.alpha, val, p.accumulate ? *out : 0.0f);
            if (p.bias != nullptr) r += p.bias[out_col];
            if (p.lora.p != nullptr) r += lora_term(p.lora, 0, out_col, p.N);
            *out = r;
        }
    };
    // Row-parallel exchange (p.tp.nranks > 0), every thread with its column:
    // the call's number is this rank's count of completed calls + 1 (the
    // counter advances only when every CTA of the grid has exited, so the whole
    // grid reads one value, and a replayed CUDA graph gets new ones).  The
    // thread stores {number, alpha * partial} as one 64-bit word into every
    // rank's receive area (slot number & 1, row of this rank), then reads the
    // column's word of every rank in rank order until each carries this number
    // (bounded) and sums their values -- the same bits on every rank.
    auto finish = [&](int col, float val) {
        if (p.tp.nranks == 0) {
            emit(col, val);
            return;
        }
        const int P = p.tp.nranks;
        const uint32_t epoch = *reinterpret_cast<volatile uint32_t*>(p.tp.state) + 1u;
        const int byte = tile_b0 + (col & (kTileBytes - 1));
        const int out_col = out_col_of(col);
        if (!(col < kCT && byte < p.R && out_col < p.N)) return;
        const int64_t slot_base = static_cast<int64_t>(epoch & 1u) * P * p.tp.n_cap;
        const unsigned long long word =
            (static_cast<unsigned long long>(epoch) << 32) | __float_as_uint(p.alpha * val);
        for (int q = 0; q < P; ++q)
            st_relaxed_sys_u64(p.tp.recv[q] + slot_base + static_cast<int64_t>(p.tp.rank) * p.tp.n_cap + out_col, word);
        const unsigned long long* mine = p.tp.recv[p.tp.rank] + slot_base + out_col;
        float sum = 0.0f;
        for (int src = 0; src < P; ++src) {
            float v = 0.0f;
            if (!wait_word_sys(mine + static_cast<int64_t>(src) * p.tp.n_cap, epoch, p.tp.wait_ns, &v)) {
                atomicOr(p.err, 1);
                return;
            }
            sum += v;
        }
        float* out = p.y + out_col;
        float r = sum + (p.accumulate ? *out : 0.0f);
        if (p.bias != nullptr) r += p.bias[out_col];
        *out = r;
    };
    // the grid's last CTA to exit advances this rank's call counter
    auto tp_exit = [&]() {  // every thread of the CTA (uniform)
        if (p.tp.nranks == 0) return;
        __syncthreads();  // every thread of the CTA has read this call's number
        if (tid != 0) return;
        __threadfence();
        const uint32_t total = gridDim.x * gridDim.y;
        if (atomicAdd(p.tp.state + 1, 1u) == total - 1) {  // the grid's last CTA
            p.tp.state[1] = 0;
            p.tp.state[0] += 1;
            __threadfence();
        }
    };
    // SwiGLU epilogue (p.swiglu; no exchange, no accumulate): every thread of
    // the CTA with its column tid; the gate column of byte b (low nibble, thread
    // b) and its up column (high nibble, thread 128 + b) meet in shared memory
    // (SwiGLU.forwardInto: silu(gate) * up, Tensor.kt:231-237).
    __shared__ float s_swig[2 * kTileBytes];
    auto swiglu_out = [&](int b, float g, float u) {
        g = fmaf(p.alpha, g, 0.0f);  // the arithmetic of emit(), so both paths give the same bits
        u = fmaf(p.alpha, u, 0.0f);
        if (p.bias != nullptr) {
            g += p.bias[b];
            u += p.bias[half + b];
        }
        if (p.lora.p != nullptr) {
            g += lora_term(p.lora, 0, b, p.N);
            u += lora_term(p.lora, 0, half + b, p.N);
        }
        p.y[b] = g / (1.0f + expf(-g)) * u;
    };
    auto finish_swiglu = [&](float val) {
        s_swig[tid] = val;
        __syncthreads();
        const int byte = tile_b0 + tid;
        if (tid < kTileBytes && byte < p.R) swiglu_out(byte, s_swig[tid], s_swig[tid + kTileBytes]);
    };
    const int S = gridDim.y;
    if (S == 1) {
        if (p.swiglu) finish_swiglu(v);
        else finish(tid, v);
        tp_exit();
        return;
    }
    if (p.cluster) {
        // (2a) the S CTAs of the tile form one thread-block cluster: each puts
        // its partial tile in its own shared memory; after the cluster barrier,
        // rank r sums columns [r * per, (r + 1) * per) over the ranks in rank
        // (= split) order through distributed shared memory; a second barrier
        // keeps every CTA's shared memory alive until all ranks have read it.
        __shared__ float cpart[kCT];
        if (tid < kCT) cpart[tid] = v;
        cluster_sync();
        if (BITS == 4 && p.swiglu) {  // rank r sums both columns of bytes [r * per, (r + 1) * per)
            const int per = (kTileBytes + S - 1) / S;
            const int b = static_cast<int>(cluster_rank()) * per + tid;
            if (tid < per && b < kTileBytes && tile_b0 + b < p.R) {
                float g = 0.0f, u = 0.0f;
                for (int j = 0; j < S; ++j) {  // split order
                    g += ld_dsmem(smem_u32(cpart + b), j);
                    u += ld_dsmem(smem_u32(cpart + (kCT - kTileBytes) + b), j);
                }
                swiglu_out(tile_b0 + b, g, u);
            }
            cluster_sync();
            return;
        }
        const int per = (kCT + S - 1) / S;
        const int col = static_cast<int>(cluster_rank()) * per + tid;
        if (tid < per && col < kCT) {
            const uint32_t local = smem_u32(cpart + col);
            float tv[kMaxSplits];
#pragma unroll
            for (int j = 0; j < kMaxSplits; ++j) tv[j] = j < S ? ld_dsmem(local, j) : 0.0f;
            float sum = 0.0f;
#pragma unroll
            for (int j = 0; j < kMaxSplits; ++j)
                if (j < S) sum += tv[j];
            emit(col, sum);
        }
        cluster_sync();
        return;
    }
    // (2b) split-K through global memory: every CTA of the tile publishes its partial tile; the last to
    // arrive sums all of them in split order (the CTA barrier orders every
    // thread's store before thread 0's acq_rel atomic; the second barrier hands
    // the acquire to the whole CTA).
    float* tile_parts = p.partials + static_cast<int64_t>(blockIdx.x) * S * kCT;
    if (tid < kCT) __stcg(tile_parts + static_cast<int64_t>(blockIdx.y) * kCT + tid, v);
    __syncthreads();
    if (tid == 0) s_last = atomic_add_acq_rel(p.tickets + blockIdx.x, 1) == S - 1;
    __syncthreads();
    if (!s_last) {
        tp_exit();
        return;
    }
    // up to 32 partial loads in flight per thread, summed in split order
    float sum = 0.0f;
    for (int s0 = 0; s0 < S; s0 += 32) {
        float tv[32];
#pragma unroll
        for (int j = 0; j < 32; ++j)
            tv[j] = s0 + j == static_cast<int>(blockIdx.y) ? v
                    : s0 + j < S && tid < kCT ? __ldcg(tile_parts + static_cast<int64_t>(s0 + j) * kCT + tid) : 0.0f;
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (s0 + j < S) sum += tv[j];
    }
    if (p.swiglu) finish_swiglu(sum);
    else finish(tid, sum);
    if (tid == 0) p.tickets[blockIdx.x] = 0;  // ready for the next launch on this workspace
    tp_exit();
}

int tiles_of(int R) { return (R + kTileBytes - 1) / kTileBytes; }

// Per-device caches below are atomics: host threads may launch on one device
// concurrently (a lost race only repeats an idempotent query).
int blocks_per_sm() {
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
    // the INT4 kernel: the INT8 one has the same shared memory and no more registers
    if (cudaFuncSetAttribute(gemv_imma_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemBytes)) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_imma_kernel<4>, kThreads, kSmemBytes) != cudaSuccess)
        n = 1;
    cudaGetLastError();
    n = std::max(n, 1);
    if (slot != nullptr) slot->store(n, std::memory_order_release);
    return n;
}

int min_splits(int K) {
    const int per = kPairs * kMaxSliceRows;
    return (K + per - 1) / per;
}

std::atomic<int>& split_override() {
    static std::atomic<int> o{[] {
        const char* v = std::getenv("KT_IMMA_SPLITS");
        return v ? std::atoi(v) : 0;
    }()};
    return o;
}

// K-splits per column tile: enough CTAs to fill the SM slots of one wave, at
// most kMaxSplits (each split adds a partial the finishing CTA must read and a
// CTA's fixed costs; measured on B200, more than 16 splits of a tile never paid
// off), at least one stage per slice, never fewer than min_splits.
int choose_splits(int R, int K, int sm_count) {
    const int tiles = tiles_of(R);
    const int slots = blocks_per_sm() * sm_count;
    const int k_stages = K / kRowsPerStage;
    int s = std::min(kMaxSplits, std::max(1, slots / tiles));
    s = std::min(s, std::max(1, k_stages / kPairs));
    const int pinned = split_override().load(std::memory_order_relaxed);
    if (pinned >= 1) s = pinned;
    s = std::max(s, min_splits(K));
    return tiles > kTicketCapEach ? min_splits(K) : s;
}

// The kernel's shared-memory and cluster-size attributes, set once per device
// (setting them on every launch costs host time on a latency-bound call).
cudaError_t prepare_kernel() {
    constexpr int kMaxDevices = 64;
    static std::atomic<bool> done[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < kMaxDevices && done[dev].load(std::memory_order_acquire)) return cudaSuccess;
    for (auto kernel : {gemv_imma_kernel<4>, gemv_imma_kernel<8>}) {
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes));
        if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    }
    if (e == cudaSuccess && dev >= 0 && dev < kMaxDevices) done[dev].store(true, std::memory_order_release);
    return e;
}

// Clusters of `c` CTAs of this kernel the GPU holds at once (cached per device).
int active_clusters(int c) {
    constexpr int kMaxDevices = 64;
    static std::atomic<int> cache[kMaxDevices][kMaxSplits + 1] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    std::atomic<int>* slot = dev >= 0 && dev < kMaxDevices ? &cache[dev][c] : nullptr;
    if (slot != nullptr) {
        const int v = slot->load(std::memory_order_acquire);
        if (v != 0) return v - 1;
    }
    int n = 0;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(1, c, 1);
    lc.blockDim = dim3(kThreads, 1, 1);
    lc.dynamicSmemBytes = kSmemBytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = c;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    if (cudaFuncSetAttribute(gemv_imma_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemBytes)) != cudaSuccess ||
        cudaFuncSetAttribute(gemv_imma_kernel<4>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess ||
        cudaOccupancyMaxActiveClusters(&n, gemv_imma_kernel<4>, &lc) != cudaSuccess)
        n = 0;
    cudaGetLastError();
    if (slot != nullptr) slot->store(n + 1, std::memory_order_release);
    return n;
}

bool clusters_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("KT_IMMA_CLUSTER");
        return v == nullptr || std::atoi(v) != 0;
    }();
    return on;
}

struct Plan {
    int splits;
    bool cluster;
};

// The split count, and whether the splits of a tile reduce inside a cluster
// (the largest count up to choose_splits' whose clusters all fit at once).
// Clusters only for short slices: measured on B200, the cluster reduction
// saves ~0.2-0.3 us where the tail dominates (slices of <= 4 stages) and
// costs ~1 us on long slices (cluster co-scheduling delays the early start of
// CTAs behind the previous kernel).
Plan plan_for(int R, int K, int sm_count, bool no_cluster = false) {
    const int s = choose_splits(R, K, sm_count);
    const int tiles = tiles_of(R);
    const int stages_per_slice = K / kRowsPerStage / (s * kPairs);
    if (!no_cluster && s > 1 && s <= kMaxSplits && clusters_enabled() && stages_per_slice <= 4) {
        for (int c = s; c >= std::max(2, min_splits(K)); --c) {
            if (active_clusters(c) >= tiles) return {c, true};
            if (split_override().load(std::memory_order_relaxed) >= 1) break;  // a pinned count is used as given
        }
    }
    return {s, false};
}

}  // namespace

void set_imma_tuning(int k_splits) { split_override().store(k_splits, std::memory_order_relaxed); }

bool gemv_imma_supported(const QView& w, int32_t m, const float* a) {
    if ((w.bits != 4 && w.bits != 8) || m != 1 || w.tmap_mma == nullptr) return false;
    if (a != nullptr && reinterpret_cast<uintptr_t>(a) % 16 != 0) return false;
    return w.columns % 32 == 0 && w.rows % kRowsPerStage == 0 && w.group_size % kRowsPerStage == 0 &&
           min_splits(w.rows) <= 65535 && (min_splits(w.rows) == 1 || tiles_of(w.bytes_per_row) <= kTicketCapEach);
}

size_t gemv_imma_workspace_bytes(const QView& w, int sm_count, bool no_cluster) {
    const Plan plan = plan_for(w.bytes_per_row, w.rows, sm_count, no_cluster);
    if (plan.splits <= 1 || plan.cluster) return 0;
    return kWorkspaceReservedBytes +
           static_cast<size_t>(tiles_of(w.bytes_per_row)) * plan.splits * (w.bits == 4 ? ct_of<4>() : ct_of<8>()) *
               sizeof(float);
}

bool norm_fused_supported(const QView& w, int32_t m, const float* a) { return gemv_imma_supported(w, m, a); }

bool swiglu_fused_supported(const QView& w, int32_t m, const float* a) {
    return gemv_imma_supported(w, m, a) && w.columns == 2 * w.bytes_per_row;
}

bool gemv_imma_tp_supported(const QView& w, int sm_count) {
    if (!gemv_imma_supported(w, 1, nullptr)) return false;
    const Plan plan = plan_for(w.bytes_per_row, w.rows, sm_count, true);
    return static_cast<int64_t>(tiles_of(w.bytes_per_row)) * plan.splits <=
           static_cast<int64_t>(blocks_per_sm()) * sm_count;
}

cudaError_t launch_gemv_imma(const QView& w, const MatmulArgs& a, int sm_count, cudaStream_t s, void* workspace,
                             size_t workspace_bytes) {
    ImmaParams p{};
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
    p.tp = a.tp;
    p.swiglu = a.swiglu;
    p.norm_w = a.norm_weight;
    p.norm_eps = a.norm_eps;
    if (a.norm_weight != nullptr && reinterpret_cast<uintptr_t>(a.norm_weight) % 16 != 0) return cudaErrorInvalidValue;
    if (a.swiglu && (a.tp.nranks > 0 || a.accumulate || w.columns != 2 * w.bytes_per_row)) return cudaErrorInvalidValue;
    const bool no_cluster = a.tp.nranks > 0;
    const Plan plan = plan_for(p.R, p.K, sm_count, no_cluster);
    p.cluster = plan.cluster ? 1 : 0;
    if (plan.splits > 1 && !plan.cluster) {
        if (workspace == nullptr || workspace_bytes < gemv_imma_workspace_bytes(w, sm_count, no_cluster))
            return cudaErrorInvalidValue;
        p.tickets = reinterpret_cast<int32_t*>(static_cast<unsigned char*>(workspace) + kGemvTicketOffset);
        p.partials = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + kWorkspaceReservedBytes);
    }
    const cudaError_t e = prepare_kernel();
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(tiles_of(p.R), plan.splits, 1);
    lc.blockDim = dim3(kThreads, 1, 1);
    lc.dynamicSmemBytes = kSmemBytes;
    lc.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = plan.splits;
    attr[1].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = plan.cluster ? 2 : 1;
    return cudaLaunchKernelEx(&lc, w.bits == 4 ? gemv_imma_kernel<4> : gemv_imma_kernel<8>, *w.tmap_mma, p);
}

}  // namespace kt
