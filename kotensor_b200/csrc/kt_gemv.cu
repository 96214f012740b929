// kt_gemv.cu -- fp32-accumulate dequantizing matmul for small m (the decode
// GEMV), MatMul.multiplyQuantized for m <= kGemvMaxM
// (Engine/kotensor/src/main/kotlin/MatMul.kt:460-536 and :599-828).
//
// The reference factors each group g and output column j as
//   c[j] += alpha * scale[g,j] * (sum_l a_l * q[l,j]  -  zero[g,j] * sum_l a_l)
// with q the raw unsigned nibble (INT4) or the signed byte (INT8)
// (combineGroup, MatMul.kt:804-828).  This kernel keeps that factoring: each
// lane owns LB contiguous packed bytes of every row it visits (INT4: 2*LB
// columns, the low nibbles for columns cb.. and the high nibbles for columns
// half+cb..; INT8: LB columns), walks a contiguous range of rows, and applies
// scale and zero once per group (or once per partial group at a range edge: the
// factoring is linear in the rows).
//
// Streaming.  Each warp owns a ring of kStages shared-memory stages of
// kStageRows rows x 32*LB bytes.  Lane 0 fills a stage with one or two 2-D TMA
// copies (cp.async.bulk.tensor, completion on the stage's mbarrier) and keeps
// kStages-1 stages in flight, so memory-level parallelism does not depend on
// registers or occupancy; every lane reads its bytes back with one vector
// shared load per row at a compile-time offset.  The group's scales and zero
// points are fetched into registers when the group starts and consumed when it
// ends.  The kernel is launched with programmatic stream serialization: the
// weight prefetch starts before the previous kernel in the stream has finished,
// and griddepcontrol.wait orders every read of x and every write of y after it.
// Every mbarrier wait is bounded (globaltimer); a timeout sets the context's
// error word and the kernel runs on to its barriers and exits.
//
// Unpacking without int->float conversions.  A nibble or byte q placed in the
// top mantissa bits of the float 2^23 (bits 0x4B000000) gives the exact float
// 2^23 + q*2^p with one LOP3 (the 2^23 pattern comes in as a kernel argument so
// the mask is the instruction's only immediate); one exact FADD removes the
// offset (q*2^p for INT4; INT8 bytes are offset to unsigned by xor 0x80 and
// 2^23 + 2^22 is removed, leaving the signed b*2^15), and fp32 FMAs accumulate
// T = sum_l a_l*q*2^p alone -- fp32-class, where accumulating the offset too
// (an earlier version) cost up to 11 bits of the accumulator.
//   INT4 low nibbles sit at bits 16-19 (p = 16), high nibbles at bits 12-15
//   (p = 12): 3 shift/permute ops + 8 LOP3 + 8 FADD + 8 FFMA per 32-bit word of
//   8 weights.  INT8 bytes sit at bits 15-22 (p = 15).
// The group epilogue: y += scale * (T*2^-p - zero * sum_l a_l).
//
// Split-K and the reduction order.  Each warp owns one contiguous row range
// ("slice").  Slice partials are reduced in a fixed order: across the 8 warps
// of a CTA (shared memory, warp order) and across the CK CTAs of a thread-block
// cluster along K (distributed shared memory, rank order).  No atomics and no
// global scratch: the same inputs give the same bits on every run.
#include <cooperative_groups.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>

#include "kt_internal.h"

namespace cg = cooperative_groups;

namespace kt {
namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kRS = kStageRows;  // rows per stage
constexpr int kStages = 4;       // stages per warp ring
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // bounded mbarrier waits: 2 s

struct GemvParams {
    const uint8_t* q;
    const float* scales;
    const uint8_t* zeros;
    const float* x;
    float* y;
    const float* bias;
    int32_t* err;
    int32_t K, N, R, gs;
    int32_t slice_rows;  // rows per warp slice (multiple of kRS)
    uint32_t magic;      // 0x4B000000, the float 2^23
    float alpha;
    int32_t accumulate;
    LoraEpilogue lora;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
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
// Waits for the mbarrier phase with a time limit; false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer();
    while (!mbar_try_wait(bar, parity)) {
        if (globaltimer() - t0 > kWaitLimitNs) return false;
    }
    return true;
}

// 2-D TMA load of a box at (x = byte column, y = row) into shared memory.  The
// destination is this CTA's own shared memory; no multicast.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

// Programmatic dependent launch: wait for the previous kernel in the stream
// before touching its outputs; let the next kernel start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// (w & MASK) | magic as a float, less the float's offset OFF: one LOP3
// (0xEA = a & b | c) and one exact FADD.
template <uint32_t MASK>
__device__ __forceinline__ float nib(uint32_t w, uint32_t magic, float off) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(w), "n"(MASK), "r"(magic));
    return __uint_as_float(d) - off;
}
constexpr float kOff4 = 8388608.0f;    // 2^23: the INT4 float 2^23 + q 2^p less 2^23 is q 2^p
constexpr float kOff8 = 12582912.0f;   // 2^23 + 2^22: the INT8 float 2^23 + (b + 128) 2^15 less this is b 2^15

// One 32-bit word of 4 packed INT4 bytes: low nibbles -> columns lo+0..3,
// high nibbles -> columns hi+0..3 (indices into the lane's T array).
template <int M, int C>
__device__ __forceinline__ void fma_int4_word(uint32_t w, uint32_t magic, const float (&xv)[M], float (&T)[M][C],
                                              int lo, int hi) {
    const uint32_t wl = w << 8, wr = w >> 8;
    const uint32_t t = __byte_perm(w, 0u, 0x4034);  // byte0 -> bits 16-23, byte3 -> bits 8-15
    const float f_lo0 = nib<0x000F0000u>(t, magic, kOff4);
    const float f_hi3 = nib<0x0000F000u>(t, magic, kOff4);
    const float f_lo1 = nib<0x000F0000u>(wl, magic, kOff4);
    const float f_hi0 = nib<0x0000F000u>(wl, magic, kOff4);
    const float f_lo2 = nib<0x000F0000u>(w, magic, kOff4);
    const float f_hi1 = nib<0x0000F000u>(w, magic, kOff4);
    const float f_lo3 = nib<0x000F0000u>(wr, magic, kOff4);
    const float f_hi2 = nib<0x0000F000u>(wr, magic, kOff4);
#pragma unroll
    for (int m = 0; m < M; ++m) {
        T[m][lo + 0] = fmaf(xv[m], f_lo0, T[m][lo + 0]);
        T[m][lo + 1] = fmaf(xv[m], f_lo1, T[m][lo + 1]);
        T[m][lo + 2] = fmaf(xv[m], f_lo2, T[m][lo + 2]);
        T[m][lo + 3] = fmaf(xv[m], f_lo3, T[m][lo + 3]);
        T[m][hi + 0] = fmaf(xv[m], f_hi0, T[m][hi + 0]);
        T[m][hi + 1] = fmaf(xv[m], f_hi1, T[m][hi + 1]);
        T[m][hi + 2] = fmaf(xv[m], f_hi2, T[m][hi + 2]);
        T[m][hi + 3] = fmaf(xv[m], f_hi3, T[m][hi + 3]);
    }
}

// One 32-bit word of 4 signed INT8 bytes -> columns at+0..3.
template <int M, int C>
__device__ __forceinline__ void fma_int8_word(uint32_t w, uint32_t magic, const float (&xv)[M], float (&T)[M][C],
                                              int at) {
    const uint32_t u = w ^ 0x80808080u;  // two's complement byte b -> unsigned b + 128
    const float f0 = nib<0x007F8000u>(u << 15, magic, kOff8);
    const float f1 = nib<0x007F8000u>(u << 7, magic, kOff8);
    const float f2 = nib<0x007F8000u>(u >> 1, magic, kOff8);
    const float f3 = nib<0x007F8000u>(u >> 9, magic, kOff8);
#pragma unroll
    for (int m = 0; m < M; ++m) {
        T[m][at + 0] = fmaf(xv[m], f0, T[m][at + 0]);
        T[m][at + 1] = fmaf(xv[m], f1, T[m][at + 1]);
        T[m][at + 2] = fmaf(xv[m], f2, T[m][at + 2]);
        T[m][at + 3] = fmaf(xv[m], f3, T[m][at + 3]);
    }
}

template <int BITS, int M, int LB>
struct Tile {
    static constexpr int C = BITS == 4 ? 2 * LB : LB;   // columns per lane
    static constexpr int WORDS = LB / 4;
    static constexpr int WB = 32 * LB;                  // packed bytes per row of a CTA tile
    static constexpr int CT = BITS == 4 ? 2 * WB : WB;   // columns per CTA tile (= 32 * C)
    static constexpr int BOX = WB < 256 ? WB : 256;     // TMA box width in bytes
    static constexpr int NBOX = WB / BOX;
    static constexpr int STAGE = kRS * WB;              // bytes per stage
    static constexpr int RING = kStages * STAGE;        // bytes per warp ring
    static constexpr int RED = kWarps * M * CT * 4;     // warp partials, reuses the rings
    static constexpr int MAIN = (kWarps * RING > RED ? kWarps * RING : RED);
    static constexpr int PART = M * CT * 4;
    static constexpr int BARS = kWarps * kStages * 8;
    static constexpr size_t SMEM = MAIN + PART + BARS;
};

template <typename T>
__device__ __forceinline__ T lds(const unsigned char* p) {
    return *reinterpret_cast<const T*>(p);
}

// Shared memory: rings[8][NS][RS][WB] (later red[8][M][C][32]) | part[M][CT] | mbarriers[8][NS].
template <int BITS, int M, int LB>
__global__ void __launch_bounds__(kThreads, 1)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap tmap, GemvParams p) {
    using S = Tile<BITS, M, LB>;
    constexpr int C = S::C;
    extern __shared__ __align__(1024) unsigned char smem[];

    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int tile_b0 = blockIdx.x * S::WB;
    const int cb = tile_b0 + lane * LB;  // this lane's first packed byte
    const bool active = cb < p.R;
    const int half = p.R;                // INT4: high-nibble columns start here

    const int slice = blockIdx.y * kWarps + warp;
    const int r_begin = min(slice * p.slice_rows, p.K);
    const int r_end = min(r_begin + p.slice_rows, p.K);
    const int n_stages = (r_end - r_begin + kRS - 1) / kRS;

    unsigned char* ring = smem + warp * S::RING;
    float* part = reinterpret_cast<float*>(smem + S::MAIN);
    const uint32_t bars = smem_u32(smem + S::MAIN + S::PART) + warp * kStages * 8;
    const uint32_t ring_s = smem_u32(ring);
    // Offset of this lane's bytes inside a stage: box (lane*LB / BOX), then row-major [row][BOX].
    const int lane_off = (lane * LB / S::BOX) * kRS * S::BOX + (lane * LB) % S::BOX;

    if (lane == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(bars + 8 * s, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    auto issue = [&](int stage) {  // lane 0 only
        const int slot = stage % kStages;
        const uint32_t bar = bars + 8 * slot;
        mbar_expect_tx(bar, S::STAGE);
#pragma unroll
        for (int b = 0; b < S::NBOX; ++b)
            tma_load_2d(ring_s + slot * S::STAGE + b * kRS * S::BOX, &tmap, tile_b0 + b * S::BOX,
                        r_begin + stage * kRS, bar);
    };
    // Weight prefetch: independent of the previous kernel in the stream.
    if (lane == 0) {
        for (int s = 0; s < kStages - 1 && s < n_stages; ++s) issue(s);
    }
    pdl_launch_dependents();
    pdl_wait();  // x and y below may belong to the previous kernel

    float y[M][C], T[M][C], rs[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
        rs[m] = 0.0f;
#pragma unroll
        for (int j = 0; j < C; ++j) y[m][j] = T[m][j] = 0.0f;
    }
    float sc[C];                                 // scales of the current group
    uint32_t zw[BITS == 4 ? 2 * S::WORDS : 1];   // packed zero points of the current group
    auto load_scales = [&](int g) {
        if (!active) return;
        const int64_t go = static_cast<int64_t>(g) * p.N;
        const float4* s_lo = reinterpret_cast<const float4*>(p.scales + go + cb);
#pragma unroll
        for (int v = 0; v < LB / 4; ++v) {
            const float4 f = __ldg(s_lo + v);
            sc[4 * v] = f.x, sc[4 * v + 1] = f.y, sc[4 * v + 2] = f.z, sc[4 * v + 3] = f.w;
        }
        if constexpr (BITS == 4) {
            const float4* s_hi = reinterpret_cast<const float4*>(p.scales + go + half + cb);
#pragma unroll
            for (int v = 0; v < LB / 4; ++v) {
                const float4 f = __ldg(s_hi + v);
                sc[LB + 4 * v] = f.x, sc[LB + 4 * v + 1] = f.y, sc[LB + 4 * v + 2] = f.z, sc[LB + 4 * v + 3] = f.w;
            }
            const uint8_t* z_lo = p.zeros + go + cb;
            const uint8_t* z_hi = p.zeros + go + half + cb;
            if constexpr (LB == 16) {
                const uint4 a = __ldg(reinterpret_cast<const uint4*>(z_lo));
                const uint4 b = __ldg(reinterpret_cast<const uint4*>(z_hi));
                zw[0] = a.x, zw[1] = a.y, zw[2] = a.z, zw[3] = a.w;
                zw[4] = b.x, zw[5] = b.y, zw[6] = b.z, zw[7] = b.w;
            } else if constexpr (LB == 8) {
                const uint2 a = __ldg(reinterpret_cast<const uint2*>(z_lo));
                const uint2 b = __ldg(reinterpret_cast<const uint2*>(z_hi));
                zw[0] = a.x, zw[1] = a.y, zw[2] = b.x, zw[3] = b.y;
            } else {
                zw[0] = __ldg(reinterpret_cast<const uint32_t*>(z_lo));
                zw[1] = __ldg(reinterpret_cast<const uint32_t*>(z_hi));
            }
        }
    };
    // Group epilogue: y += scale * (T * 2^-p - zero * rowSum); resets T and rs.
    auto finish_group = [&]() {
#pragma unroll
        for (int j = 0; j < C; ++j) {
            float pscale, zoff;
            if constexpr (BITS == 4) {
                const bool lo = j < LB;
                const int jj = lo ? j : j - LB;
                const uint32_t zb = (zw[(lo ? 0 : S::WORDS) + jj / 4] >> (8 * (jj % 4))) & 0xFFu;
                pscale = lo ? 0x1p-16f : 0x1p-12f;
                zoff = static_cast<float>(zb);
            } else {
                pscale = 0x1p-15f;
                zoff = 0.0f;
            }
#pragma unroll
            for (int m = 0; m < M; ++m) y[m][j] = fmaf(sc[j], fmaf(T[m][j], pscale, -zoff * rs[m]), y[m][j]);
        }
#pragma unroll
        for (int m = 0; m < M; ++m) {
            rs[m] = 0.0f;
#pragma unroll
            for (int j = 0; j < C; ++j) T[m][j] = 0.0f;
        }
    };

    const uint32_t magic = p.magic;
    int g = r_begin / p.gs;
    int group_end = min((g + 1) * p.gs, r_end);
    if (r_begin < r_end) load_scales(g);
    bool ok = true;

    for (int st = 0; st < n_stages; ++st) {
        const int slot = st % kStages;
        if (ok && !mbar_wait_bounded(bars + 8 * slot, (st / kStages) & 1)) {
            ok = false;
            if (lane == 0) atomicOr(p.err, 1);
        }
        __syncwarp();  // every lane is done with the slot consumed at st - 1
        if (lane == 0 && ok && st + kStages - 1 < n_stages) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(st + kStages - 1);
        }
        const int row0 = r_begin + st * kRS;
        float xs[kRS][M];
        if (row0 + kRS <= r_end) {
#pragma unroll
            for (int m = 0; m < M; ++m) {
                const float4* xp = reinterpret_cast<const float4*>(p.x + static_cast<int64_t>(m) * p.K + row0);
                const float4 a = __ldg(xp), b = __ldg(xp + 1);
                xs[0][m] = a.x, xs[1][m] = a.y, xs[2][m] = a.z, xs[3][m] = a.w;
                xs[4][m] = b.x, xs[5][m] = b.y, xs[6][m] = b.z, xs[7][m] = b.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < kRS; ++i)
#pragma unroll
                for (int m = 0; m < M; ++m)
                    xs[i][m] = row0 + i < r_end ? __ldg(p.x + static_cast<int64_t>(m) * p.K + row0 + i) : 0.0f;
        }
        const unsigned char* stage_base = ring + slot * S::STAGE + lane_off;
#pragma unroll
        for (int i = 0; i < kRS; ++i) {
            uint32_t wv[S::WORDS];
            if constexpr (LB == 16) {
                const uint4 v = lds<uint4>(stage_base + i * S::BOX);
                wv[0] = v.x, wv[1] = v.y, wv[2] = v.z, wv[3] = v.w;
            } else if constexpr (LB == 8) {
                const uint2 v = lds<uint2>(stage_base + i * S::BOX);
                wv[0] = v.x, wv[1] = v.y;
            } else {
                wv[0] = lds<uint32_t>(stage_base + i * S::BOX);
            }
#pragma unroll
            for (int m = 0; m < M; ++m) rs[m] += xs[i][m];
#pragma unroll
            for (int k = 0; k < S::WORDS; ++k) {
                if constexpr (BITS == 4) {
                    fma_int4_word<M, C>(wv[k], magic, xs[i], T, 4 * k, LB + 4 * k);
                } else {
                    fma_int8_word<M, C>(wv[k], magic, xs[i], T, 4 * k);
                }
            }
        }
        // Groups are multiples of kRS rows, so group ends fall on stage ends.
        if (row0 + kRS >= group_end) {
            finish_group();
            ++g;
            group_end = min((g + 1) * p.gs, r_end);
            if (row0 + kRS < r_end) load_scales(g);
        }
    }

    // (1) warps of the CTA, in warp order -> part[m][col-in-tile]
    __syncthreads();  // every ring is drained: its memory becomes red[warp][m][j][lane]
    float* red = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int j = 0; j < C; ++j) red[((warp * M + m) * C + j) * 32 + lane] = active ? y[m][j] : 0.0f;
    __syncthreads();
    for (int t = tid; t < M * S::CT; t += kThreads) {
        const int m = t / S::CT;
        const int jt = t % S::CT;
        int ln, j;
        if constexpr (BITS == 4) {
            const int hi = jt >= S::WB;
            const int jb = hi ? jt - S::WB : jt;
            ln = jb / LB;
            j = (hi ? LB : 0) + jb % LB;
        } else {
            ln = jt / LB;
            j = jt % LB;
        }
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) v += red[((w * M + m) * C + j) * 32 + ln];
        part[t] = v;
    }
    // (2) CTAs of the cluster along K, in rank order; CTA rank r finishes
    // columns [r*CT/CK, (r+1)*CT/CK) of every row m.
    cg::cluster_group cluster = cg::this_cluster();
    const int CK = gridDim.y;
    if (CK > 1) cluster.sync(); else __syncthreads();
    const int rank = CK > 1 ? static_cast<int>(cluster.block_rank()) : 0;
    const int j0 = rank * S::CT / CK, j1 = (rank + 1) * S::CT / CK;
    const int span = j1 - j0;
    for (int t = tid; t < M * span; t += kThreads) {
        const int m = t / span;
        const int j = j0 + t % span;
        float v;
        if (CK > 1) {
            v = 0.0f;
            for (int q = 0; q < CK; ++q) v += cluster.map_shared_rank(part, q)[m * S::CT + j];
        } else {
            v = part[m * S::CT + j];
        }
        int col, byte;
        if constexpr (BITS == 4) {
            byte = tile_b0 + (j < S::WB ? j : j - S::WB);
            col = j < S::WB ? byte : half + byte;
        } else {
            byte = tile_b0 + j;
            col = byte;
        }
        if (byte < p.R && col < p.N) {
            float* out = p.y + static_cast<int64_t>(m) * p.N + col;
            float r = fmaf(p.alpha, v, p.accumulate ? *out : 0.0f);
            if (p.bias != nullptr) r += p.bias[col];
            if (p.lora.p != nullptr) r += lora_term(p.lora, m, col, p.N);
            *out = r;
        }
    }
    if (CK > 1) cluster.sync();  // keep this CTA's shared memory alive until every rank has read it
}

// ---------------------------------------------------------------- generic fallback
// Any shape (odd N, unaligned rows, group sizes that are not multiples of 8)
// and any m: one thread per packed byte column and output row, 8 warps split
// the groups, fixed-order smem reduction.  Plain int->float conversion; used
// only where the streaming kernel's alignment rules do not hold.
__global__ void __launch_bounds__(256) matmul_generic_kernel(GemvParams p) {
    __shared__ float red[8][2][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int b = blockIdx.x * 32 + lane;  // packed byte column
    const int m = blockIdx.y;
    const bool is4 = p.zeros != nullptr;
    const int half = p.R;
    const bool active = b < p.R;
    const bool has_hi = is4 && active && b + half < p.N;
    const int G = (p.K + p.gs - 1) / p.gs;
    float y_lo = 0.0f, y_hi = 0.0f;
    const float* xr = p.x + static_cast<int64_t>(m) * p.K;
    for (int g = warp; g < G; g += 8) {
        const int r0 = g * p.gs, r1 = min(r0 + p.gs, p.K);
        float a_lo = 0.0f, a_hi = 0.0f, rs = 0.0f;
        if (active) {
            for (int r = r0; r < r1; ++r) {
                const float xv = xr[r];
                const uint8_t byte = p.q[static_cast<int64_t>(r) * p.R + b];
                rs += xv;
                if (is4) {
                    a_lo = fmaf(xv, static_cast<float>(byte & 0xF), a_lo);
                    a_hi = fmaf(xv, static_cast<float>(byte >> 4), a_hi);
                } else {
                    a_lo = fmaf(xv, static_cast<float>(static_cast<int8_t>(byte)), a_lo);
                }
            }
            const int64_t go = static_cast<int64_t>(g) * p.N;
            if (is4) {
                y_lo = fmaf(p.scales[go + b], a_lo - static_cast<float>(p.zeros[go + b]) * rs, y_lo);
                if (has_hi)
                    y_hi = fmaf(p.scales[go + half + b], a_hi - static_cast<float>(p.zeros[go + half + b]) * rs, y_hi);
            } else {
                y_lo = fmaf(p.scales[go + b], a_lo, y_lo);
            }
        }
    }
    red[warp][0][lane] = y_lo;
    red[warp][1][lane] = y_hi;
    __syncthreads();
    if (warp < 2) {
        float v = 0.0f;
        for (int w = 0; w < 8; ++w) v += red[w][warp][lane];
        const bool hi = warp == 1;
        if (active && (!hi || has_hi)) {
            const int col = hi ? half + b : b;
            float* out = p.y + static_cast<int64_t>(m) * p.N + col;
            float r = fmaf(p.alpha, v, p.accumulate ? *out : 0.0f);
            if (p.bias != nullptr) r += p.bias[col];
            if (p.lora.p != nullptr) r += lora_term(p.lora, m, col, p.N);
            *out = r;
        }
    }
}

// ---------------------------------------------------------------- dispatch

struct GemvConfig {
    int lb, ck;
};

int env_int(const char* name, int fallback) {
    const char* v = std::getenv(name);
    return v ? std::atoi(v) : fallback;
}

template <int BITS, int M, int LB>
cudaError_t launch_cfg(const QView& w, const GemvParams& p, const GemvConfig& cfg, cudaStream_t s) {
    using S = Tile<BITS, M, LB>;
    auto kernel = gemv_tma_kernel<BITS, M, LB>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(S::SMEM));
    if (e != cudaSuccess) return e;
    GemvParams q = p;
    const int slices = kWarps * cfg.ck;
    const int per = (p.K + slices - 1) / slices;
    q.slice_rows = (per + kRS - 1) / kRS * kRS;
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((p.R + S::WB - 1) / S::WB, cfg.ck, 1);
    lc.blockDim = dim3(kThreads, 1, 1);
    lc.dynamicSmemBytes = S::SMEM;
    lc.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = cfg.ck;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    lc.attrs = attr;
    lc.numAttrs = 2;
    const CUtensorMap* map = S::BOX == 128 ? w.tmap_w128 : w.tmap_w256;
    return cudaLaunchKernelEx(&lc, kernel, *map, q);
}

// Launch-shape overrides (kt_set_gemv_tuning, or KT_GEMV_LB / KT_GEMV_CK at
// first use); 0 keeps the heuristic's choice.
struct GemvOverrides {
    int lb, ck;
};
// Process-wide, set and read from any host thread.
std::atomic<int>& override_lb() {
    static std::atomic<int> v{env_int("KT_GEMV_LB", 0)};
    return v;
}
std::atomic<int>& override_ck() {
    static std::atomic<int> v{env_int("KT_GEMV_CK", 0)};
    return v;
}
GemvOverrides overrides() {
    return GemvOverrides{override_lb().load(std::memory_order_relaxed), override_ck().load(std::memory_order_relaxed)};
}

// One CTA per SM: pick bytes per lane and the K-cluster so the grid covers as
// many SMs as possible in one wave while every warp keeps >= 32 rows (so the
// per-group epilogue stays small next to the streamed rows); ties go to wider
// lanes (fewer, longer TMA boxes).
GemvConfig choose_config(int R, int K, int max_lb, int sm_count) {
    GemvConfig best{max_lb, 1};
    long best_score = -1;
    for (int lb = max_lb; lb >= 4; lb >>= 1) {
        const int tiles = (R + 32 * lb - 1) / (32 * lb);
        for (int ck = 1; ck <= 8; ++ck) {
            if (ck > 1 && K / (kWarps * ck) < 32) break;
            const long ctas = static_cast<long>(tiles) * ck;
            if (ctas > sm_count && ck > 1) break;
            const long score = std::min<long>(ctas, sm_count) * 100 + lb;
            if (score > best_score) {
                best_score = score;
                best = GemvConfig{lb, ck};
            }
        }
    }
    return best;
}

template <int BITS, int M>
cudaError_t launch_m(const QView& w, const GemvParams& p, int sm_count, cudaStream_t s) {
    // Bytes per lane: the y and T accumulators (2 x M x columns-per-lane floats) must fit in registers.
    constexpr int kMaxLB = M == 1 ? 16 : (M <= 2 ? 8 : 4);
    const GemvOverrides o = overrides();
    GemvConfig cfg = choose_config(p.R, p.K, kMaxLB, sm_count);
    if (o.lb == 4 || o.lb == 8 || o.lb == 16) cfg.lb = std::min(o.lb, kMaxLB);
    if (o.ck >= 1 && o.ck <= 8) cfg.ck = o.ck;
    if constexpr (kMaxLB >= 16) {
        if (cfg.lb == 16) return launch_cfg<BITS, M, 16>(w, p, cfg, s);
    }
    if constexpr (kMaxLB >= 8) {
        if (cfg.lb == 8) return launch_cfg<BITS, M, 8>(w, p, cfg, s);
    }
    return launch_cfg<BITS, M, 4>(w, p, cfg, s);
}

template <int BITS>
cudaError_t launch_bits(const QView& w, const GemvParams& p, int m, int sm_count, cudaStream_t s) {
    switch (m) {
        case 1: return launch_m<BITS, 1>(w, p, sm_count, s);
        case 2: return launch_m<BITS, 2>(w, p, sm_count, s);
        case 3: return launch_m<BITS, 3>(w, p, sm_count, s);
        case 4: return launch_m<BITS, 4>(w, p, sm_count, s);
        case 5: return launch_m<BITS, 5>(w, p, sm_count, s);
        case 6: return launch_m<BITS, 6>(w, p, sm_count, s);
        case 7: return launch_m<BITS, 7>(w, p, sm_count, s);
        case 8: return launch_m<BITS, 8>(w, p, sm_count, s);
        default: return cudaErrorInvalidValue;
    }
}

GemvParams make_params(const QView& w, const MatmulArgs& a) {
    GemvParams p{};
    p.q = w.q;
    p.scales = w.scales;
    p.zeros = w.bits == 4 ? w.zeros : nullptr;
    p.x = a.a;
    p.y = a.c;
    p.bias = a.bias;
    p.err = a.err;
    p.K = w.rows;
    p.N = w.columns;
    p.R = w.bytes_per_row;
    p.gs = w.group_size;
    p.slice_rows = w.rows;
    p.magic = 0x4B000000u;
    p.alpha = a.alpha;
    p.accumulate = a.accumulate;
    p.lora = a.lora;
    return p;
}

}  // namespace

void set_gemv_tuning(int lane_bytes, int cluster_k) {
    override_lb().store(lane_bytes, std::memory_order_relaxed);
    override_ck().store(cluster_k, std::memory_order_relaxed);
}

bool gemv_fast_supported(const QView& w, int32_t m, const float* a) {
    if (m < 1 || m > kGemvMaxM || w.tmap_w128 == nullptr) return false;
    // 16-byte aligned rows, 16-column aligned scale / zero rows, whole stages
    // per group and per K, 16-byte aligned activation rows.
    const bool cols_ok = w.bits == 4 ? w.columns % 32 == 0 : w.columns % 16 == 0;
    return cols_ok && w.group_size % kStageRows == 0 && w.rows % kStageRows == 0 &&
           reinterpret_cast<uintptr_t>(a) % 16 == 0;
}

cudaError_t launch_gemv(const QView& w, const MatmulArgs& args, int sm_count, cudaStream_t s) {
    const GemvParams p = make_params(w, args);
    return w.bits == 4 ? launch_bits<4>(w, p, args.m, sm_count, s) : launch_bits<8>(w, p, args.m, sm_count, s);
}

cudaError_t launch_matmul_generic(const QView& w, const MatmulArgs& args, cudaStream_t s) {
    const GemvParams p = make_params(w, args);
    int m0 = 0;
    while (m0 < args.m) {
        const int mc = std::min(args.m - m0, 65535);
        GemvParams q = p;
        q.x = p.x + static_cast<int64_t>(m0) * p.K;
        q.y = p.y + static_cast<int64_t>(m0) * p.N;
        dim3 grid((p.R + 31) / 32, mc);
        matmul_generic_kernel<<<grid, 256, 0, s>>>(q);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        m0 += mc;
    }
    return cudaSuccess;
}

}  // namespace kt
