// kt_gemv.cu -- fp32-accumulate dequantizing matmul for small m (the decode
// GEMV), MatMul.multiplyQuantized for m <= kGemvMaxM
// (Engine/kotensor/src/main/kotlin/MatMul.kt:460-536 and :599-828).
//
// The reference factors each group g and output column j as
//   c[j] += alpha * scale[g,j] * (sum_l a_l * q[l,j]  -  zero[g,j] * sum_l a_l)
// with q the raw unsigned nibble (INT4) or the signed byte (INT8)
// (combineGroup, MatMul.kt:804-828).  This kernel keeps that factoring: each
// lane owns LB contiguous packed bytes of a row (INT4: 2*LB columns, the low
// nibbles for columns cb.. and the high nibbles for columns half+cb..; INT8: LB
// columns), walks whole groups of rows, and applies scale and zero once per
// group.
//
// Unpacking without int->float conversions.  A nibble or byte q placed in the
// top mantissa bits of the float 2^23 (bits 0x4B000000) gives the exact float
// 2^23 + q*2^p with one LOP3; fp32 FMAs accumulate T = sum_l a_l*(2^23 + q*2^p)
// and the group epilogue recovers sum_l a_l*q = T*2^-p - 2^(23-p)*sum_l a_l.
//   INT4 low nibbles sit at bits 16-19 (p = 16), high nibbles at bits 12-15
//   (p = 12): 3 shift/permute ops + 8 LOP3 + 8 FFMA per 32-bit word of 8 weights.
//   INT8 bytes are offset to unsigned (xor 0x80) and sit at bits 15-22 (p = 15).
// The leading 2^23 term costs at most ~11 bits of the fp32 accumulator, a
// relative error below 1e-4 of max|c| (the tolerance is 1e-3).
//
// Split-K and the reduction order.  Partial sums over disjoint group ranges
// ("slices") are reduced in a fixed order: across the KL lanes of a warp that
// share a column chunk (xor-shuffle butterfly, commutative at every level), across
// the NW warps of a CTA (shared memory, warp order), and across the CK CTAs of a
// thread-block cluster along K (distributed shared memory, rank order).  No
// atomics and no global scratch: the same inputs give the same bits every run.
#include <cooperative_groups.h>

#include <algorithm>
#include <cstdlib>

#include "kt_internal.h"

namespace cg = cooperative_groups;

namespace kt {
namespace {

constexpr uint32_t kMagic = 0x4B000000u;  // the float 2^23

struct GemvParams {
    const uint8_t* q;
    const float* scales;
    const uint8_t* zeros;
    const float* x;
    float* y;
    const float* bias;
    int32_t K, N, R, G, gs;
    int32_t KL;  // lanes along K inside a warp (1, 2 or 4)
    float alpha;
    int32_t accumulate;
};

// Streaming loads of packed weights: read once, so skip L1 allocation.
__device__ __forceinline__ void ld_stream(const uint8_t* p, uint32_t (&w)[4]) {
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
        : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]) : "l"(p));
}
__device__ __forceinline__ void ld_stream(const uint8_t* p, uint32_t (&w)[2]) {
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(w[0]), "=r"(w[1]) : "l"(p));
}
__device__ __forceinline__ void ld_stream(const uint8_t* p, uint32_t (&w)[1]) {
    asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(w[0]) : "l"(p));
}

__device__ __forceinline__ float bits_f(uint32_t u) { return __uint_as_float(u); }

// One 32-bit word of 4 packed INT4 bytes: low nibbles -> columns lo+0..3,
// high nibbles -> columns hi+0..3 (indices into the lane's T array).
template <int M, int C>
__device__ __forceinline__ void fma_int4_word(uint32_t w, const float (&xv)[M], float (&T)[M][C], int lo, int hi) {
    const uint32_t wl = w << 8, wr = w >> 8;
    const uint32_t t = __byte_perm(w, 0u, 0x4034);  // byte0 -> bits 16-23, byte3 -> bits 8-15
    const float f_lo0 = bits_f((t & 0x000F0000u) | kMagic);
    const float f_hi3 = bits_f((t & 0x0000F000u) | kMagic);
    const float f_lo1 = bits_f((wl & 0x000F0000u) | kMagic);
    const float f_hi0 = bits_f((wl & 0x0000F000u) | kMagic);
    const float f_lo2 = bits_f((w & 0x000F0000u) | kMagic);
    const float f_hi1 = bits_f((w & 0x0000F000u) | kMagic);
    const float f_lo3 = bits_f((wr & 0x000F0000u) | kMagic);
    const float f_hi2 = bits_f((wr & 0x0000F000u) | kMagic);
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
__device__ __forceinline__ void fma_int8_word(uint32_t w, const float (&xv)[M], float (&T)[M][C], int at) {
    const uint32_t u = w ^ 0x80808080u;  // two's complement byte b -> unsigned b + 128
    const float f0 = bits_f(((u << 15) & 0x007F8000u) | kMagic);
    const float f1 = bits_f(((u << 7) & 0x007F8000u) | kMagic);
    const float f2 = bits_f(((u >> 1) & 0x007F8000u) | kMagic);
    const float f3 = bits_f(((u >> 9) & 0x007F8000u) | kMagic);
#pragma unroll
    for (int m = 0; m < M; ++m) {
        T[m][at + 0] = fmaf(xv[m], f0, T[m][at + 0]);
        T[m][at + 1] = fmaf(xv[m], f1, T[m][at + 1]);
        T[m][at + 2] = fmaf(xv[m], f2, T[m][at + 2]);
        T[m][at + 3] = fmaf(xv[m], f3, T[m][at + 3]);
    }
}

template <int BITS, int M, int LB>
struct Shape {
    static constexpr int C = BITS == 4 ? 2 * LB : LB;  // columns per lane
    static constexpr int WORDS = LB / 4;
    // rows per load batch: loads in flight per lane, bounded by registers
    static constexpr int U = LB == 16 ? 8 : (M <= 2 ? 16 : (M <= 4 ? 8 : 4));
};

// Dynamic shared memory: red[NW][M][CT] then part[M][CT], CT = columns per CTA tile.
template <int BITS, int M, int LB>
__global__ void __launch_bounds__(256) gemv_kernel(GemvParams p) {
    using S = Shape<BITS, M, LB>;
    constexpr int C = S::C;
    constexpr int U = S::U;
    extern __shared__ float smem[];

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int NW = blockDim.x >> 5;
    const int KL = p.KL;
    const int LC = 32 / KL;
    const int WB = LC * LB;                     // packed bytes per CTA tile
    const int CT = BITS == 4 ? 2 * WB : WB;     // columns per CTA tile
    const int lc = lane % LC, kl = lane / LC;
    const int tile_b0 = blockIdx.x * WB;
    const int cb = tile_b0 + lc * LB;           // this lane's first packed byte
    const bool active = cb < p.R;
    const int half = p.R;                       // INT4: high-nibble columns start here

    const int CK = gridDim.y;
    const int slices = CK * NW * KL;
    const int slice = (blockIdx.y * NW + warp) * KL + kl;
    const int g0 = static_cast<int>(static_cast<int64_t>(slice) * p.G / slices);
    const int g1 = static_cast<int>(static_cast<int64_t>(slice + 1) * p.G / slices);

    float y[M][C];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int j = 0; j < C; ++j) y[m][j] = 0.0f;

    for (int g = g0; g < g1; ++g) {
        const int r0 = g * p.gs;
        const int r1 = min(r0 + p.gs, p.K);
        float T[M][C];
        float rs[M];
#pragma unroll
        for (int m = 0; m < M; ++m) {
            rs[m] = 0.0f;
#pragma unroll
            for (int j = 0; j < C; ++j) T[m][j] = 0.0f;
        }
        for (int r = r0; r < r1; r += U) {
            uint32_t wv[U][S::WORDS];
            float xv[U][M];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int rr = r + u;
                if (active && rr < r1) {
                    ld_stream(p.q + static_cast<int64_t>(rr) * p.R + cb, wv[u]);
                } else {
#pragma unroll
                    for (int k = 0; k < S::WORDS; ++k) wv[u][k] = 0u;
                }
#pragma unroll
                for (int m = 0; m < M; ++m) xv[u][m] = rr < r1 ? __ldg(p.x + static_cast<int64_t>(m) * p.K + rr) : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
#pragma unroll
                for (int m = 0; m < M; ++m) rs[m] += xv[u][m];
#pragma unroll
                for (int k = 0; k < S::WORDS; ++k) {
                    if constexpr (BITS == 4) {
                        fma_int4_word<M, C>(wv[u][k], xv[u], T, 4 * k, LB + 4 * k);
                    } else {
                        fma_int8_word<M, C>(wv[u][k], xv[u], T, 4 * k);
                    }
                }
            }
        }
        if (active) {
            // Group epilogue: y += scale * (T * 2^-p - (offset + zero) * rowSum).
            const int64_t go = static_cast<int64_t>(g) * p.N;
            if constexpr (BITS == 4) {
                const float* s_lo = p.scales + go + cb;
                const float* s_hi = p.scales + go + half + cb;
                const uint8_t* z_lo = p.zeros + go + cb;
                const uint8_t* z_hi = p.zeros + go + half + cb;
#pragma unroll
                for (int i = 0; i < LB; ++i) {
                    const float sl = __ldg(s_lo + i), sh = __ldg(s_hi + i);
                    const float zl = 128.0f + static_cast<float>(__ldg(z_lo + i));
                    const float zh = 2048.0f + static_cast<float>(__ldg(z_hi + i));
#pragma unroll
                    for (int m = 0; m < M; ++m) {
                        y[m][i] = fmaf(sl, fmaf(T[m][i], 0x1p-16f, -zl * rs[m]), y[m][i]);
                        y[m][LB + i] = fmaf(sh, fmaf(T[m][LB + i], 0x1p-12f, -zh * rs[m]), y[m][LB + i]);
                    }
                }
            } else {
                const float* sc = p.scales + go + cb;
#pragma unroll
                for (int i = 0; i < LB; ++i) {
                    const float s = __ldg(sc + i);
#pragma unroll
                    for (int m = 0; m < M; ++m) y[m][i] = fmaf(s, fmaf(T[m][i], 0x1p-15f, -384.0f * rs[m]), y[m][i]);
                }
            }
        }
    }

    // (1) lanes of a warp that share a column chunk (butterfly over the kl bits).
    for (int off = LC; off < 32; off <<= 1) {
#pragma unroll
        for (int m = 0; m < M; ++m)
#pragma unroll
            for (int j = 0; j < C; ++j) y[m][j] += __shfl_xor_sync(0xffffffffu, y[m][j], off);
    }
    // (2) warps of the CTA, in warp order.
    float* red = smem;                             // [NW][M][CT]
    float* part = smem + static_cast<size_t>(NW) * M * CT;  // [M][CT]
    if (kl == 0) {
#pragma unroll
        for (int m = 0; m < M; ++m) {
            float* dst = red + (static_cast<size_t>(warp) * M + m) * CT;
#pragma unroll
            for (int i = 0; i < LB; ++i) {
                dst[lc * LB + i] = y[m][i];
                if constexpr (BITS == 4) dst[WB + lc * LB + i] = y[m][LB + i];
            }
        }
    }
    __syncthreads();
    for (int t = threadIdx.x; t < M * CT; t += blockDim.x) {
        float v = red[t];
        for (int w = 1; w < NW; ++w) v += red[static_cast<size_t>(w) * M * CT + t];
        part[t] = v;
    }
    // (3) CTAs of the cluster along K, in rank order; CTA rank r finishes
    // columns [r*CT/CK, (r+1)*CT/CK) of every row m.
    cg::cluster_group cluster = cg::this_cluster();
    if (CK > 1) cluster.sync(); else __syncthreads();
    const int rank = CK > 1 ? static_cast<int>(cluster.block_rank()) : 0;
    const int j0 = rank * CT / CK, j1 = (rank + 1) * CT / CK;
    const int span = j1 - j0;
    for (int t = threadIdx.x; t < M * span; t += blockDim.x) {
        const int m = t / span;
        const int j = j0 + t % span;
        float v = part[m * CT + j];
        if (CK > 1) {
            v = 0.0f;
            for (int q = 0; q < CK; ++q) v += cluster.map_shared_rank(part, q)[m * CT + j];
        }
        int col, byte;
        if constexpr (BITS == 4) {
            byte = tile_b0 + (j < WB ? j : j - WB);
            col = j < WB ? byte : half + byte;
        } else {
            byte = tile_b0 + j;
            col = byte;
        }
        if (byte < p.R && col < p.N) {
            float* out = p.y + static_cast<int64_t>(m) * p.N + col;
            float r = fmaf(p.alpha, v, p.accumulate ? *out : 0.0f);
            if (p.bias != nullptr) r += p.bias[col];
            *out = r;
        }
    }
    if (CK > 1) cluster.sync();  // keep this CTA's shared memory alive until every rank has read it
}

// ---------------------------------------------------------------- generic fallback
// Any shape (odd N, unaligned rows) and any m: one thread per packed byte
// column and output row, 8 warps split the groups, fixed-order smem reduction.
// Plain int->float conversion; used only where the streaming kernel's
// alignment rules do not hold.
__global__ void __launch_bounds__(256) matmul_generic_kernel(GemvParams p) {
    __shared__ float red[8][2][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int b = blockIdx.x * 32 + lane;  // packed byte column
    const int m = blockIdx.y;
    const bool is4 = p.zeros != nullptr;
    const int half = p.R;
    const bool active = b < p.R;
    const bool has_hi = is4 && active && b + half < p.N;
    float y_lo = 0.0f, y_hi = 0.0f;
    const float* xr = p.x + static_cast<int64_t>(m) * p.K;
    for (int g = warp; g < p.G; g += 8) {
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
            *out = r;
        }
    }
}

// ---------------------------------------------------------------- dispatch

struct GemvConfig {
    int lb, kl, nw, ck;
};

int env_int(const char* name, int fallback) {
    const char* v = std::getenv(name);
    return v ? std::atoi(v) : fallback;
}

template <int BITS, int M, int LB>
cudaError_t launch_cfg(const GemvParams& p, const GemvConfig& cfg, cudaStream_t s) {
    const int LC = 32 / cfg.kl;
    const int WB = LC * LB;
    const int CT = BITS == 4 ? 2 * WB : WB;
    const size_t smem = (static_cast<size_t>(cfg.nw) * M * CT + static_cast<size_t>(M) * CT) * sizeof(float);
    auto kernel = gemv_kernel<BITS, M, LB>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem));
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3((p.R + WB - 1) / WB, cfg.ck, 1);
    lc.blockDim = dim3(cfg.nw * 32, 1, 1);
    lc.dynamicSmemBytes = smem;
    lc.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = cfg.ck;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    GemvParams q = p;
    q.KL = cfg.kl;
    return cudaLaunchKernelEx(&lc, kernel, q);
}

// Picks lanes-along-K, warps and cluster size so that the grid covers the SMs
// with at least one group per slice.
GemvConfig choose_config(int R, int G, int lb, int sm_count) {
    GemvConfig best{lb, 1, 8, 1};
    int best_ctas = -1;
    for (int kl = 1; kl <= 4; kl <<= 1) {
        const int WB = (32 / kl) * lb;
        const int tiles = (R + WB - 1) / WB;
        for (int ck = 1; ck <= 8; ++ck) {
            const int slices = kl * 8 * ck;
            if (slices > G && ck > 1) break;
            const int ctas = tiles * ck;
            // prefer the smallest grid that reaches 2 CTAs per SM, else the largest grid
            const bool enough = ctas >= 2 * sm_count;
            const bool best_enough = best_ctas >= 2 * sm_count;
            if (best_ctas < 0 || (!best_enough && ctas > best_ctas) || (enough && best_enough && ctas < best_ctas)) {
                best = GemvConfig{lb, kl, 8, ck};
                best_ctas = ctas;
            }
        }
    }
    return best;
}

// Tuning overrides for sweeps (KT_GEMV_LB / KT_GEMV_KL / KT_GEMV_NW / KT_GEMV_CK),
// read once; 0 keeps the heuristic's choice.
struct GemvOverrides {
    int lb, kl, nw, ck;
};
const GemvOverrides& overrides() {
    static const GemvOverrides o{env_int("KT_GEMV_LB", 0), env_int("KT_GEMV_KL", 0), env_int("KT_GEMV_NW", 0),
                                 env_int("KT_GEMV_CK", 0)};
    return o;
}

template <int BITS, int M>
cudaError_t launch_m(const GemvParams& p, int sm_count, cudaStream_t s) {
    // Bytes per lane: the accumulators (2 x M x columns-per-lane floats) must fit in registers.
    constexpr int kDefaultLB = M == 1 ? 16 : (M == 2 ? 8 : 4);
    const GemvOverrides& o = overrides();
    int lb = kDefaultLB;
    if (o.lb == 4 || o.lb == 8 || o.lb == 16) lb = std::min(o.lb, kDefaultLB);
    GemvConfig cfg = choose_config(p.R, p.G, lb, sm_count);
    if (o.kl == 1 || o.kl == 2 || o.kl == 4) cfg.kl = o.kl;
    if (o.nw >= 1 && o.nw <= 8) cfg.nw = o.nw;
    if (o.ck >= 1 && o.ck <= 8) cfg.ck = o.ck;
    if constexpr (kDefaultLB == 16) {
        if (lb == 16) return launch_cfg<BITS, M, 16>(p, cfg, s);
    }
    if constexpr (kDefaultLB >= 8) {
        if (lb == 8) return launch_cfg<BITS, M, 8>(p, cfg, s);
    }
    return launch_cfg<BITS, M, 4>(p, cfg, s);
}

template <int BITS>
cudaError_t launch_bits(const GemvParams& p, int m, int sm_count, cudaStream_t s) {
    switch (m) {
        case 1: return launch_m<BITS, 1>(p, sm_count, s);
        case 2: return launch_m<BITS, 2>(p, sm_count, s);
        case 3: return launch_m<BITS, 3>(p, sm_count, s);
        case 4: return launch_m<BITS, 4>(p, sm_count, s);
        case 5: return launch_m<BITS, 5>(p, sm_count, s);
        case 6: return launch_m<BITS, 6>(p, sm_count, s);
        case 7: return launch_m<BITS, 7>(p, sm_count, s);
        case 8: return launch_m<BITS, 8>(p, sm_count, s);
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
    p.K = w.rows;
    p.N = w.columns;
    p.R = w.bytes_per_row;
    p.G = w.groups;
    p.gs = w.group_size;
    p.KL = 1;
    p.alpha = a.alpha;
    p.accumulate = a.accumulate;
    return p;
}

}  // namespace

bool gemv_fast_supported(const QView& w, int32_t m) {
    if (m < 1 || m > kGemvMaxM) return false;
    // 16-byte aligned rows and 16-column aligned scale / zero rows.
    if (w.bits == 4) return w.columns % 32 == 0;
    return w.columns % 16 == 0;
}

cudaError_t launch_gemv(const QView& w, const MatmulArgs& args, int sm_count, cudaStream_t s) {
    const GemvParams p = make_params(w, args);
    return w.bits == 4 ? launch_bits<4>(p, args.m, sm_count, s) : launch_bits<8>(p, args.m, sm_count, s);
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
