/*
 * kt_oracle.c -- CPU restatement of Kotensor's group-wise quantizer and
 * dequantizing matmul.  TEST INFRASTRUCTURE ONLY (the checker for the parity
 * tests, the smoke check and bench.py's CPU-baseline leg); see kt_oracle.h for
 * the reference citations, the JVM float semantics followed here and the
 * parity-pinning status.
 *
 * Build: gcc -O2 -std=c11 -ffp-contract=off -fno-fast-math -fPIC -shared -pthread
 */
#include "kt_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- shapes */

int32_t kto_groups(int32_t rows, int32_t group_size) {
    return (rows + group_size - 1) / group_size; /* QuantizedTensor.kt:47 */
}

int32_t kto_bytes_per_row(int32_t bits, int32_t columns) {
    /* QuantizedTensor.kt:48-49: storedColumns = columns + columns % 2 for INT4 */
    if (bits == 4) return (columns + columns % 2) / 2;
    return columns;
}

int64_t kto_size_in_bytes(int32_t bits, int32_t group_size, int32_t rows, int32_t columns) {
    /* QuantizedTensor.kt:97-98 */
    int64_t groups = kto_groups(rows, group_size);
    return (int64_t)rows * kto_bytes_per_row(bits, columns) + groups * columns * 4 +
           (bits == 4 ? groups * columns : 0);
}

/* ---------------------------------------------------------------- rounding */

/* Float.roundToInt() = Math.round(float) after a NaN check: the closest int,
 * ties toward +infinity, saturating at Int.MIN_VALUE / Int.MAX_VALUE. */
int32_t kto_round(float x, int32_t* out) {
    if (isnan(x)) return KTO_ERR_NAN;
    if (x >= 2147483648.0f) { *out = INT32_MAX; return KTO_OK; }
    if (x <= -2147483648.0f) { *out = INT32_MIN; return KTO_OK; }
    float f = floorf(x);
    /* x - f is exact for every float (|x| < 2^23 shares f's binade or a finer
     * one; |x| >= 2^23 is already an integer), so this is floor(x + 1/2)
     * evaluated without the rounding error of the addition. */
    float r = (x - f >= 0.5f) ? f + 1.0f : f;
    *out = (int32_t)r;
    return KTO_OK;
}

static inline int32_t clamp_i32(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* Kotlin Int addition wraps modulo 2^32. */
static inline int32_t wrap_add(int32_t a, int32_t b) { return (int32_t)((uint32_t)a + (uint32_t)b); }

/* ---------------------------------------------------------------- quantize */

/* QuantizedTensor.kt:280-294 */
static int32_t quantize_symmetric(const float* data, int32_t columns, int32_t row_start, int32_t row_end,
                                  int32_t column, uint8_t* qdata, float* scales, int32_t scale_index) {
    float max_abs = 0.0f;
    for (int32_t r = row_start; r < row_end; ++r) {
        float v = fabsf(data[(int64_t)r * columns + column]);
        if (v > max_abs) max_abs = v;
    }
    float scale = (max_abs > 0.0f) ? max_abs / 127.0f : 1.0f;
    scales[scale_index] = scale;
    float inverse = 1.0f / scale;
    for (int32_t r = row_start; r < row_end; ++r) {
        float prod = data[(int64_t)r * columns + column] * inverse;
        int32_t q;
        if (kto_round(prod, &q) != KTO_OK) return KTO_ERR_NAN;
        q = clamp_i32(q, -127, 127);
        qdata[(int64_t)r * columns + column] = (uint8_t)(int8_t)q;
    }
    return KTO_OK;
}

/* QuantizedTensor.kt:296-324 */
static int32_t quantize_asymmetric(const float* data, int32_t columns, int32_t half, int32_t row_start,
                                   int32_t row_end, int32_t column, uint8_t* qdata, float* scales,
                                   uint8_t* zeros, int32_t scale_index) {
    float mn = 3.40282347e+38f, mx = -3.40282347e+38f;
    for (int32_t r = row_start; r < row_end; ++r) {
        float v = data[(int64_t)r * columns + column];
        if (v < mn) mn = v;
        if (v > mx) mx = v;
    }
    if (mn > 0.0f) mn = 0.0f;
    if (mx < 0.0f) mx = 0.0f;
    float range = mx - mn;
    float scale = (range > 0.0f) ? range / 15.0f : 1.0f;
    int32_t zero;
    if (kto_round(-mn / scale, &zero) != KTO_OK) return KTO_ERR_NAN;
    zero = clamp_i32(zero, 0, 15);
    scales[scale_index] = scale;
    zeros[scale_index] = (uint8_t)zero;
    float inverse = 1.0f / scale;
    for (int32_t r = row_start; r < row_end; ++r) {
        int32_t q;
        if (kto_round(data[(int64_t)r * columns + column] * inverse, &q) != KTO_OK) return KTO_ERR_NAN;
        q = clamp_i32(wrap_add(q, zero), 0, 15);
        int64_t index = (int64_t)r * half + column % half;
        uint8_t existing = qdata[index];
        qdata[index] = (column < half) ? (uint8_t)((existing & 0xF0) | q) : (uint8_t)((existing & 0x0F) | (q << 4));
    }
    return KTO_OK;
}

int32_t kto_quantize(const float* data, int32_t rows, int32_t columns, int32_t bits, int32_t group_size,
                     uint8_t* qdata, float* scales, uint8_t* zeros) {
    if ((bits != 4 && bits != 8) || group_size <= 0 || rows <= 0 || columns <= 0) return KTO_ERR_ARG;
    if (bits == 4 && zeros == NULL) return KTO_ERR_ARG;
    int32_t groups = kto_groups(rows, group_size);
    int32_t half = kto_bytes_per_row(bits, columns);
    for (int32_t group = 0; group < groups; ++group) { /* QuantizedTensor.kt:265-276 */
        int32_t row_start = group * group_size;
        int32_t row_end = row_start + group_size < rows ? row_start + group_size : rows;
        int32_t group_offset = group * columns;
        for (int32_t c = 0; c < columns; ++c) {
            int32_t st = (bits == 8)
                             ? quantize_symmetric(data, columns, row_start, row_end, c, qdata, scales, group_offset + c)
                             : quantize_asymmetric(data, columns, half, row_start, row_end, c, qdata, scales, zeros,
                                                   group_offset + c);
            if (st != KTO_OK) return st;
        }
    }
    return KTO_OK;
}

/* ---------------------------------------------------------------- dequantize */

int32_t kto_raw_value(const uint8_t* qdata, int32_t bits, int32_t columns, int32_t row, int32_t column) {
    /* QuantizedTensor.kt:172-180: INT8 bytes are signed; INT4 is split-half packed. */
    int32_t bpr = kto_bytes_per_row(bits, columns);
    if (bits == 8) return (int32_t)(int8_t)qdata[(int64_t)row * bpr + column];
    int32_t half = bpr;
    int32_t byte = (int32_t)(int8_t)qdata[(int64_t)row * bpr + column % half];
    return column < half ? (byte & 0xF) : ((byte >> 4) & 0xF);
}

float kto_value(const uint8_t* qdata, const float* scales, const uint8_t* zeros, int32_t bits, int32_t group_size,
                int32_t columns, int32_t row, int32_t column) {
    /* QuantizedTensor.kt:182-186 */
    int64_t index = (int64_t)(row / group_size) * columns + column;
    int32_t zero = (bits == 4) ? (int32_t)zeros[index] : 0;
    return scales[index] * (float)(kto_raw_value(qdata, bits, columns, row, column) - zero);
}

void kto_dequantize_row(const uint8_t* qdata, const float* scales, const uint8_t* zeros, int32_t bits,
                        int32_t group_size, int32_t rows, int32_t columns, int32_t row, float* dest) {
    (void)rows;
    /* QuantizedTensor.kt:188-213 */
    int64_t group_offset = (int64_t)(row / group_size) * columns;
    int32_t bpr = kto_bytes_per_row(bits, columns);
    const uint8_t* q = qdata + (int64_t)row * bpr;
    if (bits == 8) {
        for (int32_t c = 0; c < columns; ++c) dest[c] = scales[group_offset + c] * (float)(int8_t)q[c];
    } else {
        int32_t half = bpr;
        for (int32_t c = 0; c < columns; ++c) {
            int32_t byte = (int32_t)(int8_t)q[c % half];
            int32_t raw = c < half ? (byte & 0xF) : ((byte >> 4) & 0xF);
            dest[c] = scales[group_offset + c] * (float)(raw - (int32_t)zeros[group_offset + c]);
        }
    }
}

void kto_dequantize(const uint8_t* qdata, const float* scales, const uint8_t* zeros, int32_t bits,
                    int32_t group_size, int32_t rows, int32_t columns, float* dest) {
    for (int32_t r = 0; r < rows; ++r)
        kto_dequantize_row(qdata, scales, zeros, bits, group_size, rows, columns, r, dest + (int64_t)r * columns);
}

/* ---------------------------------------------------------------- thread pool */

typedef struct {
    atomic_int next;
    int32_t units;
    void (*body)(void* ctx, int32_t unit);
    void* ctx;
} unit_queue;

static void* unit_worker(void* arg) {
    /* MatMul.kt:573-581: workers pull unit indices from a shared counter. */
    unit_queue* q = (unit_queue*)arg;
    for (;;) {
        int32_t unit = atomic_fetch_add(&q->next, 1);
        if (unit >= q->units) return NULL;
        q->body(q->ctx, unit);
    }
}

static void run_units(int32_t units, int32_t threads, void (*body)(void*, int32_t), void* ctx) {
    if (threads <= 1 || units <= 1) {
        for (int32_t u = 0; u < units; ++u) body(ctx, u);
        return;
    }
    if (threads > units) threads = units;
    unit_queue q;
    atomic_init(&q.next, 0);
    q.units = units;
    q.body = body;
    q.ctx = ctx;
    pthread_t* tids = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)threads);
    int32_t started = 0;
    for (int32_t t = 1; t < threads; ++t)
        if (pthread_create(&tids[t], NULL, unit_worker, &q) == 0) ++started;
        else break;
    unit_worker(&q);
    for (int32_t t = 1; t <= started; ++t) pthread_join(tids[t], NULL);
    free(tids);
}

/* ---------------------------------------------------------------- M = 1 */

enum { TILE_M = 32, TILE_N = 256, MAX_ROW_UNITS = 32, TARGET_UNITS = 48, COLUMN_SPLIT_COLUMNS = 8192,
       MIN_BLOCK_BYTES = 128, BLOCK_ALIGN = 64 };
#define UNIT_WORK 65536LL

typedef struct {
    const float* a;
    const uint8_t* qdata;
    const float* scales;
    const uint8_t* zeros;
    int32_t bits, group_size, rows, columns, bytes_per_row;
    float* c;
    float* partials;
    int32_t rows_per_unit, blocks, block_bytes;
    float alpha;
} row_job;

/* MatMul.kt:804-828 */
static void combine_group(const row_job* j, int64_t scale_offset, int32_t count, float row_sum,
                          const float* acc, float* out) {
    float alpha = j->alpha;
    if (j->bits == 4) {
        for (int32_t c = 0; c < count; ++c) {
            float zero = (float)j->zeros[scale_offset + c];
            out[c] += alpha * j->scales[scale_offset + c] * (acc[c] - zero * row_sum);
        }
    } else {
        for (int32_t c = 0; c < count; ++c) out[c] += alpha * j->scales[scale_offset + c] * acc[c];
    }
}

/* MatMul.kt:599-682 (rowUnitInto, scalar unpack path; the lookup path is
 * bit-identical to it, CHANGELOG.md:723). */
static void row_unit(void* ctx, int32_t unit) {
    const row_job* j = (const row_job*)ctx;
    int32_t n = j->columns, row_bytes = j->bytes_per_row, g = j->group_size;
    int32_t row_unit_idx = unit / j->blocks;
    int32_t r0 = row_unit_idx * j->rows_per_unit;
    int32_t r1 = r0 + j->rows_per_unit < j->rows ? r0 + j->rows_per_unit : j->rows;
    int32_t b0 = (unit % j->blocks) * j->block_bytes;
    int32_t b1 = b0 + j->block_bytes < row_bytes ? b0 + j->block_bytes : row_bytes;
    int32_t width = b1 - b0;
    int packed = j->bits == 4;
    int32_t high_columns = 0;
    if (packed) {
        int32_t hi_end = row_bytes + b1 < n ? row_bytes + b1 : n;
        high_columns = hi_end - (row_bytes + b0);
    }
    float* out = j->partials ? j->partials + (int64_t)row_unit_idx * n : j->c;
    float* low = (float*)malloc(sizeof(float) * (size_t)width);
    float* high = (float*)malloc(sizeof(float) * (size_t)width);
    int32_t row = r0;
    while (row < r1) {
        int32_t group = row / g;
        int32_t group_end = (group + 1) * g < r1 ? (group + 1) * g : r1;
        memset(low, 0, sizeof(float) * (size_t)width);
        memset(high, 0, sizeof(float) * (size_t)width);
        float row_sum = 0.0f;
        for (int32_t l = row; l < group_end; ++l) {
            float al = j->a[l];
            row_sum += al;
            const uint8_t* q = j->qdata + (int64_t)l * row_bytes + b0;
            if (packed) {
                for (int32_t c = 0; c < width; ++c) {
                    low[c] += al * (float)(q[c] & 0xF);
                    high[c] += al * (float)((q[c] >> 4) & 0xF);
                }
            } else {
                for (int32_t c = 0; c < width; ++c) low[c] += al * (float)(int8_t)q[c];
            }
        }
        combine_group(j, (int64_t)group * n + b0, width, row_sum, low, out + b0);
        if (high_columns > 0)
            combine_group(j, (int64_t)group * n + row_bytes + b0, high_columns, row_sum, high, out + row_bytes + b0);
        row = group_end;
    }
    free(low);
    free(high);
}

/* MatMul.kt:494-536 */
static void multiply_row(row_job* j, int32_t accumulate, int32_t threads) {
    int32_t k = j->rows, n = j->columns, row_bytes = j->bytes_per_row;
    int32_t groups = kto_groups(k, j->group_size);
    int64_t tu = (int64_t)k * n / UNIT_WORK;
    int32_t target_units = (int32_t)tu;
    if (tu > INT32_MAX) target_units = INT32_MAX;
    target_units = clamp_i32(target_units, 1, TARGET_UNITS);
    int32_t rows_per_unit, wanted_column_units;
    if (n >= COLUMN_SPLIT_COLUMNS) {
        rows_per_unit = k;
        wanted_column_units = target_units;
    } else {
        int32_t groups_per_unit = (groups + MAX_ROW_UNITS - 1) / MAX_ROW_UNITS;
        rows_per_unit = groups_per_unit * j->group_size < k ? groups_per_unit * j->group_size : k;
        wanted_column_units = (target_units * rows_per_unit + k - 1) / k;
    }
    int32_t row_units = (k + rows_per_unit - 1) / rows_per_unit;
    int32_t max_cu = row_bytes / MIN_BLOCK_BYTES > 1 ? row_bytes / MIN_BLOCK_BYTES : 1;
    int32_t column_units = clamp_i32(wanted_column_units, 1, max_cu);
    int32_t bb = ((row_bytes + column_units - 1) / column_units + BLOCK_ALIGN - 1) / BLOCK_ALIGN * BLOCK_ALIGN;
    int32_t block_bytes = row_bytes < bb ? row_bytes : bb;
    int32_t blocks = (row_bytes + block_bytes - 1) / block_bytes;
    float* partials = NULL;
    if (row_units > 1) partials = (float*)calloc((size_t)row_units * (size_t)n, sizeof(float));
    if (!accumulate) memset(j->c, 0, sizeof(float) * (size_t)n);
    j->partials = partials;
    j->rows_per_unit = rows_per_unit;
    j->blocks = blocks;
    j->block_bytes = block_bytes;
    run_units(row_units * blocks, threads, row_unit, j);
    if (partials) {
        for (int32_t u = 0; u < row_units; ++u)
            for (int32_t c = 0; c < n; ++c) j->c[c] += partials[(int64_t)u * n + c];
        free(partials);
    }
}

/* ---------------------------------------------------------------- M > 1 */

typedef struct {
    const float* a;
    const uint8_t* qdata;
    const float* scales;
    const uint8_t* zeros;
    int32_t bits, group_size, rows, columns, bytes_per_row;
    float* c;
    int32_t m, accumulate, tiles_n, width;
    float alpha;
} tile_job;

/* MatMul.kt:883-905 */
static void unpack_row(const tile_job* j, int32_t row, int32_t j0, int32_t len, float* out) {
    const uint8_t* q = j->qdata + (int64_t)row * j->bytes_per_row;
    if (j->bits == 8) {
        for (int32_t c = 0; c < len; ++c) out[c] = (float)(int8_t)q[j0 + c];
        return;
    }
    int32_t half = j->bytes_per_row;
    for (int32_t c = 0; c < len; ++c) {
        int32_t col = j0 + c;
        out[c] = col < half ? (float)(q[col] & 0xF) : (float)((q[col - half] >> 4) & 0xF);
    }
}

/* MatMul.kt:830-881 (scalar axpy4/axpy: y += a * x, one rounding per operation) */
static void quantized_tile(void* ctx, int32_t tile) {
    const tile_job* j = (const tile_job*)ctx;
    int32_t k = j->rows, n = j->columns;
    int32_t i0 = (tile / j->tiles_n) * TILE_M;
    int32_t j0 = (tile % j->tiles_n) * j->width;
    int32_t rows = j->m - i0 < TILE_M ? j->m - i0 : TILE_M;
    int32_t len = n - j0 < j->width ? n - j0 : j->width;
    float* ct = (float*)malloc(sizeof(float) * TILE_M * TILE_N);
    float* acc = (float*)malloc(sizeof(float) * TILE_M * TILE_N);
    float row_sums[TILE_M];
    float brow[TILE_N];
    for (int32_t r = 0; r < rows; ++r)
        for (int32_t c = 0; c < len; ++c)
            ct[r * TILE_N + c] = j->accumulate ? j->c[(int64_t)(i0 + r) * n + j0 + c] : 0.0f;
    int32_t groups = kto_groups(k, j->group_size);
    for (int32_t group = 0; group < groups; ++group) {
        int32_t k0 = group * j->group_size;
        int32_t k1 = k0 + j->group_size < k ? k0 + j->group_size : k;
        for (int32_t r = 0; r < rows; ++r) {
            memset(acc + r * TILE_N, 0, sizeof(float) * (size_t)len);
            row_sums[r] = 0.0f;
        }
        for (int32_t l = k0; l < k1; ++l) {
            unpack_row(j, l, j0, len, brow);
            for (int32_t r = 0; r < rows; ++r) {
                float ar = 1.0f * j->a[(int64_t)(i0 + r) * k + l];
                float* y = acc + r * TILE_N;
                for (int32_t c = 0; c < len; ++c) y[c] += ar * brow[c];
            }
            for (int32_t r = 0; r < rows; ++r) row_sums[r] += j->a[(int64_t)(i0 + r) * k + l];
        }
        int64_t go = (int64_t)group * n + j0;
        for (int32_t r = 0; r < rows; ++r) {
            float* y = ct + r * TILE_N;
            const float* av = acc + r * TILE_N;
            if (j->bits == 4) {
                for (int32_t c = 0; c < len; ++c)
                    y[c] += j->alpha * j->scales[go + c] * (av[c] - (float)j->zeros[go + c] * row_sums[r]);
            } else {
                for (int32_t c = 0; c < len; ++c) y[c] += j->alpha * j->scales[go + c] * av[c];
            }
        }
    }
    for (int32_t r = 0; r < rows; ++r)
        for (int32_t c = 0; c < len; ++c) j->c[(int64_t)(i0 + r) * n + j0 + c] = ct[r * TILE_N + c];
    free(ct);
    free(acc);
}

static int32_t quantized_tile_width(int32_t n) { /* MatMul.kt:488-492 */
    if (n >= TARGET_UNITS * TILE_N) return TILE_N;
    int32_t wanted = (n + TARGET_UNITS - 1) / TARGET_UNITS;
    return clamp_i32((wanted + BLOCK_ALIGN - 1) / BLOCK_ALIGN * BLOCK_ALIGN, BLOCK_ALIGN, TILE_N);
}

int32_t kto_multiply_quantized(const float* a, const uint8_t* qdata, const float* scales, const uint8_t* zeros,
                               int32_t bits, int32_t group_size, int32_t rows, int32_t columns, float* c, int32_t m,
                               int32_t accumulate, float alpha, int32_t threads) {
    /* MatMul.kt:460-486 */
    if (m < 0 || (bits != 4 && bits != 8) || group_size <= 0 || rows <= 0 || columns <= 0) return KTO_ERR_ARG;
    if (m == 0) return KTO_OK;
    if (m == 1) {
        row_job j = {a, qdata, scales, zeros, bits, group_size, rows, columns, kto_bytes_per_row(bits, columns),
                     c, NULL, 0, 0, 0, alpha};
        multiply_row(&j, accumulate, threads);
        return KTO_OK;
    }
    int32_t width = quantized_tile_width(columns);
    int32_t tiles_n = (columns + width - 1) / width;
    int32_t tiles = ((m + TILE_M - 1) / TILE_M) * tiles_n;
    tile_job j = {a, qdata, scales, zeros, bits, group_size, rows, columns, kto_bytes_per_row(bits, columns),
                  c, m, accumulate, tiles_n, width, alpha};
    run_units(tiles, threads, quantized_tile, &j);
    return KTO_OK;
}

/* ---------------------------------------------------------------- backward */

typedef struct {
    const float* dy;
    const uint8_t* qdata;
    const float* scales;
    const uint8_t* zeros;
    int32_t bits, group_size, rows, columns;
    float* dx;
    int32_t m;
} back_job;

/* MatMul.kt:983-1003 (scalar dot: four strided partial sums, then the tail) */
static float dot4(const float* a, const float* b, int32_t len) {
    float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
    int32_t j = 0;
    for (; j + 4 <= len; j += 4) {
        s0 += a[j] * b[j];
        s1 += a[j + 1] * b[j + 1];
        s2 += a[j + 2] * b[j + 2];
        s3 += a[j + 3] * b[j + 3];
    }
    float sum = (s0 + s1) + (s2 + s3);
    for (; j < len; ++j) sum += a[j] * b[j];
    return sum;
}

/* MatMul.kt:969-980 */
static void back_tile(void* ctx, int32_t tile) {
    const back_job* j = (const back_job*)ctx;
    int32_t k = j->rows, n = j->columns;
    float* wrow = (float*)malloc(sizeof(float) * (size_t)n);
    int32_t k0 = tile * TILE_M;
    int32_t k1 = k0 + TILE_M < k ? k0 + TILE_M : k;
    for (int32_t l = k0; l < k1; ++l) {
        kto_dequantize_row(j->qdata, j->scales, j->zeros, j->bits, j->group_size, k, n, l, wrow);
        for (int32_t i = 0; i < j->m; ++i) j->dx[(int64_t)i * k + l] += dot4(j->dy + (int64_t)i * n, wrow, n);
    }
    free(wrow);
}

int32_t kto_multiply_by_quantized_transposed(const float* dy, const uint8_t* qdata, const float* scales,
                                             const uint8_t* zeros, int32_t bits, int32_t group_size, int32_t rows,
                                             int32_t columns, float* dx, int32_t m, int32_t accumulate,
                                             int32_t threads) {
    /* MatMul.kt:954-981 */
    if (m < 0 || (bits != 4 && bits != 8) || group_size <= 0 || rows <= 0 || columns <= 0) return KTO_ERR_ARG;
    if (m == 0) return KTO_OK;
    if (!accumulate) memset(dx, 0, sizeof(float) * (size_t)m * (size_t)rows);
    back_job j = {dy, qdata, scales, zeros, bits, group_size, rows, columns, dx, m};
    run_units((rows + TILE_M - 1) / TILE_M, threads, back_tile, &j);
    return KTO_OK;
}

/* ---------------------------------------------------------------- float64 */

void kto_multiply_dequantized_f64(const float* a, const uint8_t* qdata, const float* scales, const uint8_t* zeros,
                                  int32_t bits, int32_t group_size, int32_t rows, int32_t columns, double* c,
                                  int32_t m) {
    float* wrow = (float*)malloc(sizeof(float) * (size_t)columns);
    memset(c, 0, sizeof(double) * (size_t)m * (size_t)columns);
    for (int32_t l = 0; l < rows; ++l) {
        kto_dequantize_row(qdata, scales, zeros, bits, group_size, rows, columns, l, wrow);
        for (int32_t i = 0; i < m; ++i) {
            double ai = (double)a[(int64_t)i * rows + l];
            double* ci = c + (int64_t)i * columns;
            for (int32_t col = 0; col < columns; ++col) ci[col] += ai * (double)wrow[col];
        }
    }
    free(wrow);
}
