/*
 * kt_oracle.h -- CPU restatement of Kotensor's group-wise quantizer and
 * dequantizing matmul.  TEST INFRASTRUCTURE ONLY: the parity tests, the
 * smoke check and bench.py's CPU-baseline leg call it as the checker.  No
 * product code path links, loads or calls it.
 *
 * Reference (paths inside the Kotensor project, Engine/kotensor/):
 *   src/main/kotlin/QuantizedTensor.kt:10-25    Quantization(bits, groupSize)
 *   src/main/kotlin/QuantizedTensor.kt:45-49    groups / storedColumns / bytesPerRow
 *   src/main/kotlin/QuantizedTensor.kt:172-249  rawValue / value / dequantizeRow / dequantize
 *   src/main/kotlin/QuantizedTensor.kt:261-324  quantize, quantizeSymmetric, quantizeAsymmetric
 *   src/main/kotlin/MatMul.kt:460-536           multiplyQuantized, multiplyQuantizedRow (unit schedule)
 *   src/main/kotlin/MatMul.kt:599-828           rowUnitInto, unpack*, combineGroup
 *   src/main/kotlin/MatMul.kt:830-952           computeQuantizedTile (M > 1)
 *   src/main/kotlin/MatMul.kt:954-1003          multiplyByQuantizedTransposed, dot
 *
 * Parity status: the reference is Kotlin and no JVM exists on this machine or
 * on the GPU box, so no reference output can be produced here, and the
 * reference ships no golden vectors for quantized results.  This oracle is
 * pinned to every known-answer test the reference's own suite holds for the
 * path (QuantizationTest.kt:38-134, DecodeKernelTest.kt:48-110: shape
 * bookkeeping, sizeInBytes, error bounds, exact zeros, bit-identity across
 * schedules and thread counts, accumulate/alpha); beyond those properties the
 * quantizer and matmul outputs are "parity unpinned" against the reference.
 *
 * Floating-point semantics follow the JVM: every float operation rounds to
 * IEEE binary32, no operation is contracted into an FMA (build with
 * -ffp-contract=off, never -ffast-math), Float.roundToInt() is Math.round
 * (nearest, ties toward +infinity, saturating to the int range) and throws on
 * NaN -- reported here as KTO_ERR_NAN.
 */
#ifndef KT_ORACLE_H
#define KT_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { KTO_OK = 0, KTO_ERR_ARG = 1, KTO_ERR_NAN = 2 };

/* Shape bookkeeping, QuantizedTensor.kt:45-49 and :97-98. */
int32_t kto_groups(int32_t rows, int32_t group_size);
int32_t kto_bytes_per_row(int32_t bits, int32_t columns);
int64_t kto_size_in_bytes(int32_t bits, int32_t group_size, int32_t rows, int32_t columns);

/* Java Math.round(float) with Kotlin's NaN check; returns KTO_ERR_NAN on NaN. */
int32_t kto_round(float x, int32_t* out);

/* QuantizedTensor.quantize(data, rows, columns, Quantization(bits, group)).
 * qdata: rows*bytesPerRow bytes (zero-initialised by the caller),
 * scales: groups*columns floats, zeros: groups*columns bytes (INT4 only, may be
 * NULL for INT8).  Returns KTO_ERR_NAN where Kotlin would throw. */
int32_t kto_quantize(const float* data, int32_t rows, int32_t columns, int32_t bits,
                     int32_t group_size, uint8_t* qdata, float* scales, uint8_t* zeros);

/* QuantizedTensor.rawValue / value / dequantizeRow / dequantize. */
int32_t kto_raw_value(const uint8_t* qdata, int32_t bits, int32_t columns, int32_t row, int32_t column);
float kto_value(const uint8_t* qdata, const float* scales, const uint8_t* zeros, int32_t bits,
                int32_t group_size, int32_t columns, int32_t row, int32_t column);
void kto_dequantize_row(const uint8_t* qdata, const float* scales, const uint8_t* zeros, int32_t bits,
                        int32_t group_size, int32_t rows, int32_t columns, int32_t row, float* dest);
void kto_dequantize(const uint8_t* qdata, const float* scales, const uint8_t* zeros, int32_t bits,
                    int32_t group_size, int32_t rows, int32_t columns, float* dest);

/* MatMul.multiplyQuantized(a, W, c, m, accumulate, alpha): scalar (non-Vector-API)
 * reference arithmetic, including the M=1 work-unit schedule and its fixed-order
 * partial reduction, run on `threads` POSIX threads (results are bit-identical
 * for every thread count, as in the reference). */
int32_t kto_multiply_quantized(const float* a, const uint8_t* qdata, const float* scales,
                               const uint8_t* zeros, int32_t bits, int32_t group_size,
                               int32_t rows, int32_t columns, float* c, int32_t m,
                               int32_t accumulate, float alpha, int32_t threads);

/* MatMul.multiplyByQuantizedTransposed(dy, W, dx, m, accumulate): scalar dot. */
int32_t kto_multiply_by_quantized_transposed(const float* dy, const uint8_t* qdata, const float* scales,
                                             const uint8_t* zeros, int32_t bits, int32_t group_size,
                                             int32_t rows, int32_t columns, float* dx, int32_t m,
                                             int32_t accumulate, int32_t threads);

/* float64 product of a with the dequantized weight (no reference counterpart:
 * the exact value the tolerance checks measure against). */
void kto_multiply_dequantized_f64(const float* a, const uint8_t* qdata, const float* scales,
                                  const uint8_t* zeros, int32_t bits, int32_t group_size,
                                  int32_t rows, int32_t columns, double* c, int32_t m);

#ifdef __cplusplus
}
#endif
#endif
