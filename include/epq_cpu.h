/*
 * epq_cpu.h -- C ABI of the CPU fused dequant-matmul (libepq_cpu.so).
 *
 * The host-side counterpart of include/epq.h for activations that live on the
 * CPU.  Replaces the reference's Rust extension (epure-runtime v0.2.4,
 * kernel/src/lib.rs:96 dequant_matmul(x, packed, scales, cb, group, four_bit),
 * bound by epure/kernels/cpu.py:37-70): the same f32 arithmetic in the same
 * order -- per output row and group, w = cb[idx] * scale rounded to f32, a
 * sequential f32 sum of x * w over the group's weights (no fused multiply-add),
 * the group sums added to the output in group order -- so results are bit-equal
 * to the reference's kernel, over a wider range of stores: 4- or 8-bit scalar
 * indices (vec = 1) and 8-bit indices of 4-weight vector codebooks (vec = 4).
 * Output rows are split over OpenMP threads.  Nothing allocates; the call is
 * synchronous.  Status codes are epq.h's (0 or negative), with
 * epq_cpu_last_error() describing a failure on the calling thread.
 */
#ifndef EPQ_CPU_H
#define EPQ_CPU_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* out[mi * ldo + r] = sum_c x[mi * k + c] * W[r, c] for mi < m, r < n (f32), with
 *   W[r, c] = cb[idx(r, c) * vec + c % vec] * scale[r * scale_stride + c / group]
 * and idx(r, c) read from row r of `packed` (row_bytes bytes per row):
 *   vec = 1, bits = 4: two indices per byte, even c in the low nibble;
 *   vec = 1, bits = 8: one byte per weight;
 *   vec = 4, bits = 8: one byte per 4 weights.
 * threads <= 0 uses every available thread. */
int epq_cpu_linear(const float* x, int64_t m, int64_t k, const uint8_t* packed, int64_t row_bytes,
                   int32_t bits, int32_t vec, int32_t levels, const float* cb, const float* scale,
                   int64_t scale_stride, int64_t group, int64_t n, float* out, int64_t ldo,
                   int32_t threads);

/* Threads a call with threads <= 0 uses. */
int epq_cpu_threads(void);

/* Description of the last failure on the calling thread. */
const char* epq_cpu_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* EPQ_CPU_H */
