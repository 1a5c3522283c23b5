/*
 * TEST INFRASTRUCTURE ONLY -- never linked into the product library.
 *
 * CPU restatement of the reference's fused CPU kernel, epure-runtime
 * kernel/src/lib.rs (Rust, pyo3 + rayon).  Only tests/, the smoke check and
 * bench.py's CPU-baseline leg may load this.
 *
 * What is restated, and where it comes from:
 *   build_lut      lib.rs:36-40   lut[i] = cb[i] * scale, one table per group
 *   row_dot        lib.rs:47-88   per output row: for each group, build the
 *                                 LUT, then for each activation row a
 *                                 sequential f32 sum acc += x[k] * lut[idx],
 *                                 then out[mi] += acc
 *   dequant_matmul lib.rs:96-151  rows in parallel (rayon par_chunks_mut ->
 *                                 OpenMP here), result transposed [n,m]->[m,n]
 *
 * The summation order is the reference's: products are rounded to f32 before
 * each add (Rust does not contract mul+add into FMA), terms are added in k
 * order inside a group, and group sums are added to the output in group
 * order.  Build with -ffp-contract=off and without -ffast-math so the C
 * compiler keeps that order.
 *
 * Extension beyond the reference (the reference has no vector codebook):
 * vec = 4 means one index per 4 consecutive weights along k and a codebook of
 * `levels` entries of 4 floats.  The per-group LUT then holds levels*4 floats,
 * lut[e*4+p] = cb[e*4+p] * scale, and weight k reads lut[idx[k/4]*4 + k%4].
 * With vec = 1 this is exactly the reference's table.
 *
 * Index layouts (row-major, one row of `row_bytes` per output row):
 *   vec=1, four_bit=1 : two indices per byte, even k in the low nibble
 *                       (lib.rs:69-79, runtime.py _pack4)
 *   vec=1, four_bit=0 : one u8 index per weight (lib.rs:80-84)
 *   vec=4             : one u8 index per 4 weights
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static void build_lut(const float* cb, int n_entries, float scale, float* lut) {
    for (int i = 0; i < n_entries; ++i) lut[i] = cb[i] * scale;
}

static void row_dot(const float* x, int64_t m, int64_t k, const uint8_t* packed_row,
                    const float* scales_row, const float* cb, int levels, int vec,
                    int64_t group, int four_bit, float* out /* [m] */) {
    float lut[1024];
    const int n_entries = levels * vec;
    int64_t gi = 0;
    for (int64_t start = 0; start < k; start += group, ++gi) {
        const int64_t end = (start + group < k) ? start + group : k;
        build_lut(cb, n_entries, scales_row[gi], lut);
        for (int64_t mi = 0; mi < m; ++mi) {
            const float* xrow = x + mi * k;
            float acc = 0.0f;
            if (vec == 4) {
                for (int64_t kk = start; kk < end; ++kk) {
                    const int e = packed_row[kk >> 2];
                    acc += xrow[kk] * lut[e * 4 + (kk & 3)];
                }
            } else if (four_bit) {
                int64_t kk = start;
                while (kk < end) {
                    const uint8_t byte = packed_row[kk >> 1];
                    acc += xrow[kk] * lut[byte & 0x0F];
                    if (kk + 1 < end) acc += xrow[kk + 1] * lut[byte >> 4];
                    kk += 2;
                }
            } else {
                for (int64_t kk = start; kk < end; ++kk) acc += xrow[kk] * lut[packed_row[kk]];
            }
            out[mi] += acc;
        }
    }
}

/* out[m, n] = x[m, k] @ dequant(packed)[n, k]^T.
 * packed: [n, row_bytes] row-major; scales: [n, n_groups] f32; cb: [levels*vec] f32.
 * threads <= 0 means "all OpenMP threads".  Returns 0, or -1 on a bad argument. */
int epq_oracle_dequant_matmul(const float* x, int64_t m, int64_t k, const uint8_t* packed,
                              int64_t n, int64_t row_bytes, const float* scales,
                              int64_t n_groups, const float* cb, int levels, int vec,
                              int64_t group, int four_bit, float* out, int threads) {
    if (!x || !packed || !scales || !cb || !out) return -1;
    if (m < 0 || n < 0 || k <= 0 || group <= 0) return -1;
    if (vec != 1 && vec != 4) return -1;
    if (levels <= 0 || levels * vec > 1024) return -1;
    if (vec == 4 && (k % 4) != 0) return -1;
    if (n_groups < (k + group - 1) / group) return -1;
    float* tmp = (float*)calloc((size_t)(m * n > 0 ? m * n : 1), sizeof(float));
    if (!tmp) return -1;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#else
    (void)threads;
#endif
    int64_t row;
#pragma omp parallel for schedule(static)
    for (row = 0; row < n; ++row) {
        row_dot(x, m, k, packed + row * row_bytes, scales + row * n_groups, cb, levels, vec,
                group, four_bit, tmp + row * m);
    }
    /* lib.rs:141-146: accumulated [n, m], handed back as [m, n]. */
    for (int64_t r = 0; r < n; ++r)
        for (int64_t mi = 0; mi < m; ++mi) out[mi * n + r] = tmp[r * m + mi];
    free(tmp);
    return 0;
}

/* lib.rs:155-157 `threads()`: how many workers the parallel loop will use. */
int epq_oracle_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
