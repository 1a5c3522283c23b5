// CPU fused dequant-matmul (include/epq_cpu.h): the product path behind
// epure.kernels.cpu.linear for CPU activations.
//
// Arithmetic contract (the reference's kernel/src/lib.rs:36-151): for output
// row r and activation row mi, out = sum over groups g (in order) of
// acc_g = sum over the group's columns c (in order) of x[mi, c] * w[r, c], with
// w[r, c] = cb[e] * scale[r, g] rounded to f32 and every product rounded to f32
// before it is added (built with -ffp-contract=off, so no FMA).  The reference
// forms w through a per-group table of cb * scale; each table entry is that
// same single rounding, so forming w on the fly gives the same bits without
// building a levels * vec table per group (1,024 entries for a 256 x 4 vector
// codebook, more work than the group's 128 weights).
//
// Work split: output rows in blocks over OpenMP threads; within a row, groups
// outermost so a group's index bytes and activations stay in L1 while every
// activation row walks them.  Built for x86-64 with an AVX2 clone chosen at
// load time where the CPU has it.
#include <omp.h>
#include <stdarg.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>

#include "epq_cpu.h"

namespace {

thread_local char g_err[256] = "";

int fail(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

enum { kOk = 0, kEInval = -1, kEShape = -2, kEUnsupported = -8 };

// Index of column c in a row: the three byte layouts of the header.
template <int kVec, int kBits>
inline int index_of(const uint8_t* row, int64_t c) {
    if (kVec == 4) return row[c >> 2];
    if (kBits == 4) {
        const uint8_t b = row[c >> 1];
        return (c & 1) ? (b >> 4) : (b & 0x0F);
    }
    return row[c];
}

template <int kVec, int kBits>
__attribute__((target_clones("avx2", "default")))
void rows_range(const float* x, int64_t m, int64_t k, const uint8_t* packed, int64_t row_bytes,
                const float* cb, const float* scale, int64_t scale_stride, int64_t group, int64_t r0,
                int64_t r1, float* out, int64_t ldo) {
    for (int64_t r = r0; r < r1; ++r) {
        const uint8_t* row = packed + r * row_bytes;
        const float* srow = scale + r * scale_stride;
        for (int64_t mi = 0; mi < m; ++mi) out[mi * ldo + r] = 0.0f;
        int64_t g = 0;
        for (int64_t c0 = 0; c0 < k; c0 += group, ++g) {
            const int64_t c1 = std::min(k, c0 + group);
            const float s = srow[g];
            for (int64_t mi = 0; mi < m; ++mi) {
                const float* xr = x + mi * k;
                float acc = 0.0f;
                for (int64_t c = c0; c < c1; ++c) {
                    const int e = index_of<kVec, kBits>(row, c);
                    const float w = cb[kVec == 4 ? (e << 2) + (c & 3) : e] * s;
                    const float prod = xr[c] * w;
                    acc = acc + prod;
                }
                out[mi * ldo + r] += acc;
            }
        }
    }
}

using RowsFn = void (*)(const float*, int64_t, int64_t, const uint8_t*, int64_t, const float*, const float*,
                        int64_t, int64_t, int64_t, int64_t, float*, int64_t);

}  // namespace

extern "C" {

const char* epq_cpu_last_error(void) { return g_err; }

int epq_cpu_threads(void) { return omp_get_max_threads(); }

int epq_cpu_linear(const float* x, int64_t m, int64_t k, const uint8_t* packed, int64_t row_bytes,
                   int32_t bits, int32_t vec, int32_t levels, const float* cb, const float* scale,
                   int64_t scale_stride, int64_t group, int64_t n, float* out, int64_t ldo,
                   int32_t threads) {
    if (m < 0 || k < 0 || n < 0 || group <= 0) return fail(kEInval, "epq_cpu_linear: negative size or group");
    if (m == 0 || n == 0) return kOk;
    if (!x || !packed || !cb || !scale || !out) return fail(kEInval, "epq_cpu_linear: NULL pointer");
    RowsFn fn = nullptr;
    int64_t need = 0;
    if (vec == 4 && bits == 8) {
        if (k % 4) return fail(kEShape, "epq_cpu_linear: k=%lld not a multiple of 4", (long long)k);
        fn = rows_range<4, 8>;
        need = k / 4;
    } else if (vec == 1 && bits == 8) {
        fn = rows_range<1, 8>;
        need = k;
    } else if (vec == 1 && bits == 4) {
        if (levels > 16) return fail(kEInval, "epq_cpu_linear: %d levels in 4-bit indices", levels);
        fn = rows_range<1, 4>;
        need = (k + 1) / 2;
    } else {
        return fail(kEUnsupported, "epq_cpu_linear: vec=%d bits=%d", vec, bits);
    }
    if (levels <= 0 || levels > 256) return fail(kEInval, "epq_cpu_linear: levels=%d", levels);
    if (row_bytes < need) return fail(kEShape, "epq_cpu_linear: row_bytes=%lld < %lld", (long long)row_bytes,
                                      (long long)need);
    if (ldo < n) return fail(kEShape, "epq_cpu_linear: ldo < n");
    if (scale_stride < (k + group - 1) / group) return fail(kEShape, "epq_cpu_linear: scale_stride too small");
    const int nt = threads > 0 ? threads : omp_get_max_threads();
    // Blocks of rows sized so every thread gets several (load balance) and a
    // block's rows share cache lines of the output only at its edges.
    const int64_t block = std::max<int64_t>(16, n / (int64_t(nt) * 8));
    const int64_t nblocks = (n + block - 1) / block;
#pragma omp parallel for num_threads(nt) schedule(dynamic, 1)
    for (int64_t b = 0; b < nblocks; ++b) {
        const int64_t r0 = b * block, r1 = std::min(n, r0 + block);
        fn(x, m, k, packed, row_bytes, cb, scale, scale_stride, group, r0, r1, out, ldo);
    }
    return kOk;
}

}  // extern "C"
