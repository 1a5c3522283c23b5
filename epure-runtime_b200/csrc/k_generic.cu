// General-purpose kernels for every store format the ABI accepts: any vec /
// bits / layout / group, any number of activation rows.  They are tiled SIMT
// code with fp32 accumulation.  The batch-1 bandwidth kernel (k_gemv_lut.cu)
// covers the decode hot path; these cover everything else (scalar reference
// codebooks, prefill-sized batches, the backward, materialize, re-layout).
//
// Semantics follow the reference:
//   forward      out = x @ (cb[idx] * scale)^T            epure/kernels/_triton.py:56-107
//   materialize  W = cb.to(dt)[idx] * scale.to(dt)        epure/runtime.py:78-89
//   embedding    rows ids of that W, nothing else built   epure/runtime.py:129-160
//   backward     dX = dY W; dscale, dcb as the autograd of materialize
//                (epure/finetune.py:26-28, fine-tuning/README.md:64-68)
#include "epq_common.cuh"

namespace epq {
namespace {

constexpr int kBM = 32, kBN = 64, kBK = 32;  // forward tile: m x n, k-step
constexpr int kMaxCb = 1024;                 // levels * vec

// Codebook values to fp32 shared memory (unrounded).
__device__ __forceinline__ void load_cb_shared(const StoreD& s, float* cbs) {
    const int ncb = s.levels * s.vec;
    for (int i = threadIdx.x; i < ncb; i += blockDim.x) cbs[i] = load_f(s.cb, s.cb_dtype, i);
}

__device__ __forceinline__ float weight_at(const StoreD& s, const float* cbs, int64_t r,
                                           int64_t c) {
    const int e = index_at(s, r, c);
    const float v = cbs[e * s.vec + (s.vec == 4 ? (c & 3) : 0)];
    return v * scale_at(s, r, c / s.group);
}

// out[m, n] = x[m, :] . W[n, :]; 256 threads, each a 2 (m) x 4 (n) block.
__global__ void __launch_bounds__(256) linear_generic_kernel(StoreD s, const void* __restrict__ x,
                                                             int x_dtype, int64_t M, int64_t ldx,
                                                             void* __restrict__ out, int64_t ldo,
                                                             int out_dtype) {
    __shared__ float cbs[kMaxCb];
    __shared__ float xs[kBK][kBM + 1];
    __shared__ float ws[kBK][kBN + 1];
    load_cb_shared(s, cbs);
    const int64_t m0 = (int64_t)blockIdx.y * kBM, n0 = (int64_t)blockIdx.x * kBN;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[2][4] = {};
    for (int64_t k0 = 0; k0 < s.k; k0 += kBK) {
        __syncthreads();
        for (int i = threadIdx.x; i < kBM * kBK; i += 256) {
            const int mm = i / kBK, kk = i % kBK;
            const int64_t gm = m0 + mm, gk = k0 + kk;
            xs[kk][mm] = (gm < M && gk < s.k) ? load_f(x, x_dtype, gm * ldx + gk) : 0.f;
        }
        for (int i = threadIdx.x; i < kBN * kBK; i += 256) {
            const int nn = i / kBK, kk = i % kBK;
            const int64_t gn = n0 + nn, gk = k0 + kk;
            ws[kk][nn] = (gn < s.n && gk < s.k) ? weight_at(s, cbs, gn, gk) : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < kBK; ++kk) {
            float a[2], b[4];
            for (int i = 0; i < 2; ++i) a[i] = xs[kk][ty * 2 + i];
            for (int j = 0; j < 4; ++j) b[j] = ws[kk][tx + 16 * j];
            for (int i = 0; i < 2; ++i)
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
    }
    for (int i = 0; i < 2; ++i) {
        const int64_t gm = m0 + ty * 2 + i;
        if (gm >= M) continue;
        for (int j = 0; j < 4; ++j) {
            const int64_t gn = n0 + tx + 16 * j;
            if (gn < s.n) store_f(out, out_dtype, gm * ldo + gn, acc[i][j]);
        }
    }
}

// dX[m, c] = sum_r dY[m, r] W[r, c]; tile 32 (m) x 64 (c), loop over r.
__global__ void __launch_bounds__(256) bwd_dx_kernel(StoreD s, const void* __restrict__ dy,
                                                     int64_t ldy, int act_dtype, int64_t M,
                                                     void* __restrict__ dx, int64_t lddx,
                                                     int dx_dtype) {
    __shared__ float cbs[kMaxCb];
    __shared__ float ys[kBK][kBM + 1];   // [r][m]
    __shared__ float ws[kBK][kBN + 1];   // [r][c]
    load_cb_shared(s, cbs);
    const int64_t m0 = (int64_t)blockIdx.y * kBM, c0 = (int64_t)blockIdx.x * kBN;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[2][4] = {};
    for (int64_t r0 = 0; r0 < s.n; r0 += kBK) {
        __syncthreads();
        for (int i = threadIdx.x; i < kBM * kBK; i += 256) {
            const int mm = i / kBK, rr = i % kBK;
            const int64_t gm = m0 + mm, gr = r0 + rr;
            ys[rr][mm] = (gm < M && gr < s.n) ? load_f(dy, act_dtype, gm * ldy + gr) : 0.f;
        }
        for (int i = threadIdx.x; i < kBN * kBK; i += 256) {
            const int cc = i % kBN, rr = i / kBN;
            const int64_t gc = c0 + cc, gr = r0 + rr;
            ws[rr][cc] = (gc < s.k && gr < s.n) ? weight_at(s, cbs, gr, gc) : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int rr = 0; rr < kBK; ++rr) {
            float a[2], b[4];
            for (int i = 0; i < 2; ++i) a[i] = ys[rr][ty * 2 + i];
            for (int j = 0; j < 4; ++j) b[j] = ws[rr][tx + 16 * j];
            for (int i = 0; i < 2; ++i)
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
    }
    for (int i = 0; i < 2; ++i) {
        const int64_t gm = m0 + ty * 2 + i;
        if (gm >= M) continue;
        for (int j = 0; j < 4; ++j) {
            const int64_t gc = c0 + tx + 16 * j;
            if (gc < s.k) store_f(dx, dx_dtype, gm * lddx + gc, acc[i][j]);
        }
    }
}

// dW tile (64 rows x 64 cols, never stored) reduced into dscale and dcb.
constexpr int kWT = 64, kMT = 16, kMaxGroupsInTile = kWT + 2;
__global__ void __launch_bounds__(256) bwd_dw_kernel(StoreD s, const void* __restrict__ x,
                                                     int64_t ldx, const void* __restrict__ dy,
                                                     int64_t ldy, int act_dtype, int64_t M,
                                                     float* __restrict__ dscale,
                                                     float* __restrict__ dcb) {
    __shared__ float cbs[kMaxCb];
    __shared__ float hist[kMaxCb];
    __shared__ float dss[kWT][kMaxGroupsInTile];
    __shared__ float ys[kMT][kWT + 1];   // [m][r]
    __shared__ float xs[kMT][kWT + 1];   // [m][c]
    load_cb_shared(s, cbs);
    const int ncb = s.levels * s.vec;
    for (int i = threadIdx.x; i < ncb; i += 256) hist[i] = 0.f;
    for (int i = threadIdx.x; i < kWT * kMaxGroupsInTile; i += 256) (&dss[0][0])[i] = 0.f;
    const int64_t r0 = (int64_t)blockIdx.y * kWT, c0 = (int64_t)blockIdx.x * kWT;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    float acc[4][4] = {};  // rows ty*4+i, cols tx + 16*j
    for (int64_t mb = 0; mb < M; mb += kMT) {
        __syncthreads();
        for (int i = threadIdx.x; i < kMT * kWT; i += 256) {
            const int mm = i / kWT, q = i % kWT;
            const int64_t gm = mb + mm;
            ys[mm][q] = (gm < M && r0 + q < s.n) ? load_f(dy, act_dtype, gm * ldy + r0 + q) : 0.f;
            xs[mm][q] = (gm < M && c0 + q < s.k) ? load_f(x, act_dtype, gm * ldx + c0 + q) : 0.f;
        }
        __syncthreads();
#pragma unroll 4
        for (int mm = 0; mm < kMT; ++mm) {
            float a[4], b[4];
            for (int i = 0; i < 4; ++i) a[i] = ys[mm][ty * 4 + i];
            for (int j = 0; j < 4; ++j) b[j] = xs[mm][tx + 16 * j];
            for (int i = 0; i < 4; ++i)
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
    }
    __syncthreads();
    const int64_t g0 = c0 / s.group;
    for (int i = 0; i < 4; ++i) {
        const int64_t r = r0 + ty * 4 + i;
        if (r >= s.n) continue;
        for (int j = 0; j < 4; ++j) {
            const int64_t c = c0 + tx + 16 * j;
            if (c >= s.k) continue;
            const int e = index_at(s, r, c);
            const int slot = e * s.vec + (s.vec == 4 ? (int)(c & 3) : 0);
            const int64_t g = c / s.group;
            const float dw = acc[i][j];
            atomicAdd(&dss[ty * 4 + i][g - g0], dw * cbs[slot]);
            atomicAdd(&hist[slot], dw * scale_at(s, r, g));
        }
    }
    __syncthreads();
    if (dcb) {
        for (int i = threadIdx.x; i < ncb; i += 256)
            if (hist[i] != 0.f) atomicAdd(&dcb[i], hist[i]);
    }
    if (dscale) {
        const int64_t g_last = (c0 + kWT - 1 < s.k ? c0 + kWT - 1 : s.k - 1) / s.group;
        const int ngt = (int)(g_last - g0 + 1);
        for (int i = threadIdx.x; i < kWT * ngt; i += 256) {
            const int rr = i / ngt, gl = i % ngt;
            const int64_t r = r0 + rr;
            if (r < s.n) atomicAdd(&dscale[r * s.ng + g0 + gl], dss[rr][gl]);
        }
    }
}

__global__ void materialize_kernel(StoreD s, void* __restrict__ w, int64_t ldw, int out_dtype) {
    const int64_t total = s.n * s.k;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = t / s.k, c = t - r * s.k;
        const int e = index_at(s, r, c);
        const float cv = round_to(load_f(s.cb, s.cb_dtype, e * s.vec + (s.vec == 4 ? (c & 3) : 0)),
                                  out_dtype);
        const float sv = round_to(scale_at(s, r, c / s.group), out_dtype);
        store_f(w, out_dtype, r * ldw + c, cv * sv);
    }
}

// PackedEmbedding.forward: out[i, :] = W[ids[i], :] with materialize's rounding,
// decoding only the requested rows.  An id outside [0, n) yields a zero row and
// sets g_embed_bad (reported by epq_device_error).
__device__ int g_embed_bad = 0;

__global__ void embedding_kernel(StoreD s, const int64_t* __restrict__ ids, int64_t n_ids,
                                 void* __restrict__ out, int64_t ldo, int out_dtype) {
    const int64_t total = n_ids * s.k;
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = t / s.k, c = t - i * s.k;
        int64_t r = ids[i];
        if (r < 0) r += s.n;          // negative ids count from the end, as torch indexing does
        if (r < 0 || r >= s.n) {
            if (c == 0) atomicExch(&g_embed_bad, 1);
            store_f(out, out_dtype, i * ldo + c, 0.f);
            continue;
        }
        const int e = index_at(s, r, c);
        const float cv = round_to(load_f(s.cb, s.cb_dtype, e * s.vec + (s.vec == 4 ? (c & 3) : 0)),
                                  out_dtype);
        const float sv = round_to(scale_at(s, r, c / s.group), out_dtype);
        store_f(out, out_dtype, i * ldo + c, cv * sv);
    }
}

// EPQ_LAYOUT_TILED: one thread per 16-byte chunk (16 rows of one index position).
__global__ void relayout_tiled_kernel(const uint8_t* __restrict__ src, int64_t n, int64_t kpos,
                                      int64_t p, int64_t rb, int64_t chunks,
                                      uint8_t* __restrict__ dst) {
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < chunks;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t l = t % p, gb = t / p;
        const int64_t b = gb % rb, g = gb / rb;
        const int64_t j = g * p + l;
        uint32_t words[4] = {0, 0, 0, 0};
        for (int rr = 0; rr < 16; ++rr) {
            const int64_t r = b * 16 + rr;
            const uint32_t v = (r < n && j < kpos) ? src[r * kpos + j] : 0u;
            words[rr >> 2] |= v << (8 * (rr & 3));
        }
        reinterpret_cast<uint4*>(dst)[t] = make_uint4(words[0], words[1], words[2], words[3]);
    }
}

// EPQ_LAYOUT_MMA16: one thread per 16-byte chunk (lane t of a tile: rows
// rb*16 + t/4 and + 8, positions t%4 + 4s of its group, s = 0..7).
__global__ void relayout_mma16_kernel(const uint8_t* __restrict__ src, int64_t n, int64_t kpos,
                                      int64_t ng, int64_t chunks, uint8_t* __restrict__ dst) {
    for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < chunks;
         t += (int64_t)gridDim.x * blockDim.x) {
        const int64_t lane = t & 31, bg = t >> 5;
        const int64_t g = bg % ng, b = bg / ng;
        uint32_t words[4] = {0, 0, 0, 0};
        for (int h = 0; h < 2; ++h) {
            const int64_t r = b * 16 + 8 * h + (lane >> 2);
            for (int s = 0; s < 8; ++s) {
                const int64_t j = g * 32 + 4 * s + (lane & 3);
                const uint32_t v = (r < n && j < kpos) ? src[r * kpos + j] : 0u;
                words[2 * h + (s >> 2)] |= v << (8 * (s & 3));
            }
        }
        reinterpret_cast<uint4*>(dst)[t] = make_uint4(words[0], words[1], words[2], words[3]);
    }
}

int grid_1d(int64_t work, int threads) {
    int64_t b = cdiv(work, threads);
    if (b > 148 * 32) b = 148 * 32;
    return (int)(b < 1 ? 1 : b);
}

}  // namespace

int launch_linear_generic(const StoreD& s, const void* x, int x_dtype, int64_t m, int64_t ldx,
                          void* out, int64_t ldo, int out_dtype, cudaStream_t st) {
    if (m == 0 || s.n == 0) return EPQ_OK;
    dim3 grid((unsigned)cdiv(s.n, kBN), (unsigned)cdiv(m, kBM));
    if (grid.y > 65535) return set_error(EPQ_EUNSUPPORTED, "linear: m=%lld too large", (long long)m);
    linear_generic_kernel<<<grid, 256, 0, st>>>(s, x, x_dtype, m, ldx, out, ldo, out_dtype);
    return check_launch("linear_generic_kernel");
}

int launch_bwd_generic(const StoreD& s, const void* x, int64_t ldx, const void* dy, int64_t ldy,
                       int act_dtype, int64_t m, void* dx, int64_t lddx, int dx_dtype,
                       float* dscale, float* dcb, cudaStream_t st) {
    if (dscale && cudaMemsetAsync(dscale, 0, sizeof(float) * s.n * s.ng, st) != cudaSuccess)
        return check_launch("memset dscale");
    if (dcb && cudaMemsetAsync(dcb, 0, sizeof(float) * s.levels * s.vec, st) != cudaSuccess)
        return check_launch("memset dcb");
    if (dx && m > 0 && s.k > 0) {
        dim3 grid((unsigned)cdiv(s.k, kBN), (unsigned)cdiv(m, kBM));
        if (grid.y > 65535) return set_error(EPQ_EUNSUPPORTED, "bwd: m too large");
        bwd_dx_kernel<<<grid, 256, 0, st>>>(s, dy, ldy, act_dtype, m, dx, lddx, dx_dtype);
        int rc = check_launch("bwd_dx_kernel");
        if (rc) return rc;
    }
    if ((dscale || dcb) && m > 0 && s.n > 0) {
        dim3 grid((unsigned)cdiv(s.k, kWT), (unsigned)cdiv(s.n, kWT));
        if (grid.y > 65535) return set_error(EPQ_EUNSUPPORTED, "bwd: n too large");
        bwd_dw_kernel<<<grid, 256, 0, st>>>(s, x, ldx, dy, ldy, act_dtype, m, dscale, dcb);
        return check_launch("bwd_dw_kernel");
    }
    return EPQ_OK;
}

int launch_materialize(const StoreD& s, void* w, int64_t ldw, int out_dtype, cudaStream_t st) {
    if (s.n * s.k == 0) return EPQ_OK;
    materialize_kernel<<<grid_1d(s.n * s.k, 256), 256, 0, st>>>(s, w, ldw, out_dtype);
    return check_launch("materialize_kernel");
}

int launch_embedding(const StoreD& s, const int64_t* ids, int64_t n_ids, void* out, int64_t ldo,
                     int out_dtype, cudaStream_t st) {
    if (n_ids * s.k == 0) return EPQ_OK;
    embedding_kernel<<<grid_1d(n_ids * s.k, 256), 256, 0, st>>>(s, ids, n_ids, out, ldo, out_dtype);
    return check_launch("embedding_kernel");
}

int embed_read_device_error(int* flag) {
    if (cudaMemcpyFromSymbol(flag, g_embed_bad, sizeof(int)) != cudaSuccess)
        return check_launch("read embedding error flag");
    return EPQ_OK;
}

int64_t layout_bytes(int layout, int64_t n, int64_t k, int vec, int group) {
    if (layout == EPQ_LAYOUT_TILED) return cdiv(k, group) * cdiv(n, 16) * (group / vec) * 16;
    if (layout == EPQ_LAYOUT_MMA16) return cdiv(k, group) * cdiv(n, 16) * 512;
    return -1;
}

int launch_relayout(const uint8_t* src, int layout, int64_t n, int64_t k, int vec, int group,
                    uint8_t* dst, cudaStream_t st) {
    const int64_t kpos = k / vec, ng = cdiv(k, group);
    if (layout == EPQ_LAYOUT_TILED) {
        const int64_t p = group / vec, rb = cdiv(n, 16);
        const int64_t chunks = ng * rb * p;
        if (chunks == 0) return EPQ_OK;
        relayout_tiled_kernel<<<grid_1d(chunks, 256), 256, 0, st>>>(src, n, kpos, p, rb, chunks, dst);
        return check_launch("relayout_tiled_kernel");
    }
    const int64_t rb = cdiv(n, 16), chunks = ng * rb * 32;
    if (chunks == 0) return EPQ_OK;
    relayout_mma16_kernel<<<grid_1d(chunks, 256), 256, 0, st>>>(src, n, kpos, ng, chunks, dst);
    return check_launch("relayout_mma16_kernel");
}

}  // namespace epq
