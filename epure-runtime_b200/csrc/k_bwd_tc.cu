// Compressed-state backward on the 5th-generation tensor cores: the gradients
// of the codebook and of the group scales, with the indices frozen and the
// dense weight gradient never written.
//
//   dW = dY^T X                       [n, k]  (contraction over the m rows)
//   dscale[r, g] = sum_{c in g} dW[r, c] cb[idx(r, c)]
//   dcb[e, p]   += sum_{idx(r, c) = e, c % 4 = p} dW[r, c] scale[r, g(c)]
//
// Reference: the autograd of PackedWeight.materialize used by fine-tuning
// (epure/runtime.py:78-89 through epure/finetune.py:49-102; the formulas as in
// fine-tuning/README.md:64-68), which materialises dW densely.
//
// Design (B200, sm_100a).  One CTA owns a 128-row x 128-column tile of dW --
// exactly one scale group of 128 rows -- and contracts it over all m:
// * warp 0 loads, per 64-row slice of m, two 64 x 64 boxes of dY (columns r)
//   and two of X (columns c) with 2-D TMA (128-byte swizzle, zero fill past the
//   matrix, this CTA only).  Both tiles are MN-major for the MMA (the 64
//   contiguous elements of a swizzle row run along r resp. c), so neither
//   operand is transposed in memory;
// * warp 1 issues tcgen05.mma (kind::f16, M = N = 128, A and B MN-major) into
//   a 128 x 128 fp32 accumulator in TMEM, 4 MMAs (k = 16) per slice, and
//   commits each slice to its "empty" barrier;
// * warps 2-5 then read the tile row by row (thread = row r = TMEM lane), look
//   up the row's 32 codebook indices of the group, and reduce: dscale[r, g] as
//   one dot product per row (each (r, g) has exactly one owner: a plain store),
//   dcb through a shared-memory histogram [levels][4] (shared atomics) flushed
//   to global memory with one float atomic per entry per CTA.
// * Bounded mbarrier waits (device error flag + CTA abort word), TMEM released
//   after the last commit has landed, warp-collective TMEM loads reached by
//   whole warps.
#include "epq_common.cuh"
#include "epq_sm100.cuh"

namespace epq {
namespace {

using namespace sm100;

constexpr int kBT = 128;          // tile: 128 weight rows x 128 columns (one group)
constexpr int kMS = 64;           // m rows per stage
constexpr int kStages = 6;
constexpr int kHalf = 64 * 64 * 2;                 // one 64 x 64 box
constexpr int kStageBytes = 4 * kHalf;             // dY (2 boxes) + X (2 boxes)
constexpr int kCbOff = kStages * kStageBytes;      // fp32 codebook [256][4]
constexpr int kHistOff = kCbOff + 4096;            // fp32 histogram [256][4]
constexpr int kBarOff = kHistOff + 4096;
constexpr int kSmem = 1024 + kBarOff + 256;
constexpr int kThreads = 192;
constexpr uint32_t kWaitLimit = 1u << 22;
static_assert(kSmem <= 232448, "shared memory");

__device__ int g_bwd_wait_timeout = 0;

struct BwdParams {
    const uint8_t* idx;
    const void* scale;
    const void* cb;
    float* dscale;      // [n, ng] (may be null)
    float* dcb;         // [levels * 4] (may be null)
    int64_t s_n, s_g, kpos;
    int layout, scale_dtype, cb_dtype, levels;
    int n, k, ng, rb, m;
};

// The 32 index bytes of row r, group g, in position order (4 per word).
__device__ __forceinline__ void row_group_bytes(const BwdParams& P, int64_t r, int g, uint32_t (&w)[8]) {
    if (P.layout == EPQ_LAYOUT_MMA16) {
        // piece q (lane 4 (r % 8) + q, half (r / 8) % 2) holds positions q + 4 s, s = 0..7
        uint2 pc[4];
        const uint8_t* b = P.idx + (((int64_t)(r >> 4) * P.ng + g) * 32 + 4 * (r & 7)) * 16 + 8 * ((r >> 3) & 1);
#pragma unroll
        for (int q = 0; q < 4; ++q) pc[q] = ldg_nc_v2(b + 16 * q);
#pragma unroll
        for (int i = 0; i < 8; ++i) {       // word i = positions 4i .. 4i+3 = byte s = i of pieces 0..3
            const int s = i;
            const uint32_t b0 = ((s < 4 ? pc[0].x : pc[0].y) >> (8 * (s & 3))) & 0xFFu;
            const uint32_t b1 = ((s < 4 ? pc[1].x : pc[1].y) >> (8 * (s & 3))) & 0xFFu;
            const uint32_t b2 = ((s < 4 ? pc[2].x : pc[2].y) >> (8 * (s & 3))) & 0xFFu;
            const uint32_t b3 = ((s < 4 ? pc[3].x : pc[3].y) >> (8 * (s & 3))) & 0xFFu;
            w[i] = b0 | (b1 << 8) | (b2 << 16) | (b3 << 24);
        }
    } else if (P.layout == EPQ_LAYOUT_TILED) {
        const uint8_t* b = P.idx + (((int64_t)g * P.rb + (r >> 4)) * 32) * 16 + (r & 15);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            w[i] = ldg_nc_u8(b + (4 * i) * 16) | (ldg_nc_u8(b + (4 * i + 1) * 16) << 8) |
                   (ldg_nc_u8(b + (4 * i + 2) * 16) << 16) | (ldg_nc_u8(b + (4 * i + 3) * 16) << 24);
        }
    } else {
        const uint8_t* b = P.idx + r * P.kpos + (int64_t)g * 32;
        const uint4 a = ldg_nc_v4(b), c = ldg_nc_v4(b + 16);
        w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
        w[4] = c.x; w[5] = c.y; w[6] = c.z; w[7] = c.w;
    }
}

template <bool kBf16>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_dw_tc_kernel(const __grid_constant__ CUtensorMap ymap, const __grid_constant__ CUtensorMap xmap,
                     const __grid_constant__ BwdParams P) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;
    uint8_t* sgen = smem_raw + (sbase - raw);
    float* cbs = reinterpret_cast<float*>(sgen + kCbOff);
    float* hist = reinterpret_cast<float*>(sgen + kHistOff);
    const uint32_t bar0 = sbase + kBarOff;
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto empty = [&](int s) { return bar0 + 64u + 8u * s; };
    const uint32_t accum = bar0 + 128u;
    const uint32_t tslot = bar0 + 136u;
    volatile int* abortp = reinterpret_cast<volatile int*>(sgen + kBarOff + 140);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = blockIdx.x * kBT;
    const int g = blockIdx.y;
    const int c0 = g * kBT;
    const int nst = (P.m + kMS - 1) / kMS;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        mbar_init(accum, 1);
        *abortp = 0;
        mbar_init_fence();
    }
    if (warp == 1) tmem_alloc(tslot, kBT);
    for (int i = threadIdx.x; i < 1024; i += kThreads) {
        cbs[i] = (i < P.levels * 4) ? load_f(P.cb, P.cb_dtype, i) : 0.f;
        hist[i] = 0.f;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sgen + kBarOff + 136);

    if (warp == 0) {
        if (lane == 0) {
            tma_prefetch_desc(&ymap);
            tma_prefetch_desc(&xmap);
            int issued = 0;
            for (int kb = 0; kb < nst; ++kb) {
                const int s = kb % kStages;
                if (!mbar_wait_bounded(empty(s), ((kb / kStages) & 1) ^ 1, abortp, &g_bwd_wait_timeout,
                                       kWaitLimit))
                    break;
                const uint32_t st = sbase + s * kStageBytes;
                mbar_expect_tx(full(s), kStageBytes);
                tma_load_2d(st, &ymap, full(s), r0, kb * kMS);
                tma_load_2d(st + kHalf, &ymap, full(s), r0 + 64, kb * kMS);
                tma_load_2d(st + 2 * kHalf, &xmap, full(s), c0, kb * kMS);
                tma_load_2d(st + 3 * kHalf, &xmap, full(s), c0 + 64, kb * kMS);
                ++issued;
            }
            const int first = issued > kStages ? issued - kStages : 0;
            for (int kb = first; kb < issued; ++kb)
                for (uint32_t i = 0; i < kWaitLimit; ++i)
                    if (mbar_try_wait(full(kb % kStages), (kb / kStages) & 1)) break;
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16<kBf16, kBT, kBT, true, true>();
            for (int kb = 0; kb < nst; ++kb) {
                const int s = kb % kStages;
                if (!mbar_wait_bounded(full(s), (kb / kStages) & 1, abortp, &g_bwd_wait_timeout, kWaitLimit))
                    break;
                tc_fence_after();
                const uint32_t st = sbase + s * kStageBytes;
#pragma unroll
                for (int kk = 0; kk < kMS / 16; ++kk) {
                    const uint64_t ad = desc_mnmajor_sw128(st + kk * 2048, kHalf, 1024);
                    const uint64_t bd = desc_mnmajor_sw128(st + 2 * kHalf + kk * 2048, kHalf, 1024);
                    mma_f16_ss(tmem, ad, bd, idesc, (kb | kk) != 0);
                }
                mma_commit(empty(s));
            }
            mma_commit(accum);
            for (uint32_t i = 0; i < kWaitLimit; ++i)
                if (mbar_try_wait(accum, 0)) break;
        }
        __syncwarp();
    } else {
        // ---------------- epilogue: thread = weight row r ----------------
        const int sub = warp & 3;
        const int64_t r = (int64_t)r0 + 32 * sub + lane;
        const bool rv = r < P.n;
        uint32_t w[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        float sc = 0.f;
        if (rv) {
            row_group_bytes(P, r, g, w);
            sc = load_f(P.scale, P.scale_dtype, r * P.s_n + (int64_t)g * P.s_g);
        }
        const bool got = mbar_wait_bounded(accum, 0, abortp, &g_bwd_wait_timeout, kWaitLimit);
        const bool all = __all_sync(0xffffffffu, got);
        tc_fence_after();
        float ds = 0.f;
#pragma unroll 1
        for (int cc = 0; cc < kBT / 32; ++cc) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem + ((uint32_t)(sub * 32) << 16) + cc * 32, v);
            if (rv && all) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {     // positions 8 cc + q
                    const int jj = 8 * cc + q;
                    const uint32_t e = (w[jj >> 2] >> (8 * (jj & 3))) & 0xFFu;
                    const float4 cv = *reinterpret_cast<const float4*>(cbs + 4 * e);
                    const float d0 = __uint_as_float(v[4 * q]), d1 = __uint_as_float(v[4 * q + 1]);
                    const float d2 = __uint_as_float(v[4 * q + 2]), d3 = __uint_as_float(v[4 * q + 3]);
                    ds = fmaf(d0, cv.x, ds);
                    ds = fmaf(d1, cv.y, ds);
                    ds = fmaf(d2, cv.z, ds);
                    ds = fmaf(d3, cv.w, ds);
                    if (P.dcb) {
                        atomicAdd(hist + 4 * e, d0 * sc);
                        atomicAdd(hist + 4 * e + 1, d1 * sc);
                        atomicAdd(hist + 4 * e + 2, d2 * sc);
                        atomicAdd(hist + 4 * e + 3, d3 * sc);
                    }
                }
            }
        }
        if (rv && all && P.dscale) P.dscale[r * P.ng + g] = ds;
        asm volatile("bar.sync 1, 128;" ::: "memory");     // epilogue warps: histogram complete
        if (P.dcb && all) {
            for (int i = threadIdx.x - 64; i < P.levels * 4; i += 128)
                if (hist[i] != 0.f) atomicAdd(P.dcb + i, hist[i]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kBT);
    }
}


}  // namespace

int bwd_tc_read_device_error(int* flag) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_bwd_wait_timeout, sizeof(int)) != cudaSuccess)
        return check_launch("epq_device_error");
    *flag = v;
    return EPQ_OK;
}

bool bwd_tc_eligible(const StoreD& s, int64_t m, int act_dtype, const void* x, int64_t ldx,
                     const void* dy, int64_t ldy) {
    const bool lay = s.layout == EPQ_LAYOUT_MMA16 || s.layout == EPQ_LAYOUT_TILED ||
                     (s.layout == EPQ_LAYOUT_ROWS && (reinterpret_cast<uintptr_t>(s.idx) & 15) == 0);
    return lay && s.vec == 4 && s.bits == 8 && s.group == 128 && s.levels <= 256 && s.k % 128 == 0 &&
           m >= 64 && m < (int64_t(1) << 31) && s.n < (1 << 30) && s.n * 1 >= 1 &&
           (act_dtype == EPQ_BF16 || act_dtype == EPQ_F16) &&
           (reinterpret_cast<uintptr_t>(x) & 15) == 0 && (reinterpret_cast<uintptr_t>(dy) & 15) == 0 &&
           ldx % 8 == 0 && ldy % 8 == 0 && s.ng <= 65535;
}

// dscale / dcb through the tensor cores; dcb must be zeroed by the caller.
int launch_bwd_dw_tc(const StoreD& s, const void* x, int64_t ldx, const void* dy, int64_t ldy,
                     int act_dtype, int64_t m, float* dscale, float* dcb, cudaStream_t st) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return set_error(EPQ_EUNSUPPORTED, "device ordinal %d", dev);
    CUtensorMap ymap, xmap;
    int rc = make_tmap_2d(&ymap, dy, act_dtype, s.n, m, ldy, 64, kMS, "linear_bwd");
    if (rc) return rc;
    rc = make_tmap_2d(&xmap, x, act_dtype, s.k, m, ldx, 64, kMS, "linear_bwd");
    if (rc) return rc;
    BwdParams P{};
    P.idx = s.idx;
    P.scale = s.scale;
    P.cb = s.cb;
    P.dscale = dscale;
    P.dcb = dcb;
    P.s_n = s.s_n;
    P.s_g = s.s_g;
    P.kpos = s.kpos;
    P.layout = s.layout;
    P.scale_dtype = s.scale_dtype;
    P.cb_dtype = s.cb_dtype;
    P.levels = s.levels;
    P.n = (int)s.n;
    P.k = (int)s.k;
    P.ng = (int)s.ng;
    P.rb = (int)s.rb;
    P.m = (int)m;
    const bool bf = act_dtype == EPQ_BF16;
    auto kern = bf ? bwd_dw_tc_kernel<true> : bwd_dw_tc_kernel<false>;
    const int arc = set_smem_limit(reinterpret_cast<const void*>(kern), kSmem, "cudaFuncSetAttribute(bwd_dw_tc_kernel)");
    if (arc != EPQ_OK) return arc;
    const dim3 grid((unsigned)cdiv(s.n, kBT), (unsigned)s.ng);
    kern<<<grid, kThreads, kSmem, st>>>(ymap, xmap, P);
    return check_launch("bwd_dw_tc_kernel");
}

}  // namespace epq
