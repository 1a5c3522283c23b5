// Backward activation gradient on the 5th-generation tensor cores:
//   dX[m, c] = sum_r dY[m, r] W[r, c],  W[r, 4j+p] = cb[idx[r, j], p] * scale[r, g(j)].
//
// Reference: the autograd of F.linear(x, materialize(dtype)) (epure/runtime.py:
// 78-89, 123-124), which multiplies dY by the materialised weight.
//
// Design (B200, sm_100a): the forward tensor-core GEMM with the weight decoded
// along its rows instead of along k.  One CTA computes a 128 (columns c of W =
// one scale group) x BN (rows of dY) tile of dX^T; the contraction runs over
// the store's rows r in stages of 64:
// * warp 0 loads the dY tile (2-D TMA, 128-byte swizzle, zero fill past the
//   matrix) and, with bulk copies into the same stage, the 64 x 32 index bytes
//   of the stage's four 16-row blocks (the store's own EPQ_LAYOUT_MMA16 or
//   EPQ_LAYOUT_TILED tiles) and the 64 group scales;
// * warps 2-9 decode W^T straight into TENSOR MEMORY: thread = column c = TMEM
//   lane, two warps per lane quarter each taking 32 of the stage's 64 rows.
//   Per row: the index byte, one 2-byte codebook component from a 16-way
//   replicated codebook (the 4 lanes sharing an index byte read the same
//   8-byte word; 8 index bytes per warp land in 8 different bank pairs), times
//   the row's scale in the activation type (the reference's
//   cb.to(dtype)[idx] * scale.to(dtype)); row pairs are packed into 32-bit
//   TMEM columns and stored with tcgen05.st;
// * warp 1 issues tcgen05.mma (kind::f16, A from TMEM, B = the dY tile in
//   shared memory, fp32 D in TMEM columns 0 .. BN-1);
// * warps 2-9 then read D (tcgen05.ld) and write dX in the requested dtype.
// Bounded waits, warp-uniform collective TMEM instructions, TMEM released after
// the last commit, as in the forward kernel.
#include "epq_common.cuh"
#include "epq_sm100.cuh"

namespace epq {
namespace {

using namespace sm100;

constexpr int kCols = 128;                 // columns of W per tile (one group)
constexpr int kRS = 64;                    // rows of W per stage
constexpr int kDecWarps = 8;
constexpr int kThreads = 64 + kDecWarps * 32;
constexpr int kReplicaBytes = 256 * 16 * 8;
constexpr int kIdxStage = 4 * 512;         // four 16-row blocks of one group
constexpr int kScStage = 256;              // 64 scales, up to fp32
constexpr int kMaxStages = 8;
constexpr int kAStageCols = kRS / 2;
constexpr uint32_t kACol0 = 256;
constexpr uint32_t kTmemCols = 512;
constexpr int kSmemLimit = 232448;
constexpr uint32_t kWaitLimit = 1u << 22;

__device__ int g_dx_wait_timeout = 0;

template <int BN>
struct Cfg {
    static constexpr int kXStage = BN * kRS * 2;
    static constexpr int kStageBytes = kXStage + kIdxStage + kScStage;
    static constexpr int kStagesRaw = (kSmemLimit - 1024 - 256 - kReplicaBytes) / kStageBytes;
    static constexpr int kStages = kStagesRaw > kMaxStages ? kMaxStages : kStagesRaw;
    static constexpr int kXOff = kReplicaBytes;
    static constexpr int kIdxOff = kXOff + kStages * kXStage;
    static constexpr int kScOff = kIdxOff + kStages * kIdxStage;
    static constexpr int kBarOff = kScOff + kStages * kScStage;
    static constexpr int kSmem = 1024 + kBarOff + 256;
    static_assert(kStages >= 2, "stages");
    static_assert(kSmem <= kSmemLimit, "shared memory");
};

struct DxParams {
    const uint8_t* idx;
    const void* scale;     // group-major: scale(r, g) at g * s_g + r
    int64_t s_g;
    const void* cb;
    void* dx;
    int64_t lddx;
    int cb_dtype, scale_f32, levels;
    int n, k, ng, rb, m, out_dtype;
};

template <bool kBf16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if constexpr (kBf16) {
        __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    } else {
        __half2 v = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
}
template <bool kBf16>
__device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b) {
    if constexpr (kBf16) {
        __nv_bfloat162 r = __hmul2(*reinterpret_cast<__nv_bfloat162*>(&a),
                                   *reinterpret_cast<__nv_bfloat162*>(&b));
        return *reinterpret_cast<uint32_t*>(&r);
    } else {
        __half2 r = __hmul2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
        return *reinterpret_cast<uint32_t*>(&r);
    }
}
__device__ __forceinline__ uint32_t lds_u8(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds_u16(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds_u32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

template <bool kBf16, int kLayout, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    bwd_dx_tc_kernel(const __grid_constant__ CUtensorMap ymap, const __grid_constant__ DxParams P) {
    using C = Cfg<BN>;
    constexpr int S_ = C::kStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;
    uint8_t* sgen = smem_raw + (sbase - raw);
    const uint32_t xst0 = sbase + C::kXOff, ist0 = sbase + C::kIdxOff, sst0 = sbase + C::kScOff;
    const uint32_t bar0 = sbase + C::kBarOff;
    auto full_x = [&](int s) { return bar0 + 8u * s; };
    auto full_w = [&](int s) { return bar0 + 64u + 8u * s; };
    auto empty = [&](int s) { return bar0 + 128u + 8u * s; };
    const uint32_t accum = bar0 + 192u;
    const uint32_t tslot = bar0 + 200u;
    volatile int* abortp = reinterpret_cast<volatile int*>(sgen + C::kBarOff + 204);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = blockIdx.x;                 // column tile = scale group
    const int m0 = blockIdx.y * BN;
    const int nkb = P.n / kRS;
    const uint32_t esz = P.scale_f32 ? 4u : 2u;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S_; ++s) {
            mbar_init(full_x(s), 1);
            mbar_init(full_w(s), kDecWarps);
            mbar_init(empty(s), 1);
        }
        mbar_init(accum, 1);
        *abortp = 0;
        mbar_init_fence();
    }
    if (warp == 1) tmem_alloc(tslot, kTmemCols);
    uint2* conv = reinterpret_cast<uint2*>(sgen + C::kXOff);
    for (int e = threadIdx.x; e < 256; e += kThreads) {
        uint2 v = make_uint2(0u, 0u);
        if (e < P.levels) {
            const int64_t b = (int64_t)e * 4;
            v.x = pack2<kBf16>(load_f(P.cb, P.cb_dtype, b), load_f(P.cb, P.cb_dtype, b + 1));
            v.y = pack2<kBf16>(load_f(P.cb, P.cb_dtype, b + 2), load_f(P.cb, P.cb_dtype, b + 3));
        }
        conv[e] = v;
    }
    __syncthreads();
    for (int slot = threadIdx.x; slot < 256 * 16; slot += kThreads)
        reinterpret_cast<uint2*>(sgen)[slot] = conv[slot >> 4];
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sgen + C::kBarOff + 200);

    if (warp == 0) {
        // ---------------- dY tiles (TMA) + index tiles and scales (bulk copies) ----------------
        if (lane == 0) {
            tma_prefetch_desc(&ymap);
            int issued = 0;
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % S_;
                if (!mbar_wait_bounded(empty(s), ((kb / S_) & 1) ^ 1, abortp, &g_dx_wait_timeout, kWaitLimit))
                    break;
                mbar_expect_tx(full_x(s), C::kXStage + kIdxStage + kRS * esz);
                tma_load_2d(xst0 + s * C::kXStage, &ymap, full_x(s), kb * kRS, m0);
                const int rb0 = kb * (kRS / 16);
                if constexpr (kLayout == EPQ_LAYOUT_MMA16) {
                    for (int q = 0; q < 4; ++q)
                        bulk_g2s(ist0 + s * kIdxStage + 512 * q,
                                 P.idx + ((int64_t)(rb0 + q) * P.ng + g) * 512, 512, full_x(s));
                } else {
                    bulk_g2s(ist0 + s * kIdxStage, P.idx + ((int64_t)g * P.rb + rb0) * 512, kIdxStage,
                             full_x(s));
                }
                bulk_g2s(sst0 + s * kScStage,
                         static_cast<const uint8_t*>(P.scale) + ((int64_t)g * P.s_g + (int64_t)kb * kRS) * esz,
                         kRS * esz, full_x(s));
                ++issued;
            }
            const int first = issued > S_ ? issued - S_ : 0;
            for (int kb = first; kb < issued; ++kb)
                for (uint32_t i = 0; i < kWaitLimit; ++i)
                    if (mbar_try_wait(full_x(kb % S_), (kb / S_) & 1)) break;
        }
    } else if (warp == 1) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16<kBf16, kCols, BN>();
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % S_;
                const uint32_t par = (kb / S_) & 1;
                if (!mbar_wait_bounded(full_x(s), par, abortp, &g_dx_wait_timeout, kWaitLimit)) break;
                if (!mbar_wait_bounded(full_w(s), par, abortp, &g_dx_wait_timeout, kWaitLimit)) break;
                tc_fence_after();
                const uint32_t ta = tmem + kACol0 + s * kAStageCols;
                const uint64_t bd = desc_kmajor_sw128(xst0 + s * C::kXStage);
#pragma unroll
                for (int kk = 0; kk < kRS / 16; ++kk)
                    mma_f16_ts(tmem, ta + 8 * kk, bd + 2 * kk, idesc, (kb | kk) != 0);
                mma_commit(empty(s));
            }
            mma_commit(accum);
            for (uint32_t i = 0; i < kWaitLimit; ++i)
                if (mbar_try_wait(accum, 0)) break;
        }
        __syncwarp();
    } else {
        // ---------------- decode W^T rows into TMEM ----------------
        const int sub = warp & 3, half = (warp - 2) >> 2;
        const int cl = 32 * sub + lane;          // column within the group = TMEM lane
        const int j = cl >> 2, p = cl & 3;       // index position, codebook component
        const uint32_t rep = sbase + (uint32_t)(j & 7) * 8u + 2u * p;
        const uint32_t trow = tmem + ((uint32_t)(32 * sub) << 16) + kACol0 + 16 * half;
        // byte offset of (row rr of a 16-row block, position j) inside that block's tile
        auto boff = [&](int rr) -> uint32_t {
            if constexpr (kLayout == EPQ_LAYOUT_MMA16)
                return (uint32_t)((4 * (rr & 7) + (j & 3)) * 16 + 8 * (rr >> 3) + (j >> 2));
            else
                return (uint32_t)(j * 16 + rr);
        };
        uint32_t bo[16];
#pragma unroll
        for (int rr = 0; rr < 16; ++rr) bo[rr] = boff(rr);
        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb % S_;
            const bool w_ok = mbar_wait_bounded(full_x(s), (kb / S_) & 1, abortp, &g_dx_wait_timeout,
                                                kWaitLimit) &&
                              mbar_wait_bounded(empty(s), ((kb / S_) & 1) ^ 1, abortp, &g_dx_wait_timeout,
                                                kWaitLimit);
            if (!__all_sync(0xffffffffu, w_ok)) break;
            tc_fence_after();
            const uint32_t ib = ist0 + s * kIdxStage + 1024u * half;   // rows 32 half .. +31: blocks 2 half, +1
            const uint32_t sb = sst0 + s * kScStage + 32u * half * esz;
            uint32_t v[16];
#pragma unroll
            for (int q = 0; q < 16; ++q) {            // rows 2q, 2q+1 of this warp's 32
                const int r0 = 2 * q, r1 = 2 * q + 1;
                const uint32_t e0 = lds_u8(ib + 512u * (r0 >> 4) + bo[r0 & 15]);
                const uint32_t e1 = lds_u8(ib + 512u * (r1 >> 4) + bo[r1 & 15]);
                const uint32_t c0 = lds_u16(rep + e0 * 128u), c1 = lds_u16(rep + e1 * 128u);
                uint32_t sc;
                if (P.scale_f32) {
                    const uint2 f = make_uint2(lds_u32(sb + 8u * q), lds_u32(sb + 8u * q + 4u));
                    sc = pack2<kBf16>(__uint_as_float(f.x), __uint_as_float(f.y));
                } else {
                    const uint32_t h = lds_u32(sb + 4u * q);
                    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h));
                    sc = pack2<kBf16>(f.x, f.y);
                }
                v[q] = mul2<kBf16>(c0 | (c1 << 16), sc);
            }
            tmem_st_32x32b_x16(trow + s * kAStageCols, v);
            tmem_st_wait();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(full_w(s));
        }

        // ---------------- epilogue: TMEM -> dX ----------------
        const bool got = mbar_wait_bounded(accum, 0, abortp, &g_dx_wait_timeout, kWaitLimit);
        tc_fence_after();
        const int64_t c = (int64_t)g * kCols + cl;
        const bool cv = got && c < P.k;
#pragma unroll 1
        for (int cc = half * (BN / 64); cc < (half + 1) * (BN / 64); ++cc) {
            if (m0 + cc * 32 >= P.m) break;
            uint32_t d[32];
            tmem_ld_32x32b_x32(tmem + ((uint32_t)(sub * 32) << 16) + cc * 32, d);
            if (cv) {
#pragma unroll
                for (int q = 0; q < 32; ++q) {
                    const int mm = m0 + cc * 32 + q;
                    if (mm < P.m) store_f(P.dx, P.out_dtype, (int64_t)mm * P.lddx + c, __uint_as_float(d[q]));
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}


template <bool kBf16, int kLayout, int BN>
int launch_dx(const CUtensorMap& ymap, const DxParams& P, int bi, cudaStream_t st, int dev) {
    using C = Cfg<BN>;
    auto kern = bwd_dx_tc_kernel<kBf16, kLayout, BN>;
    (void)bi;
    (void)dev;
    const int arc = set_smem_limit(reinterpret_cast<const void*>(kern), C::kSmem, "cudaFuncSetAttribute(bwd_dx_tc_kernel)");
    if (arc != EPQ_OK) return arc;
    const dim3 grid((unsigned)P.ng, (unsigned)cdiv(P.m, BN));
    kern<<<grid, kThreads, C::kSmem, st>>>(ymap, P);
    return check_launch("bwd_dx_tc_kernel");
}

template <bool kBf16, int kLayout>
int launch_dx_bn(int bn, const CUtensorMap& ymap, const DxParams& P, cudaStream_t st, int dev) {
    if (bn == 256) return launch_dx<kBf16, kLayout, 256>(ymap, P, 2, st, dev);
    if (bn == 128) return launch_dx<kBf16, kLayout, 128>(ymap, P, 1, st, dev);
    return launch_dx<kBf16, kLayout, 64>(ymap, P, 0, st, dev);
}

}  // namespace

int dx_tc_read_device_error(int* flag) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_dx_wait_timeout, sizeof(int)) != cudaSuccess)
        return check_launch("epq_device_error");
    *flag = v;
    return EPQ_OK;
}

bool dx_tc_eligible(const StoreD& s, int64_t m, int act_dtype, const void* dy, int64_t ldy) {
    const int64_t esz = s.scale_dtype == EPQ_F32 ? 4 : 2;
    return (s.layout == EPQ_LAYOUT_MMA16 || s.layout == EPQ_LAYOUT_TILED) && s.bits == 8 && s.vec == 4 &&
           s.group == 128 && s.levels <= 256 && s.p == 32 && s.k % 128 == 0 && s.n % 64 == 0 &&
           m > 16 && (act_dtype == EPQ_BF16 || act_dtype == EPQ_F16) &&
           (s.scale_dtype == EPQ_F16 || s.scale_dtype == EPQ_F32) && s.s_n == 1 && (s.s_g % 16) == 0 &&
           s.s_g >= s.rb * 16 && (reinterpret_cast<uintptr_t>(s.scale) % (16 * esz)) == 0 &&
           (reinterpret_cast<uintptr_t>(s.idx) & 15) == 0 && (reinterpret_cast<uintptr_t>(dy) & 15) == 0 &&
           ldy % 8 == 0 && s.n < (1 << 30) && s.k < (1 << 30) && s.ng <= 65535;
}

int launch_bwd_dx_tc(const StoreD& s, const void* dy, int64_t ldy, int act_dtype, int64_t m, void* dx,
                     int64_t lddx, int dx_dtype, cudaStream_t st) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return set_error(EPQ_EUNSUPPORTED, "device ordinal %d", dev);
    const int bn = m >= 256 ? 256 : (m > 64 ? 128 : 64);
    if (cdiv(m, bn) > 65535) return set_error(EPQ_EUNSUPPORTED, "linear_bwd: m too large");
    CUtensorMap ymap;
    int rc = make_tmap_2d(&ymap, dy, act_dtype, s.n, m, ldy, kRS, bn, "linear_bwd");
    if (rc) return rc;
    DxParams P{};
    P.idx = s.idx;
    P.scale = s.scale;
    P.s_g = s.s_g;
    P.cb = s.cb;
    P.dx = dx;
    P.lddx = lddx;
    P.cb_dtype = s.cb_dtype;
    P.scale_f32 = s.scale_dtype == EPQ_F32;
    P.levels = s.levels;
    P.n = (int)s.n;
    P.k = (int)s.k;
    P.ng = (int)s.ng;
    P.rb = (int)s.rb;
    P.m = (int)m;
    P.out_dtype = dx_dtype;
    const bool bf = act_dtype == EPQ_BF16;
    const bool mma16 = s.layout == EPQ_LAYOUT_MMA16;
    if (bf)
        return mma16 ? launch_dx_bn<true, EPQ_LAYOUT_MMA16>(bn, ymap, P, st, dev)
                     : launch_dx_bn<true, EPQ_LAYOUT_TILED>(bn, ymap, P, st, dev);
    return mma16 ? launch_dx_bn<false, EPQ_LAYOUT_MMA16>(bn, ymap, P, st, dev)
                 : launch_dx_bn<false, EPQ_LAYOUT_TILED>(bn, ymap, P, st, dev);
}

}  // namespace epq
