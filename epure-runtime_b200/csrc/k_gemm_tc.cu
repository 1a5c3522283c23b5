// Batched / prefill (M > 16) dequant-GEMM on the 5th-generation tensor cores:
// out[m, r] = sum_c x[m, c] W[r, c],  W[r, 4j+p] = cb[idx[r, j], p] * scale[r, g(j)].
//
// Reference op: epure/kernels/_triton.py:56-107 (_dequant_matmul: per K-tile the
// weight tile is gathered from the codebook, scaled, and fed to tl.dot) and the
// bf16 fallback of PackedLinear.forward, F.linear(x, materialize(bf16))
// (epure/runtime.py:78-89, 123-124).
//
// Design (B200, sm_100a):
// * One CTA computes a 128 (weight rows) x BN (activation rows) tile of out^T
//   with tcgen05.mma (cta_group::1, kind::f16): A = the dequantised weight tile
//   (M = 128) held in TENSOR MEMORY, B = the activation tile (N = BN) in shared
//   memory, D = fp32 in TMEM columns 0 .. BN-1.
// * Pipeline stages of 64 k (one 128-byte swizzle atom of 16-bit values):
//   - warp 0 (one thread) loads the activation tile with a 2-D TMA copy
//     (128-byte swizzle, rows past M zero-filled, this CTA only) into a ring of
//     up to 8 shared-memory stages;
//   - warps 2-9 decode the weight tile straight into TMEM: thread = one weight
//     row = one TMEM lane (warp w owns lanes 32 (w % 4) .. +31; two warps share
//     a lane quarter, each filling half of the stage's 32 columns).  Each index
//     byte gathers one 8-byte codebook entry (already converted to the
//     activation type) from a 16-way replicated codebook in shared memory
//     (lane l reads copy l % 16: no bank conflicts), is multiplied by the row's
//     group scale in the activation type -- exactly the reference's
//     cb.to(dtype)[idx] * scale.to(dtype) -- and lands in TMEM with
//     tcgen05.st.  Weight stages occupy TMEM columns 256 + 32 s;
//   - warp 1 (one thread) issues 4 MMAs (k = 16 each) per stage, A from TMEM,
//     and commits them to the stage's "empty" barrier, which frees both the
//     activation stage and the weight stage.
//   The dequantised weights never touch shared memory: the shared-memory port
//   carries only the activation tiles (read by the tensor core) and the
//   codebook gathers.
// * After the k loop warps 2-9 read the accumulator with tcgen05.ld (warp w:
//   32 weight rows, half of the activation columns) and write the output in
//   the requested dtype: per activation row, 32 consecutive outputs per warp.
// * Index layouts: EPQ_LAYOUT_MMA16 (per (16-row block, group) 512-byte tiles,
//   lane t = 4 (r % 8) + q holds rows r, r + 8 at positions q + 4 s: a row's
//   group is four 8-byte pieces) and EPQ_LAYOUT_TILED (per (group, 16-row
//   block) 32 positions x 16 rows: one byte per position).  Index bytes and
//   scales are loaded per row into registers, two or three groups ahead of use.
// * Every mbarrier wait is bounded; a wait that gives up sets a device error
//   flag and a CTA-wide abort word, the kernel runs to its end, and TMEM is
//   released only after the last commit has landed.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <climits>
#include <mutex>

#include "epq_common.cuh"
#include "epq_sm100.cuh"

namespace epq {
namespace {

using namespace sm100;

constexpr int kRows = 128;                 // weight rows per tile (UMMA M)
constexpr int kKStage = 64;                // k per pipeline stage
constexpr int kDecWarps = 8;               // decode + epilogue warps (one 16-row block each)
constexpr int kThreads = 64 + kDecWarps * 32;
constexpr int kReplicaBytes = 256 * 16 * 8;
constexpr int kMaxStages = 8;
constexpr int kAStageCols = kKStage / 2;     // TMEM columns of one weight stage (2 x 16 bit each)
constexpr uint32_t kACol0 = 256;             // weight stages live in TMEM columns 256 ..
constexpr uint32_t kTmemCols = 512;          // accumulator in 0 .. BN-1
static_assert(kACol0 + kMaxStages * kAStageCols <= kTmemCols, "TMEM columns");
constexpr int kSmemLimit = 232448;         // 227 KB per CTA
constexpr uint32_t kWaitLimit = 1u << 22;

__device__ int g_tc_wait_timeout = 0;

template <int BN>
struct Cfg {
    static constexpr int kXStage = BN * kKStage * 2;
    static constexpr int kStagesRaw = (kSmemLimit - 1024 - 256 - kReplicaBytes) / kXStage;
    static constexpr int kStages = kStagesRaw > kMaxStages ? kMaxStages : kStagesRaw;
    static constexpr int kXOff = kReplicaBytes;
    static constexpr int kBarOff = kXOff + kStages * kXStage;
    static constexpr int kSmem = 1024 + kBarOff + 256;
    static_assert(kStages >= 2, "stages");
    static_assert(kSmem <= kSmemLimit, "shared memory");
    static_assert(BN <= (int)kACol0, "accumulator columns");
};

struct TcStore {
    const uint8_t* idx;
    const void* scale;    // group-major: scale(r, g) at g * s_g + r
    int64_t s_g;
    const void* cb;
    void* out;
    int64_t ldo;
    int cb_dtype, scale_dtype, levels;
    int n, ng, rb;        // rows, groups, 16-row blocks
    int tile0;            // first global row tile of this store
};

struct TcParams {
    TcStore st[kLutMaxStores];
    int count, m, k, out_dtype;
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
template <bool kBf16, int kLayout, int BN>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ TcParams P) {
    using C = Cfg<BN>;
    constexpr int S_ = C::kStages;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t sbase = (raw + 1023u) & ~1023u;
    uint8_t* sgen = smem_raw + (sbase - raw);
    const uint32_t xst0 = sbase + C::kXOff;
    const uint32_t bar0 = sbase + C::kBarOff;
    auto full_x = [&](int s) { return bar0 + 8u * s; };
    auto full_w = [&](int s) { return bar0 + 64u + 8u * s; };
    auto empty = [&](int s) { return bar0 + 128u + 8u * s; };
    const uint32_t accum = bar0 + 192u;
    const uint32_t tslot = bar0 + 200u;
    volatile int* abortp = reinterpret_cast<volatile int*>(sgen + C::kBarOff + 204);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile = blockIdx.x;
    int si = 0;
    while (si + 1 < P.count && tile >= P.st[si + 1].tile0) ++si;
    const TcStore& S = P.st[si];
    const int rt = tile - S.tile0;       // 128-row tile within the store
    const int m0 = blockIdx.y * BN;
    const int nkb = P.k / kKStage;

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
    // Codebook -> 16 interleaved copies in the activation type: entries are converted
    // once into the first activation stage (free until the k loop starts), then fanned
    // out with consecutive lanes writing consecutive copies.
    uint2* conv = reinterpret_cast<uint2*>(sgen + C::kXOff);
    for (int e = threadIdx.x; e < 256; e += kThreads) {
        uint2 v = make_uint2(0u, 0u);
        if (e < S.levels) {
            const int64_t b = (int64_t)e * 4;
            v.x = pack2<kBf16>(load_f(S.cb, S.cb_dtype, b), load_f(S.cb, S.cb_dtype, b + 1));
            v.y = pack2<kBf16>(load_f(S.cb, S.cb_dtype, b + 2), load_f(S.cb, S.cb_dtype, b + 3));
        }
        conv[e] = v;
    }
    __syncthreads();
    for (int slot = threadIdx.x; slot < 256 * 16; slot += kThreads)
        reinterpret_cast<uint2*>(sgen)[slot] = conv[slot >> 4];
    // The activation stages are written by TMA (async proxy) after this point.
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(sgen + C::kBarOff + 200);

    if (warp == 0) {
        // ---------------- activation tiles (TMA) ----------------
        if (lane == 0) {
            tma_prefetch_desc(&xmap);
            int issued = 0;
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % S_;
                const uint32_t par = ((kb / S_) & 1) ^ 1;
                if (!mbar_wait_bounded(empty(s), par, abortp, &g_tc_wait_timeout, kWaitLimit)) break;
                mbar_expect_tx(full_x(s), C::kXStage);
                tma_load_2d(xst0 + s * C::kXStage, &xmap, full_x(s), kb * kKStage, m0);
                ++issued;
            }
            // Every copy issued must land before the CTA can exit.
            const int first = issued > S_ ? issued - S_ : 0;
            for (int kb = first; kb < issued; ++kb) {
                const int s = kb % S_;
                for (uint32_t i = 0; i < kWaitLimit; ++i)
                    if (mbar_try_wait(full_x(s), (kb / S_) & 1)) break;
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issue (one thread): A from TMEM, B from shared memory ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16<kBf16, kRows, BN>();
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % S_;
                const uint32_t par = (kb / S_) & 1;
                if (!mbar_wait_bounded(full_x(s), par, abortp, &g_tc_wait_timeout, kWaitLimit)) break;
                if (!mbar_wait_bounded(full_w(s), par, abortp, &g_tc_wait_timeout, kWaitLimit)) break;
                tc_fence_after();
                const uint32_t ta = tmem + kACol0 + s * kAStageCols;
                const uint64_t bd = desc_kmajor_sw128(xst0 + s * C::kXStage);
#pragma unroll
                for (int kk = 0; kk < kKStage / 16; ++kk)
                    mma_f16_ts(tmem, ta + 8 * kk, bd + 2 * kk, idesc, (kb | kk) != 0);
                mma_commit(empty(s));
            }
            mma_commit(accum);
            // The accumulator (and every MMA) is complete before TMEM can be released.
            for (uint32_t i = 0; i < kWaitLimit; ++i)
                if (mbar_try_wait(accum, 0)) break;
        }
        __syncwarp();
    } else {
        // ---------------- decode: thread = one weight row (TMEM lane) ----------------
        // Warp w owns TMEM lanes 32 (w % 4) .. +31; warps 2-5 fill the first half of each
        // stage's 16 index positions, warps 6-9 the second half (layout dependent split).
        const int sub = warp & 3, c2 = (warp - 2) >> 2;
        const uint32_t rep_lane = sbase + (lane & 15) * 8;
        const int rb = rt * 8 + 2 * sub + (lane >> 4);      // 16-row block of this row
        const int r16 = lane & 15;
        const bool ok = rb < S.rb;
        const int64_t row = (int64_t)rb * 16 + r16;
        const int ng = S.ng;
        const uint32_t trow = tmem + ((uint32_t)(32 * sub) << 16) + kACol0;
        int kb = 0;
        if constexpr (kLayout == EPQ_LAYOUT_MMA16) {
            // Row r's 32 positions of a group sit in four 8-byte pieces (lanes t = 4 (r%8) + q,
            // q = 0..3, half (r/8)%2); this warp takes q = 2 c2 and 2 c2 + 1: positions
            // q + 4 s, i.e. local positions {2 c2, 2 c2 + 1} + 4 s_l of each stage.
            const uint8_t* ip = S.idx + ((int64_t)rb * ng) * 512 + (4 * (r16 & 7) + 2 * c2) * 16 +
                                8 * ((r16 >> 3) & 1);
            uint2 a0{}, b0{}, a1{}, b1{}, a2{}, b2{};
            uint32_t s0 = 0, s1 = 0, s2 = 0;
            auto fetch = [&](int g, uint2& a, uint2& b, uint32_t& sc) {
                if (ok && g < ng) {
                    a = ldg_nc_v2(ip + (int64_t)g * 512);
                    b = ldg_nc_v2(ip + (int64_t)g * 512 + 16);
                    const float f = load_f(S.scale, S.scale_dtype, (int64_t)g * S.s_g + row);
                    sc = pack2<kBf16>(f, f);
                }
            };
            fetch(0, a0, b0, s0);
            fetch(1, a1, b1, s1);
            fetch(2, a2, b2, s2);
            for (int g = 0; g < ng; ++g) {
                const uint2 ca = a0, cbb = b0;
                const uint32_t cs = s0;
                a0 = a1; b0 = b1; s0 = s1;
                a1 = a2; b1 = b2; s1 = s2;
                fetch(g + 3, a2, b2, s2);
#pragma unroll
                for (int half = 0; half < 2; ++half, ++kb) {
                    const int s = kb % S_;
                    // tcgen05.st below is warp-collective: the whole warp continues or stops
                    const bool w_ok = mbar_wait_bounded(empty(s), ((kb / S_) & 1) ^ 1, abortp,
                                                        &g_tc_wait_timeout, kWaitLimit);
                    if (!__all_sync(0xffffffffu, w_ok)) break;
                    tc_fence_after();
                    const uint32_t wa = half ? ca.y : ca.x, wb = half ? cbb.y : cbb.x;
                    const uint32_t t0 = trow + s * kAStageCols + 4 * c2;
#pragma unroll
                    for (int sl = 0; sl < 4; ++sl) {
                        const uint2 va = lds64(rep_lane + ((wa >> (8 * sl)) & 0xFFu) * 128u);
                        const uint2 vb = lds64(rep_lane + ((wb >> (8 * sl)) & 0xFFu) * 128u);
                        tmem_st_32x32b_x4(t0 + 8 * sl, mul2<kBf16>(va.x, cs), mul2<kBf16>(va.y, cs),
                                          mul2<kBf16>(vb.x, cs), mul2<kBf16>(vb.y, cs));
                    }
                    tmem_st_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(full_w(s));
                }
                if (__any_sync(0xffffffffu, *abortp != 0)) break;
            }
        } else {
            // EPQ_LAYOUT_TILED: byte ((g RB + rb) 32 + p) 16 + r16; this warp takes local
            // positions 8 c2 .. 8 c2 + 7 of each stage (16 contiguous TMEM columns).
            const uint8_t* ip = S.idx + ((int64_t)rb * 32 + 8 * c2) * 16 + r16;
            const int64_t gstride = (int64_t)S.rb * 512;
            uint32_t w0[4] = {}, w1[4] = {};
            uint32_t s0 = 0, s1 = 0;
            auto fetch = [&](int g, uint32_t (&w)[4], uint32_t& sc) {
                if (ok && g < ng) {
                    const uint8_t* p = ip + g * gstride;
#pragma unroll
                    for (int hq = 0; hq < 4; ++hq) {   // (half, quad): positions 16 (hq/2) + 4 (hq%2) ..
                        const int p0 = 16 * (hq >> 1) + 4 * (hq & 1);
                        const uint32_t e0 = ldg_nc_u8(p + (p0 + 0) * 16), e1 = ldg_nc_u8(p + (p0 + 1) * 16);
                        const uint32_t e2 = ldg_nc_u8(p + (p0 + 2) * 16), e3 = ldg_nc_u8(p + (p0 + 3) * 16);
                        w[hq] = e0 | (e1 << 8) | (e2 << 16) | (e3 << 24);
                    }
                    const float f = load_f(S.scale, S.scale_dtype, (int64_t)g * S.s_g + row);
                    sc = pack2<kBf16>(f, f);
                }
            };
            fetch(0, w0, s0);
            fetch(1, w1, s1);
            for (int g = 0; g < ng; ++g) {
                uint32_t cw[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) cw[i] = w0[i];
                const uint32_t cs = s0;
#pragma unroll
                for (int i = 0; i < 4; ++i) w0[i] = w1[i];
                s0 = s1;
                fetch(g + 2, w1, s1);
#pragma unroll
                for (int half = 0; half < 2; ++half, ++kb) {
                    const int s = kb % S_;
                    // tcgen05.st below is warp-collective: the whole warp continues or stops
                    const bool w_ok = mbar_wait_bounded(empty(s), ((kb / S_) & 1) ^ 1, abortp,
                                                        &g_tc_wait_timeout, kWaitLimit);
                    if (!__all_sync(0xffffffffu, w_ok)) break;
                    tc_fence_after();
                    uint32_t v[16];
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const uint32_t w = cw[2 * half + (j >> 2)];
                        const uint2 e = lds64(rep_lane + ((w >> (8 * (j & 3))) & 0xFFu) * 128u);
                        v[2 * j] = mul2<kBf16>(e.x, cs);
                        v[2 * j + 1] = mul2<kBf16>(e.y, cs);
                    }
                    tmem_st_32x32b_x16(trow + s * kAStageCols + 16 * c2, v);
                    tmem_st_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(full_w(s));
                }
                if (__any_sync(0xffffffffu, *abortp != 0)) break;
            }
        }

        // ---------------- epilogue: TMEM -> out ----------------
        // Warp w reads TMEM lanes 32 (w % 4) .. +31 (32 weight rows); warps 2-5 take the
        // first half of the activation columns, warps 6-9 the second.
        const bool got = mbar_wait_bounded(accum, 0, abortp, &g_tc_wait_timeout, kWaitLimit);
        tc_fence_after();
        const int64_t r = (int64_t)rt * kRows + sub * 32 + lane;     // weight row = output column
        const bool rv = got && r < S.n;
#pragma unroll 1
        for (int cc = c2 * (BN / 64); cc < (c2 + 1) * (BN / 64); ++cc) {
            if (m0 + cc * 32 >= P.m) break;
            uint32_t v[32];
            tmem_ld_32x32b_x32(tmem + ((uint32_t)(sub * 32) << 16) + cc * 32, v);
            if (rv) {
#pragma unroll
                for (int q = 0; q < 32; ++q) {
                    const int mm = m0 + cc * 32 + q;
                    if (mm < P.m) store_f(S.out, P.out_dtype, (int64_t)mm * S.ldo + r, __uint_as_float(v[q]));
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

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

}  // namespace

// 2-D tensor map over a row-major [outer, inner] matrix of 16-bit elements with row
// stride `ld` (elements), box {box_inner, box_outer}, 128-byte swizzle, zero fill.
int make_tmap_2d(CUtensorMap* map, const void* base, int dtype, int64_t inner, int64_t outer,
                 int64_t ld, int box_inner, int box_outer, const char* who) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
    if (!enc) return set_error(EPQ_EUNSUPPORTED, "%s: cuTensorMapEncodeTiled unavailable", who);
    const cuuint64_t gdim[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    const cuuint64_t gstride[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult cr = enc(map, dtype == EPQ_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                  : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                            2, const_cast<void*>(base), gdim, gstride, box, estride,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return set_error(EPQ_EINVAL, "%s: tensor map (error %d)", who, (int)cr);
    return EPQ_OK;
}

// 2-D tensor map without swizzle over `outer` rows of `inner` elements of
// `elem_bytes` (2 or 4) with a row stride of `ld` elements; box {box_inner,
// box_outer}; out-of-range boxes are zero-filled.
int make_tmap_2d_plain(CUtensorMap* map, const void* base, int elem_bytes, int64_t inner, int64_t outer,
                       int64_t ld, int box_inner, int box_outer, const char* who) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = encode_fn();
    if (!enc) return set_error(EPQ_EUNSUPPORTED, "%s: cuTensorMapEncodeTiled unavailable", who);
    const cuuint64_t gdim[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    const cuuint64_t gstride[1] = {(cuuint64_t)(ld * elem_bytes)};
    const cuuint32_t box[2] = {(cuuint32_t)box_inner, (cuuint32_t)box_outer};
    const cuuint32_t estride[2] = {1, 1};
    const CUresult cr = enc(map, elem_bytes == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT16,
                            2, const_cast<void*>(base), gdim, gstride, box, estride,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return set_error(EPQ_EINVAL, "%s: tensor map (error %d)", who, (int)cr);
    return EPQ_OK;
}

namespace {


template <bool kBf16, int kLayout, int BN>
int launch_tc(const CUtensorMap& xmap, const TcParams& P, int tiles, int bi, cudaStream_t st,
              int dev) {
    using C = Cfg<BN>;
    auto kern = gemm_tc_kernel<kBf16, kLayout, BN>;
    (void)bi;
    (void)dev;
    const int arc = set_smem_limit(reinterpret_cast<const void*>(kern), C::kSmem, "cudaFuncSetAttribute(gemm_tc_kernel)");
    if (arc != EPQ_OK) return arc;
    const dim3 grid(tiles, (unsigned)cdiv(P.m, BN));
    kern<<<grid, kThreads, C::kSmem, st>>>(xmap, P);
    return check_launch("gemm_tc_kernel");
}

template <bool kBf16, int kLayout>
int launch_bn(int bn, const CUtensorMap& xmap, const TcParams& P, int tiles, cudaStream_t st,
              int dev) {
    if (bn == 256) return launch_tc<kBf16, kLayout, 256>(xmap, P, tiles, 2, st, dev);
    if (bn == 128) return launch_tc<kBf16, kLayout, 128>(xmap, P, tiles, 1, st, dev);
    return launch_tc<kBf16, kLayout, 64>(xmap, P, tiles, 0, st, dev);
}

}  // namespace

int tc_read_device_error(int* flag) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_tc_wait_timeout, sizeof(int)) != cudaSuccess)
        return check_launch("epq_device_error");
    *flag = v;
    return EPQ_OK;
}

bool tc_eligible(const StoreD& s, int64_t m, int x_dtype) {
    const int64_t esz = s.scale_dtype == EPQ_F32 ? 4 : 2;
    return (s.layout == EPQ_LAYOUT_MMA16 || s.layout == EPQ_LAYOUT_TILED) && s.bits == 8 &&
           s.vec == 4 && s.group == 128 && s.levels <= 256 && s.p == 32 && m > 16 &&
           (x_dtype == EPQ_BF16 || x_dtype == EPQ_F16) &&
           (s.scale_dtype == EPQ_F16 || s.scale_dtype == EPQ_F32) && s.s_n == 1 &&
           (s.s_g % 16) == 0 && s.s_g >= s.rb * 16 &&
           (reinterpret_cast<uintptr_t>(s.scale) % (16 * esz)) == 0 &&
           (reinterpret_cast<uintptr_t>(s.idx) & 15) == 0 && s.k % 128 == 0 && s.n > 0 &&
           s.n < (1 << 30) && s.k > 0 && s.k < (1 << 30);
}

int launch_linear_tc(const StoreD* s, int count, const void* x, int x_dtype, int64_t m, int64_t ldx,
                     void* const* outs, const int64_t* ldo, int out_dtype, cudaStream_t st) {
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx % 8))
        return set_error(EPQ_EALIGN, "linear: x must be 16-byte aligned with ldx a multiple of 8");
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return set_error(EPQ_EUNSUPPORTED, "device ordinal %d", dev);
    for (int i = 1; i < count; ++i)
        if (s[i].layout != s[0].layout)
            return set_error(EPQ_ELAYOUT, "linear: fused stores need one layout");
    const int bn = m >= 256 ? 256 : (m > 64 ? 128 : 64);
    if (cdiv(m, bn) > 65535) return set_error(EPQ_EUNSUPPORTED, "linear: m too large");

    TcParams P{};
    P.count = count;
    P.m = (int)m;
    P.k = (int)s[0].k;
    P.out_dtype = out_dtype;
    int64_t tiles = 0;
    for (int i = 0; i < count; ++i) {
        TcStore& S = P.st[i];
        S.idx = s[i].idx;
        S.scale = s[i].scale;
        S.s_g = s[i].s_g;
        S.cb = s[i].cb;
        S.out = outs[i];
        S.ldo = ldo ? ldo[i] : s[i].n;
        S.cb_dtype = s[i].cb_dtype;
        S.scale_dtype = s[i].scale_dtype;
        S.levels = s[i].levels;
        S.n = (int)s[i].n;
        S.ng = (int)s[i].ng;
        S.rb = (int)s[i].rb;
        S.tile0 = (int)tiles;
        tiles += cdiv(s[i].n, kRows);
    }
    if (tiles >= (int64_t(1) << 31) - 1) return set_error(EPQ_EUNSUPPORTED, "linear: too many rows");

    CUtensorMap xmap;
    const int trc = make_tmap_2d(&xmap, x, x_dtype, P.k, m, ldx, kKStage, bn, "linear");
    if (trc) return trc;

    const bool bf = x_dtype == EPQ_BF16;
    const bool mma16 = s[0].layout == EPQ_LAYOUT_MMA16;
    if (bf) {
        return mma16 ? launch_bn<true, EPQ_LAYOUT_MMA16>(bn, xmap, P, (int)tiles, st, dev)
                     : launch_bn<true, EPQ_LAYOUT_TILED>(bn, xmap, P, (int)tiles, st, dev);
    }
    return mma16 ? launch_bn<false, EPQ_LAYOUT_MMA16>(bn, xmap, P, (int)tiles, st, dev)
                 : launch_bn<false, EPQ_LAYOUT_TILED>(bn, xmap, P, (int)tiles, st, dev);
}

}  // namespace epq
