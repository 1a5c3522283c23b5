// Small-batch (M <= 16) dequant-GEMV for 4-weight vector codebooks on the
// tensor cores: out[m, r] = sum_c x[m, c] W[r, c],
// W[r, 4j+p] = cb[idx[r, j], p] * scale[r, g(j)].
//
// Reference op: epure/kernels/_triton.py:56-107 (_dequant_matmul, table mode):
// gather cb[idx] per weight, multiply by the group scale, tl.dot with x.
//
// Design (B200, sm_100a).  The op is HBM-bound (1 index byte per 4 weights),
// so everything is built around a cheap gather per index byte and a low
// instruction count per byte:
// * mma.m16n8k16 with A = 16 dequantised weight rows x 16 k and B = the
//   activations (8 columns = 8 activation rows; two MMAs when M > 8).  The k
//   axis is permuted so that the four k slots a thread holds for one A row
//   ({2q, 2q+1, 2q+8, 2q+9}) are the four weights of ONE codebook vector: a
//   thread's A fragment for a row is exactly one 8-byte codebook entry, one
//   64-bit shared load.  B is permuted the same way, so a thread's B fragment
//   is 4 consecutive activations (one 64-bit load).
// * The codebook is replicated 16 times in shared memory (copy c in bank pair
//   c) and lane l reads copy l % 16, so the random gathers of a half-warp never
//   share a bank.  Codebook values are converted to the activation type
//   (cb.to(dtype), as the reference's bf16 path does); the group scale
//   multiplies the fp32 accumulator, once per row per group.
// * Index layout EPQ_LAYOUT_MMA16: per (16-row block, group) a 512-byte tile;
//   lane 4*r + q holds the indices of rows r and r + 8 at positions q + 4s,
//   s = 0..7.  Tiles run group-fastest, so the 32 groups of one 16-row block
//   ("chunk") are one contiguous 16 KB run.
// * A producer warp streams chunks with TMA bulk copies (cp.async.bulk, into this
//   CTA's shared memory only) into a 4-stage shared-memory ring guarded by mbarriers: one
//   16 KB copy for the indices and one 32/64-byte copy per group for the
//   scales (stored group-major, rows padded to 16).  16 consumer warps each
//   take two tiles of a chunk; per tile a lane does 16 gathers (PRMT + IMAD +
//   LDS.64), 8 MMAs and 8 activation loads from shared memory.
// * Full rows per CTA, no split over k between CTAs: one CTA per SM owns a
//   contiguous range of 16-row blocks; per block the consumer warps' sums are
//   added in warp order through shared memory (deterministic).  No workspace,
//   no atomics.  With programmatic dependent launch the producer starts
//   streaming weights before the previous kernel (which produces x) finishes.
// * Every mbarrier wait is bounded; a wait that gives up sets a device error
//   flag (read by epq_device_error) and the kernel runs to completion.
#include <climits>

#include "epq_common.cuh"

namespace epq {
namespace {

constexpr int kConsumerWarps = 16;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;       // + one producer warp
constexpr int kStages = 4;
constexpr int kChunkGroups = 32;                // groups per chunk
constexpr int kStageIdx = kChunkGroups * 512;   // 16 KB of index tiles
constexpr int kStageBytes = kStageIdx + kChunkGroups * 64;
constexpr int kReplicaBytes = 256 * 16 * 8;     // 256 entries x 16 copies x 8 B
constexpr int kRedFloats = kConsumerWarps * 16 * 16;   // [warp][16 rows][16 m]
constexpr int kBarOffset = kReplicaBytes + 2 * kRedFloats * 4;
constexpr int kStageOffset = kBarOffset + 128;
constexpr int kFixedSmem = kStageOffset + kStages * kStageBytes;
constexpr int kMaxXSmem = 64 * 1024;            // activations staged in shared memory up to this
constexpr uint32_t kWaitLimit = 1u << 22;       // bounded mbarrier waits

__device__ int g_mma_wait_timeout = 0;

struct MmaStore {
    const uint8_t* idx;   // EPQ_LAYOUT_MMA16
    const void* scale;    // group-major: scale(r, g) at g * s_g + r; s_g % 16 == 0
    int64_t s_g;
    const void* cb;
    void* out;
    int64_t ldo;
    int cb_dtype, levels;
    int n, ng, rb;
    int unit0;            // first global unit (16-row block) of this store
};

struct MmaParams {
    MmaStore st[kLutMaxStores];
    const void* x;
    int64_t ldx;
    int count, m, k, kpad, out_dtype;
    int total_units, chunks_per_unit;
};

template <bool kBf16>
__device__ __forceinline__ uint32_t cvt_pair(float a, float b) {
    if constexpr (kBf16) {
        __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    } else {
        __half2 v = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&v);
    }
}

template <bool kBf16>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    if constexpr (kBf16) {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
            "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    } else {
        asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
            "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr));
    return v;
}
template <bool kF32>
__device__ __forceinline__ float lds_scale(uint32_t addr) {
    if constexpr (kF32) {
        float v;
        asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
        return v;
    } else {
        unsigned short h;
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(addr));
        return __half2float(__ushort_as_half(h));
    }
}

// --- mbarrier / bulk copy -----------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Waits for the phase with the given parity; gives up after kWaitLimit polls.
__device__ __forceinline__ void mbar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, parity)) return;
    atomicExch(&g_mma_wait_timeout, 1);
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Codebook of store S -> 16 interleaved copies in the activation type (consumer threads).
template <bool kBf16>
__device__ void build_replica(const MmaStore& S, uint2* rep) {
    for (int slot = threadIdx.x; slot < 256 * 16; slot += kConsumers) {
        const int e = slot >> 4;
        uint2 v = make_uint2(0u, 0u);
        if (e < S.levels) {
            const int64_t b = (int64_t)e * 4;
            v.x = cvt_pair<kBf16>(load_f(S.cb, S.cb_dtype, b), load_f(S.cb, S.cb_dtype, b + 1));
            v.y = cvt_pair<kBf16>(load_f(S.cb, S.cb_dtype, b + 2), load_f(S.cb, S.cb_dtype, b + 3));
        }
        rep[slot] = v;
    }
}

__device__ __forceinline__ int store_of(const MmaParams& P, int u) {
    int si = 0;
    while (si + 1 < P.count && u >= P.st[si + 1].unit0) ++si;
    return si;
}

template <bool kBf16, int kNT, bool kScaleF32, bool kXSmem>
__global__ void __launch_bounds__(kThreads, 1) gemv_mma_kernel(const __grid_constant__ MmaParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint2* rep = reinterpret_cast<uint2*>(smem);
    float* red = reinterpret_cast<float*>(smem + kReplicaBytes);   // [2][warp][16 rows][16 m]
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    const uint32_t bar_full = sbase + kBarOffset;          // kStages x 8 B
    const uint32_t bar_empty = bar_full + 8 * kStages;     // kStages x 8 B
    const uint32_t stage0 = sbase + kStageOffset;
    uint16_t* xs = reinterpret_cast<uint16_t*>(smem + kFixedSmem);   // [m][kpad] when kXSmem
    constexpr int kScaleBytes = kScaleF32 ? 4 : 2;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // Contiguous, balanced range of units (16-row blocks) for this CTA.
    const int U = P.total_units, G = gridDim.x;
    const int u_begin = (int)((int64_t)U * blockIdx.x / G);
    const int u_end = (int)((int64_t)U * (blockIdx.x + 1) / G);
    const int cpu = P.chunks_per_unit;
    const int n_chunks = (u_end - u_begin) * cpu;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, kConsumerWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ---------------- producer: stream chunks into the ring ----------------
        int si = store_of(P, u_begin);
        int s_next = si + 1 < P.count ? P.st[si + 1].unit0 : INT_MAX;
        int u = u_begin, c = 0;
        for (int i = 0; i < n_chunks; ++i) {
            const int stage = i % kStages;
            if (i >= kStages) mbar_wait(bar_empty + 8 * stage, ((i / kStages) - 1) & 1);
            if (u >= s_next) {
                si = store_of(P, u);
                s_next = si + 1 < P.count ? P.st[si + 1].unit0 : INT_MAX;
            }
            const MmaStore& S = P.st[si];
            const int rb = u - S.unit0;
            const int g0 = c * kChunkGroups;
            const int ngc = min(kChunkGroups, S.ng - g0);
            const uint32_t dst = stage0 + stage * kStageBytes;
            const uint32_t sb = 16 * kScaleBytes;   // one group's 16 scales
            if (lane == 0) mbar_expect_tx(bar_full + 8 * stage, ngc * (512 + sb));
            __syncwarp();
            if (lane == 0)
                bulk_g2s(dst, S.idx + ((int64_t)rb * S.ng + g0) * 512, ngc * 512, bar_full + 8 * stage);
            if (lane < ngc) {
                const char* src = static_cast<const char*>(S.scale) +
                                  ((int64_t)(g0 + lane) * S.s_g + (int64_t)rb * 16) * kScaleBytes;
                bulk_g2s(dst + kStageIdx + lane * 64, src, sb, bar_full + 8 * stage);
            }
            if (++c == cpu) {
                c = 0;
                ++u;
            }
        }
        pdl_trigger();
        return;
    }

    // ---------------- consumers ----------------
    const int gq = lane >> 2, q = lane & 3;
    int cur = store_of(P, u_begin);
    int c_next = cur + 1 < P.count ? P.st[cur + 1].unit0 : INT_MAX;
    if (u_begin < u_end) {
        if constexpr (kBf16) build_replica<true>(P.st[cur], rep);
        else build_replica<false>(P.st[cur], rep);
    }
    pdl_trigger();
    pdl_wait();   // x (and the output buffers) belong to the previous kernel until here

    // Activation B fragments: lane (gq, q) supplies column gq = activation row
    // min(gq, m - 1) (columns >= m are computed and never stored).
    const int xr0 = gq < P.m ? gq : P.m - 1;
    const int xr1 = gq + 8 < P.m ? gq + 8 : P.m - 1;
    const uint16_t* xg0 = static_cast<const uint16_t*>(P.x) + (int64_t)xr0 * P.ldx + 4 * q;
    const uint16_t* xg1 = static_cast<const uint16_t*>(P.x) + (int64_t)xr1 * P.ldx + 4 * q;
    uint32_t xs0 = 0, xs1 = 0;
    if constexpr (kXSmem) {
        const int per_row = P.kpad >> 2;
        const int chunks = P.m * per_row;
        for (int i = threadIdx.x; i < chunks; i += kConsumers) {
            const int row = i / per_row, c4 = (i - row * per_row) * 4;
            uint2 v = make_uint2(0u, 0u);
            if (c4 < P.k)
                v = *reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(P.x) + (int64_t)row * P.ldx + c4);
            *reinterpret_cast<uint2*>(xs + row * P.kpad + c4) = v;
        }
        const uint32_t xsb = static_cast<uint32_t>(__cvta_generic_to_shared(xs));
        xs0 = xsb + (xr0 * P.kpad + 4 * q) * 2;
        xs1 = xsb + (xr1 * P.kpad + 4 * q) * 2;
    }
    consumers_sync();

    const uint32_t rep_lane = sbase + (lane & 15) * 8;
    const int k_lane = P.k - 4 * q;   // global-load path: column c is in range iff c < k_lane
    float acc[kNT][4];
#pragma unroll
    for (int h = 0; h < kNT; ++h) acc[h][0] = acc[h][1] = acc[h][2] = acc[h][3] = 0.f;
    int parity = 0;
    int u = u_begin, c = 0;
    for (int i = 0; i < n_chunks; ++i) {
        const int stage = i % kStages;
        if (c == 0 && u >= c_next) {
            // New store (CTA-uniform): rebuild the codebook replica.
            consumers_sync();
            cur = store_of(P, u);
            c_next = cur + 1 < P.count ? P.st[cur + 1].unit0 : INT_MAX;
            if constexpr (kBf16) build_replica<true>(P.st[cur], rep);
            else build_replica<false>(P.st[cur], rep);
            consumers_sync();
        }
        const int ng = P.st[cur].ng;
        const int g0 = c * kChunkGroups;
        const int ngc = min(kChunkGroups, ng - g0);
        mbar_wait(bar_full + 8 * stage, (i / kStages) & 1);
        const uint32_t sdst = stage0 + stage * kStageBytes;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
            const int gl = warp + kConsumerWarps * t;   // group within the chunk
            if (gl < ngc) {
                const uint4 w = lds128(sdst + gl * 512 + lane * 16);
                const float s0 = lds_scale<kScaleF32>(sdst + kStageIdx + gl * 64 + gq * kScaleBytes);
                const float s1 = lds_scale<kScaleF32>(sdst + kStageIdx + gl * 64 + (gq + 8) * kScaleBytes);
                float d[2][kNT][4];
#pragma unroll
                for (int e = 0; e < 2; ++e)
#pragma unroll
                    for (int h = 0; h < kNT; ++h) d[e][h][0] = d[e][h][1] = d[e][h][2] = d[e][h][3] = 0.f;
                const int cbase = (g0 + gl) * 128;
                const uint32_t wlo[2] = {w.x, w.y}, whi[2] = {w.z, w.w};
#pragma unroll
                for (int s = 0; s < 8; ++s) {
                    const int col = cbase + 16 * s;
                    const uint32_t sel = 0x4440u | (s & 3);
                    const uint32_t elo = __byte_perm(wlo[s >> 2], 0u, sel);
                    const uint32_t ehi = __byte_perm(whi[s >> 2], 0u, sel);
                    const uint2 alo = lds64(rep_lane + elo * 128u);
                    const uint2 ahi = lds64(rep_lane + ehi * 128u);
                    uint2 bx, by;
                    if constexpr (kXSmem) {
                        bx = lds64(xs0 + col * 2);
                        if constexpr (kNT == 2) by = lds64(xs1 + col * 2);
                    } else {
                        bx = col < k_lane ? __ldg(reinterpret_cast<const uint2*>(xg0 + col)) : make_uint2(0u, 0u);
                        if constexpr (kNT == 2)
                            by = col < k_lane ? __ldg(reinterpret_cast<const uint2*>(xg1 + col)) : make_uint2(0u, 0u);
                    }
                    mma16816<kBf16>(d[s & 1][0], alo.x, ahi.x, alo.y, ahi.y, bx.x, bx.y);
                    if constexpr (kNT == 2) mma16816<kBf16>(d[s & 1][1], alo.x, ahi.x, alo.y, ahi.y, by.x, by.y);
                }
#pragma unroll
                for (int h = 0; h < kNT; ++h) {
                    acc[h][0] = fmaf(d[0][h][0] + d[1][h][0], s0, acc[h][0]);
                    acc[h][1] = fmaf(d[0][h][1] + d[1][h][1], s0, acc[h][1]);
                    acc[h][2] = fmaf(d[0][h][2] + d[1][h][2], s1, acc[h][2]);
                    acc[h][3] = fmaf(d[0][h][3] + d[1][h][3], s1, acc[h][3]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_empty + 8 * stage);   // this warp is done with the stage
        if (++c == cpu) {
            // End of a 16-row block: add the warps' sums in warp order, write 16 rows.
            const MmaStore& S = P.st[cur];
            float* rb_buf = red + parity * kRedFloats;
            float* mine = rb_buf + warp * 256;     // [16 rows][16 m]
#pragma unroll
            for (int h = 0; h < kNT; ++h) {
                const int m0 = 8 * h + 2 * q;
                mine[gq * 16 + m0] = acc[h][0];
                mine[gq * 16 + m0 + 1] = acc[h][1];
                mine[(gq + 8) * 16 + m0] = acc[h][2];
                mine[(gq + 8) * 16 + m0 + 1] = acc[h][3];
                acc[h][0] = acc[h][1] = acc[h][2] = acc[h][3] = 0.f;
            }
            consumers_sync();
            if (threadIdx.x < 256) {
                const int mm = threadIdx.x >> 4, rr = threadIdx.x & 15;   // 16 x 16
                const int row = (u - S.unit0) * 16 + rr;
                if (mm < P.m && row < S.n) {
                    float sum = 0.f;
#pragma unroll
                    for (int ww = 0; ww < kConsumerWarps; ++ww) sum += rb_buf[ww * 256 + rr * 16 + mm];
                    store_f(S.out, P.out_dtype, mm * S.ldo + row, sum);
                }
            }
            parity ^= 1;
            c = 0;
            ++u;
        }
    }
}

int g_sms[64] = {0};
bool g_attr[16][64] = {{false}};

int sm_count(int dev) {
    if (g_sms[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
            v = 148;
        g_sms[dev] = v;
    }
    return g_sms[dev];
}

}  // namespace

int mma_read_device_error(int* flag) {
    if (cudaMemcpyFromSymbol(flag, g_mma_wait_timeout, sizeof(int)) != cudaSuccess)
        return check_launch("read gemv_mma error flag");
    return EPQ_OK;
}

bool mma_eligible(const StoreD& s, int64_t m, int x_dtype) {
    const int64_t esz = s.scale_dtype == EPQ_F32 ? 4 : 2;
    return s.layout == EPQ_LAYOUT_MMA16 && s.bits == 8 && s.vec == 4 && s.group == 128 &&
           s.levels <= 256 && m >= 1 && m <= 16 && (x_dtype == EPQ_BF16 || x_dtype == EPQ_F16) &&
           (s.scale_dtype == EPQ_F16 || s.scale_dtype == EPQ_F32) && s.s_n == 1 &&
           (s.s_g % 16) == 0 && s.s_g >= s.rb * 16 &&
           (reinterpret_cast<uintptr_t>(s.scale) % (16 * esz)) == 0 &&
           (reinterpret_cast<uintptr_t>(s.idx) & 15) == 0 && s.n > 0 && s.n < (1 << 30) &&
           s.k > 0 && s.k < (1 << 30);
}

int launch_linear_mma(const StoreD* s, int count, const void* x, int x_dtype, int64_t m, int64_t ldx,
                      void* const* outs, const int64_t* ldo, int out_dtype, cudaStream_t st) {
    if ((reinterpret_cast<uintptr_t>(x) & 7) || (ldx & 3))
        return set_error(EPQ_EALIGN, "linear: x must be 8-byte aligned with ldx a multiple of 4");
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return set_error(EPQ_EUNSUPPORTED, "device ordinal %d", dev);
    const bool bf = x_dtype == EPQ_BF16;
    const int nt = m > 8 ? 2 : 1;
    const bool sf32 = s[0].scale_dtype == EPQ_F32;
    for (int i = 1; i < count; ++i)
        if ((s[i].scale_dtype == EPQ_F32) != sf32)
            return set_error(EPQ_EDTYPE, "linear: fused stores need one scale dtype");
    const int64_t kpad = s[0].ng * 128;
    const int64_t xbytes = m * kpad * 2;
    const bool xsm = xbytes <= kMaxXSmem;
    const int smem = kFixedSmem + (xsm ? (int)xbytes : 0);
    const int variant = (bf ? 1 : 0) + (nt == 2 ? 2 : 0) + (sf32 ? 4 : 0) + (xsm ? 8 : 0);
    using KernT = void (*)(MmaParams);
    static const KernT kernels[16] = {
        gemv_mma_kernel<false, 1, false, false>, gemv_mma_kernel<true, 1, false, false>,
        gemv_mma_kernel<false, 2, false, false>, gemv_mma_kernel<true, 2, false, false>,
        gemv_mma_kernel<false, 1, true, false>,  gemv_mma_kernel<true, 1, true, false>,
        gemv_mma_kernel<false, 2, true, false>,  gemv_mma_kernel<true, 2, true, false>,
        gemv_mma_kernel<false, 1, false, true>,  gemv_mma_kernel<true, 1, false, true>,
        gemv_mma_kernel<false, 2, false, true>,  gemv_mma_kernel<true, 2, false, true>,
        gemv_mma_kernel<false, 1, true, true>,   gemv_mma_kernel<true, 1, true, true>,
        gemv_mma_kernel<false, 2, true, true>,   gemv_mma_kernel<true, 2, true, true>};
    const KernT kern = kernels[variant];
    if (!g_attr[variant][dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 kFixedSmem + kMaxXSmem) != cudaSuccess)
            return check_launch("cudaFuncSetAttribute(gemv_mma_kernel)");
        g_attr[variant][dev] = true;
    }
    MmaParams P{};
    P.count = count;
    P.x = x;
    P.ldx = ldx;
    P.m = (int)m;
    P.k = (int)s[0].k;
    P.kpad = (int)kpad;
    P.out_dtype = out_dtype;
    P.chunks_per_unit = (int)cdiv(s[0].ng, kChunkGroups);
    int64_t units = 0;
    for (int i = 0; i < count; ++i) {
        MmaStore& S = P.st[i];
        S.idx = s[i].idx;
        S.scale = s[i].scale;
        S.s_g = s[i].s_g;
        S.cb = s[i].cb;
        S.out = outs[i];
        S.ldo = ldo ? ldo[i] : s[i].n;
        S.cb_dtype = s[i].cb_dtype;
        S.levels = s[i].levels;
        S.n = (int)s[i].n;
        S.ng = (int)s[i].ng;
        S.rb = (int)s[i].rb;
        S.unit0 = (int)units;
        units += S.rb;
    }
    if (units >= (int64_t(1) << 30)) return set_error(EPQ_EUNSUPPORTED, "linear: too many rows");
    P.total_units = (int)units;
    int grid = sm_count(dev);
    if (grid > units) grid = (int)units;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, P) != cudaSuccess) return check_launch("gemv_mma_kernel");
    return check_launch("gemv_mma_kernel");
}

}  // namespace epq
