// Small-batch (M <= 16) dequant-GEMV for 4-weight vector codebooks on the
// tensor cores: out[m, r] = sum_c x[m, c] W[r, c],
// W[r, 4j+p] = cb[idx[r, j], p] * scale[r, g(j)].
//
// Reference op: epure/kernels/_triton.py:56-107 (_dequant_matmul, table mode):
// gather cb[idx] per weight, multiply by the group scale, tl.dot with x.  The
// weight it contracts is the reference's own, rounded as the bf16 / fp16 path
// rounds it (epure/runtime.py:78-89, PackedWeight.materialize):
//     W = dtype( dtype(cb[idx]) * dtype(scale) )
// i.e. the codebook and the scale are each rounded to the activation type and
// their product is rounded once more.  This kernel forms exactly that value
// for every weight (a bf16x2 / f16x2 multiply of the gathered codebook pair by
// the row's rounded scale), so its only difference from the reference's
// F.linear(x, materialize(dtype)) is the fp32 summation order.
//
// Design (B200, sm_100a).  The op is HBM-bound (1 index byte per 4 weights),
// and at batch 1 the binding on-chip resource is the shared-memory gather of
// the codebook (8 bytes per index byte), so everything is built around one
// conflict-free 64-bit gather per index and a short instruction stream:
// * mma.m16n8k16 with A = 16 decoded weight rows x 16 k and B = the
//   activations (8 columns = 8 activation rows; two MMAs when M > 8).  The k
//   axis is permuted so that the four k slots a thread holds for one A row
//   ({2q, 2q+1, 2q+8, 2q+9}) are the four weights of ONE codebook vector: a
//   thread's A fragment for a row is one 8-byte codebook entry (one 64-bit
//   shared load) times the row's scale (two packed multiplies).
// * The codebook is replicated 16 times in shared memory at a 64 KiB-aligned
//   window address (entry e, copy c at e * 256 + c * 8; the other half of each
//   256-byte row holds the second store of a paired launch) and lane l reads
//   copy l % 16: one byte permute forms the gather's whole address, and a
//   half-warp's random gathers never share a bank pair.
// * Activations are staged in shared memory in the B-fragment order of two
//   consecutive k-steps per 16-byte word: one 128-bit load feeds two MMAs, and
//   the four lanes of a row read one contiguous 64-byte run (no conflicts).
// * Index layout EPQ_LAYOUT_MMA16: per (16-row block, group) a 512-byte tile;
//   lane 4*r + q holds the indices of rows r and r + 8 at positions q + 4s,
//   s = 0..7.  Tiles run group-fastest, so the groups of one 16-row block are
//   one contiguous run.
// * A producer warp streams 32-group chunks through a 3-stage shared-memory
//   ring guarded by mbarriers, two copies per chunk into this CTA's shared
//   memory only: the index tiles (cp.async.bulk, one contiguous run) and the
//   chunk's 16 x 32 scales (one 2-D cp.async.bulk.tensor box over the
//   group-major scales), both with an evict-first L2 policy (the weights are
//   read once per call).  16 consumer warps each take two tiles of a chunk,
//   interleaved so their gathers and MMAs overlap.
// * Full rows per CTA (no split over k between CTAs): one CTA per SM owns a
//   contiguous range of 16-row blocks ("units").  At the end of a unit every
//   consumer warp drops its partial sums into one of kSlots shared-memory slots
//   and arrives on the slot's mbarrier; a dedicated reducer warp adds the 16
//   warps' sums in warp order (deterministic), runs the epilogue and frees the
//   slot.  No CTA-wide barrier per unit and no consumer warp held up by a
//   reduction, so warps run ahead by up to the ring depth.
// * Fused decode glue (epq_decode_linear): the prologue can replace x by
//   RMSNorm(x) (weight 1) while staging it, the epilogue can add the result
//   into a residual stream in place (h = h + dtype(out)), and a paired launch
//   of two stores (gate, up) can emit dtype(silu(dtype(g)) * dtype(u)) -- the
//   Llama / Qwen3 block's rounding points, so a decode token needs five
//   launches per layer.
// * With programmatic dependent launch the producer starts streaming weights
//   before the previous kernel (which produces x) finishes.
// * Every mbarrier wait is bounded; a wait that gives up sets a device error
//   flag (read by epq_device_error) and the kernel runs to completion.
#include <algorithm>
#include <climits>
#include <new>
#include <vector>

#include "epq_common.cuh"
#include "epq_decode.h"
#include "epq_rope.cuh"
#include "epq_sm100.cuh"

namespace epq {
namespace {

constexpr int kConsumerWarps = 16;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kProducerWarp = kConsumerWarps;   // streams the ring
constexpr int kReducerWarp = kConsumerWarps + 1; // sums finished units and runs the epilogue
constexpr int kThreads = kConsumers + 64;
constexpr int kStages = 3;
constexpr int kSlots = kStages + 1;             // unit reduction slots (see the ring argument below)
constexpr int kChunkGroups = 32;                // groups per chunk
constexpr int kTileSets = kChunkGroups / kConsumerWarps;   // tiles a consumer warp takes per chunk
static_assert(kTileSets * kConsumerWarps == kChunkGroups, "consumer warps must divide a chunk");
constexpr int kStageIdx = kChunkGroups * 512;   // 16 KB of index tiles
constexpr int kStageBytes = kStageIdx + kChunkGroups * 64;
constexpr int kBarBytes = 256;                  // ring and slot mbarriers
constexpr int kCbStageBytes = 2048;             // codebook staging for the replica build / RMSNorm scratch
constexpr int kMaxXSmem = 64 * 1024;            // activations staged in shared memory up to this
constexpr int kMaxSmem = 227 * 1024;
// Shared-window layout.  The dynamic block starts at a small window address
// `base`; the codebook replicas sit at the fixed, 64 KiB-aligned window range
// [kRepWin, 2 kRepWin): entry e occupies bytes e * 256 + [0, 256), the first
// 128 the 16 copies of store part 0 (8 B each), the next 128 those of part 1.
// Because the low 16 bits of kRepWin are zero, one byte permute of an index
// word and a per-lane constant yields a gather's whole window address.  Below
// it: mbarriers + counters, then the stage ring (so base + kLowBytes <=
// kRepWin); above it: the reduction slots, then the staged activations.
constexpr uint32_t kRepWin = 65536;
constexpr uint32_t kLowBytes = kBarBytes + kStages * kStageBytes + kCbStageBytes;
constexpr uint32_t kHighWin = 2 * kRepWin;
constexpr uint32_t kWaitLimit = 1u << 22;       // bounded mbarrier waits

__device__ int g_mma_wait_timeout = 0;

struct MmaStore {
    CUtensorMap smap;     // the scales as a [groups][rows] tensor, box {16 rows, 32 groups}
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
    int parts;            // 2: each unit is the same block of stores 0 and 1 (SiLU pair), else 1
    int prologue, epilogue;
    float eps;
    int slot_floats;      // floats of one reduction slot: parts * warps * 16 rows * m
    int x_off;            // byte offset of the staged activations
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

// Packed multiply with one rounding of the exact product (torch's bf16 / fp16 mul).
template <bool kBf16>
__device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b) {
    uint32_t d;
    if constexpr (kBf16) asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    else asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
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
// A 128-bit shared load into `v` done only by lanes with `p` set; the others keep
// `v` without issuing a request (so a warp whose upper lanes are idle costs one
// shared-memory wavefront instead of four).
__device__ __forceinline__ void lds128_if(uint4& v, uint32_t addr, int p) {
    asm volatile(
        "{\n .reg .pred q;\n setp.ne.b32 q, %5, 0;\n"
        " @q ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n}\n"
        : "+r"(v.x), "+r"(v.y), "+r"(v.z), "+r"(v.w)
        : "r"(addr), "r"(p));
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

// Activation type helpers on 16-bit raw values.
template <bool kBf16>
__device__ __forceinline__ float act_to_f(uint32_t raw16) {
    if constexpr (kBf16) return __uint_as_float(raw16 << 16);
    else return __half2float(__ushort_as_half((unsigned short)raw16));
}
template <bool kBf16>
__device__ __forceinline__ uint32_t f_to_act(float v) {
    if constexpr (kBf16) return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v));
    else return (uint32_t)__half_as_ushort(__float2half_rn(v));
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
// The weight stream (index tiles and scales) is read once per call: evict-first in
// L2, so that it does not push the KV rows, activations and codebooks out.
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                         uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void tma_load_2d_stream(uint32_t dst, const void* tmap, uint32_t bar, int c0, int c1,
                                                   uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(tmap), "r"(c0), "r"(c1), "r"(bar), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
}

// Shared-memory barriers at the start of the dynamic block: the ring's full /
// empty pairs, then per reduction slot a "full" barrier (the 16 consumer warps
// have written their partial sums) and a "free" one (the reducer warp is done).
struct Bars {
    uint32_t full, empty, slot_full, slot_free;
    __device__ explicit Bars(uint32_t sbase)
        : full(sbase), empty(sbase + 8 * kStages), slot_full(sbase + 16 * kStages),
          slot_free(sbase + 16 * kStages + 8 * kSlots) {}
};
static_assert(16 * kStages + 16 * kSlots <= kBarBytes, "barrier block");

__device__ __forceinline__ void init_bars(const Bars& B) {
    for (int s = 0; s < kStages; ++s) {
        mbar_init(B.full + 8 * s, 1);
        mbar_init(B.empty + 8 * s, kConsumerWarps);
    }
    for (int s = 0; s < kSlots; ++s) {
        mbar_init(B.slot_full + 8 * s, kConsumerWarps);
        mbar_init(B.slot_free + 8 * s, 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Codebook of store S -> 16 copies in the activation type in its half (`part`)
// of the replica block: entry e, copy c at byte e * 256 + part * 128 + c * 8;
// lane l reads copy l % 16, so a half-warp's random gathers never share a bank
// pair.  Consumer threads 0..255 first convert one entry each into `stage`
// (2 KB); after a consumer barrier thread t writes slots t, t + 512, ..., so a
// warp's 32 stores cover two 128-byte runs (no bank conflicts).
template <bool kBf16>
__device__ void build_replica(const MmaStore& S, uint2* rep, int part, uint2* stage) {
    const int t = threadIdx.x;
    if (t < 256) {
        uint2 v = make_uint2(0u, 0u);
        if (t < S.levels) {
            const int64_t b = (int64_t)t * 4;
            v.x = cvt_pair<kBf16>(load_f(S.cb, S.cb_dtype, b), load_f(S.cb, S.cb_dtype, b + 1));
            v.y = cvt_pair<kBf16>(load_f(S.cb, S.cb_dtype, b + 2), load_f(S.cb, S.cb_dtype, b + 3));
        }
        stage[t] = v;
    }
    consumers_sync();
#pragma unroll
    for (int i = 0; i < 4096 / kConsumers; ++i) {
        const int slot = t + i * kConsumers;   // entry slot / 16, copy slot % 16
        rep[(slot >> 4) * 32 + part * 16 + (slot & 15)] = stage[slot >> 4];
    }
}

// kT (1 .. kTileSets) tiles of one chunk, interleaved so their gathers and MMAs
// overlap: tile t is group gl0 + kConsumerWarps t of the chunk (one 16-row block x
// 128 weights), its products go to accumulator chain t.  Lanes whose B column is past the m
// activation rows (xact0 / xact1 zero) load no activations: their columns of
// the product are never stored, so they multiply zeros.
template <bool kBf16, int kNT, bool kScaleF32, bool kXSmem, int kT>
__device__ __forceinline__ void mma_tiles(float (&acc)[kTileSets][kNT][4], const uint32_t sdst, const int gl0, const int g0,
                                          const uint32_t lanebase, const uint32_t xs0, const uint32_t xs1,
                                          const uint16_t* xg0, const uint16_t* xg1, const int k_lane,
                                          const int lane, const int xact0, const int xact1) {
    constexpr int kScaleBytes = kScaleF32 ? 4 : 2;
    const int gq = lane >> 2;
    uint32_t wlo[kT][2], whi[kT][2], sc0[kT], sc1[kT];
#pragma unroll
    for (int t = 0; t < kT; ++t) {
        const int gl = gl0 + kConsumerWarps * t;
        const uint4 w = lds128(sdst + gl * 512 + lane * 16);
        wlo[t][0] = w.x;
        wlo[t][1] = w.y;
        whi[t][0] = w.z;
        whi[t][1] = w.w;
        // The rows' scales rounded to the activation type, twice per register.
        const float s0 = lds_scale<kScaleF32>(sdst + kStageIdx + (gl * 16 + gq) * kScaleBytes);
        const float s1 = lds_scale<kScaleF32>(sdst + kStageIdx + (gl * 16 + gq + 8) * kScaleBytes);
        sc0[t] = cvt_pair<kBf16>(s0, s0);
        sc1[t] = cvt_pair<kBf16>(s1, s1);
    }
    // The B fragments keep their registers across the four k-step pairs: a lane that
    // loads no activations keeps the zeros set here once per tile (its product columns
    // are never stored).
    uint4 bx[kT], by[kT];
#pragma unroll
    for (int t = 0; t < kT; ++t) bx[t] = by[t] = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int p = 0; p < 4; ++p) {
#pragma unroll
        for (int t = 0; t < kT; ++t) {
            const int gidx = g0 + gl0 + kConsumerWarps * t;
            if constexpr (kXSmem) {
                lds128_if(bx[t], xs0 + (gidx * 4 + p) * 64, xact0);
                if constexpr (kNT == 2) lds128_if(by[t], xs1 + (gidx * 4 + p) * 64, xact1);
            } else {
                // Global loads: lanes past m read row m - 1 (their columns are never stored).
                const int col = gidx * 128 + 32 * p;
                const uint2 z = make_uint2(0u, 0u);
                const uint2 b0 = col < k_lane ? __ldg(reinterpret_cast<const uint2*>(xg0 + col)) : z;
                const uint2 b1 = col + 16 < k_lane ? __ldg(reinterpret_cast<const uint2*>(xg0 + col + 16)) : z;
                bx[t] = make_uint4(b0.x, b0.y, b1.x, b1.y);
                if constexpr (kNT == 2) {
                    const uint2 c0 = col < k_lane ? __ldg(reinterpret_cast<const uint2*>(xg1 + col)) : z;
                    const uint2 c1 = col + 16 < k_lane ? __ldg(reinterpret_cast<const uint2*>(xg1 + col + 16)) : z;
                    by[t] = make_uint4(c0.x, c0.y, c1.x, c1.y);
                }
            }
        }
#pragma unroll
        for (int hs = 0; hs < 2; ++hs) {
            const int s = 2 * p + hs;
            // window address = byte 0 of lanebase (part * 128 + copy * 8), byte 1
            // the index (entry * 256), bytes 2-3 of lanebase (kRepWin >> 16)
            const uint32_t sel = 0x7604u | ((uint32_t)(s & 3) << 4);
            uint2 alo[kT], ahi[kT];
#pragma unroll
            for (int t = 0; t < kT; ++t) {
                alo[t] = lds64(__byte_perm(wlo[t][s >> 2], lanebase, sel));
                ahi[t] = lds64(__byte_perm(whi[t][s >> 2], lanebase, sel));
            }
#pragma unroll
            for (int t = 0; t < kT; ++t) {
                const uint32_t a0 = mul2<kBf16>(alo[t].x, sc0[t]), a2 = mul2<kBf16>(alo[t].y, sc0[t]);
                const uint32_t a1 = mul2<kBf16>(ahi[t].x, sc1[t]), a3 = mul2<kBf16>(ahi[t].y, sc1[t]);
                mma16816<kBf16>(acc[t][0], a0, a1, a2, a3, hs ? bx[t].z : bx[t].x, hs ? bx[t].w : bx[t].y);
                if constexpr (kNT == 2)
                    mma16816<kBf16>(acc[t][1], a0, a1, a2, a3, hs ? by[t].z : by[t].x, hs ? by[t].w : by[t].y);
            }
        }
    }
}

__device__ __forceinline__ int store_of(const MmaParams& P, int u) {
    int si = 0;
    while (si + 1 < P.count && u >= P.st[si + 1].unit0) ++si;
    return si;
}

// Element offset of activation (row, col) in the staged B-fragment order: per
// group, per pair of k-steps p (s = 2p, 2p+1), per lane column q, 8 values
// {x[c0 .. c0+3], x[c0+16 .. c0+19]} with c0 = 128 g + 32 p + 4 q.
__device__ __forceinline__ int xperm(int row, int kpad, int col) {
    const int g = col >> 7, s = (col >> 4) & 7, q = (col >> 2) & 3, j = col & 3;
    return row * kpad + (((g * 4 + (s >> 1)) * 4 + q) << 3) + ((s & 1) << 2) + j;
}

// Loads of data another CTA of a persistent program wrote during this launch go
// to L2 (.cg): L1 is not coherent across SMs, and a program reuses its
// activation buffers layer after layer.  A single launch reads only what the
// previous kernel wrote, so it may use plain loads.
template <bool kProg>
__device__ __forceinline__ uint2 ld_x8(const uint16_t* p) {
    if constexpr (kProg) return __ldcg(reinterpret_cast<const uint2*>(p));
    else return *reinterpret_cast<const uint2*>(p);
}
template <bool kProg>
__device__ __forceinline__ float ld_act(const void* p, int dt, int64_t o) {
    if constexpr (kProg) {
        const unsigned short r = __ldcg(static_cast<const unsigned short*>(p) + o);
        return dt == EPQ_BF16 ? __uint_as_float((uint32_t)r << 16) : __half2float(__ushort_as_half(r));
    } else {
        return load_f(p, dt, o);
    }
}

// The CTA's contiguous, balanced range of units (16-row blocks) of a linear.
__device__ __forceinline__ void unit_range(int U, int& u_begin, int& u_end) {
    const int G = gridDim.x;
    u_begin = (int)((int64_t)U * blockIdx.x / G);
    u_end = (int)((int64_t)U * (blockIdx.x + 1) / G);
}

// Producer warp: streams the chunks of units [u_begin, u_end) of P into the
// ring.  `ring` counts the ring positions used so far (a persistent program
// keeps counting across its linears, so the stage parities line up).
template <bool kScaleF32>
__device__ __forceinline__ void produce_linear(const MmaParams& P, int u_begin, int u_end, uint32_t bar_full,
                                               uint32_t bar_empty, uint32_t stage0, int lane, uint32_t& ring) {
    constexpr int kScaleBytes = kScaleF32 ? 4 : 2;
    const uint64_t pol = evict_first_policy();
    const int cpu = P.chunks_per_unit, parts = P.parts, count = P.count;
    const int n_chunks = (u_end - u_begin) * cpu * parts;
    int si = parts == 2 ? 0 : store_of(P, u_begin);
    int s_next = (parts == 1 && si + 1 < count) ? P.st[si + 1].unit0 : INT_MAX;
    int u = u_begin, part = 0, c = 0;
    // Ring position `ring` as (stage, phase); a stage is refilled once the consumers
    // have released its previous use (phase - 1), nothing to wait for on the first lap.
    uint32_t stage = ring % kStages, phase = (ring / kStages) & 1;
    bool lapped = ring >= (uint32_t)kStages;
    ring += (uint32_t)n_chunks;
    for (int j = 0; j < n_chunks; ++j) {
        if (lapped) mbar_wait(bar_empty + 8 * stage, phase ^ 1);
        int rb;
        if (parts == 2) {
            si = part;
            rb = u;
        } else {
            if (u >= s_next) {
                si = store_of(P, u);
                s_next = si + 1 < count ? P.st[si + 1].unit0 : INT_MAX;
            }
            rb = u - P.st[si].unit0;
        }
        const MmaStore& S = P.st[si];
        const int g0 = c * kChunkGroups;
        const int ngc = min(kChunkGroups, S.ng - g0);
        const uint32_t dst = stage0 + stage * kStageBytes;
        // Two copies per chunk: the index tiles (one contiguous run) and the
        // scales of its 16 rows x 32 groups (one 2-D tensor box; groups past
        // the store's last are zero-filled, and the full box is counted).
        if (lane == 0) {
            mbar_expect_tx(bar_full + 8 * stage, ngc * 512 + kChunkGroups * 16 * kScaleBytes);
            bulk_g2s(dst, S.idx + ((int64_t)rb * S.ng + g0) * 512, ngc * 512, bar_full + 8 * stage, pol);
            tma_load_2d_stream(dst + kStageIdx, &S.smap, bar_full + 8 * stage, rb * 16, g0, pol);
        }
        __syncwarp();
        if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
            lapped = true;
        }
        if (++c == cpu) {
            c = 0;
            if (++part == parts) {
                part = 0;
                ++u;
            }
        }
    }
}

// Consumers: the codebook replica(s) of the store(s) the CTA's first unit reads
// (nothing when the CTA has no unit).  Ends with a consumer barrier.
template <bool kBf16>
__device__ __forceinline__ void prepare_linear(const MmaParams& P, int u_begin, int u_end, uint2* rep,
                                               uint2* cb_stage) {
    if (u_begin >= u_end) return;
    const int cur = P.parts == 2 ? 0 : store_of(P, u_begin);
    for (int r = 0; r < P.parts; ++r) {
        if (r) consumers_sync();   // the staging area is reused
        build_replica<kBf16>(P.st[P.parts == 2 ? r : cur], rep, r, cb_stage);
    }
    consumers_sync();   // the staging area is the RMSNorm scratch next
}

// Consumers: stage x (kXSmem; RMSNorm prologue), run the chunks of units
// [u_begin, u_end) from the ring, reduce each unit and run the epilogue.
// prepare_linear must have run for this range.
template <bool kBf16, int kNT, bool kScaleF32, bool kXSmem, bool kProg>
__device__ __forceinline__ void run_linear(const MmaParams& P, int u_begin, int u_end, uint8_t* smem,
                                           uint32_t sbase, uint32_t& ring, uint32_t& uc) {
    const Bars B(sbase);
    const uint32_t stage0 = sbase + kBarBytes;
    uint2* rep = reinterpret_cast<uint2*>(smem + (kRepWin - sbase));
    float* slots = reinterpret_cast<float*>(smem + (kHighWin - sbase));
    uint16_t* xs = reinterpret_cast<uint16_t*>(smem + (P.x_off - sbase));   // [m][kpad] when kXSmem
    uint2* cb_stage = reinterpret_cast<uint2*>(smem + kBarBytes + kStages * kStageBytes);
    float* scratch = reinterpret_cast<float*>(cb_stage);   // RMSNorm partial sums (m x 16 floats)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cpu = P.chunks_per_unit, parts = P.parts, count = P.count, M = P.m;
    const int n_chunks = (u_end - u_begin) * cpu * parts;
    const int gq = lane >> 2, q = lane & 3;
    int cur = parts == 2 ? 0 : store_of(P, u_begin);
    int c_next = (parts == 1 && cur + 1 < count) ? P.st[cur + 1].unit0 : INT_MAX;

    // Activation B fragments: lane (gq, q) supplies column gq = activation row
    // min(gq, m - 1) (columns >= m are computed and never stored).
    const int xr0 = gq < M ? gq : M - 1;
    const int xr1 = gq + 8 < M ? gq + 8 : M - 1;
    const uint16_t* xg0 = static_cast<const uint16_t*>(P.x) + (int64_t)xr0 * P.ldx + 4 * q;
    const uint16_t* xg1 = static_cast<const uint16_t*>(P.x) + (int64_t)xr1 * P.ldx + 4 * q;
    uint32_t xs0 = 0, xs1 = 0;
    if constexpr (kXSmem) {
        // Stage x (or RMSNorm(x)) in the permuted B-fragment order.
        const int per_row = P.kpad >> 2;
        const bool norm = P.prologue == EPQ_PRO_RMSNORM;
        for (int row = 0; row < M; ++row) {
            float ss = 0.f;
            for (int i = threadIdx.x; i < per_row; i += kConsumers) {
                const int c4 = i * 4;
                uint2 v = make_uint2(0u, 0u);
                if (c4 < P.k) v = ld_x8<kProg>(static_cast<const uint16_t*>(P.x) + (int64_t)row * P.ldx + c4);
                if (norm) {
                    const float a = act_to_f<kBf16>(v.x & 0xffffu), b = act_to_f<kBf16>(v.x >> 16);
                    const float c = act_to_f<kBf16>(v.y & 0xffffu), d = act_to_f<kBf16>(v.y >> 16);
                    ss += a * a + b * b + c * c + d * d;
                }
                *reinterpret_cast<uint2*>(xs + xperm(row, P.kpad, c4)) = v;
            }
            if (norm) {
                for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
                if (lane == 0) scratch[row * kConsumerWarps + warp] = ss;
            }
        }
        if (norm) {
            consumers_sync();
            for (int row = 0; row < M; ++row) {
                float ss = 0.f;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w) ss += scratch[row * kConsumerWarps + w];
                const float r = rsqrtf(ss / (float)P.k + P.eps);
                for (int i = threadIdx.x; i < per_row; i += kConsumers) {
                    uint2* p = reinterpret_cast<uint2*>(xs + xperm(row, P.kpad, i * 4));
                    const uint2 v = *p;
                    uint2 y;
                    y.x = f_to_act<kBf16>(act_to_f<kBf16>(v.x & 0xffffu) * r) |
                          (f_to_act<kBf16>(act_to_f<kBf16>(v.x >> 16) * r) << 16);
                    y.y = f_to_act<kBf16>(act_to_f<kBf16>(v.y & 0xffffu) * r) |
                          (f_to_act<kBf16>(act_to_f<kBf16>(v.y >> 16) * r) << 16);
                    *p = y;
                }
            }
        }
        const uint32_t xsb = static_cast<uint32_t>(__cvta_generic_to_shared(xs));
        xs0 = xsb + (xr0 * P.kpad + 8 * q) * 2;
        xs1 = xsb + (xr1 * P.kpad + 8 * q) * 2;
    }
    consumers_sync();

    const int k_lane = P.k - 4 * q;   // global-load path: column c is in range iff c < k_lane
    const int xact0 = gq < M, xact1 = gq + 8 < M;   // this lane's B columns are activation rows
    const uint32_t lane16 = (kRepWin & 0xffff0000u) | ((uint32_t)(lane & 15) << 3);
    // Two accumulator chains (the two tiles a warp takes per chunk) keep dependent MMAs apart.
    float acc[kTileSets][kNT][4];
#pragma unroll
    for (int e = 0; e < kTileSets; ++e)
#pragma unroll
        for (int h = 0; h < kNT; ++h) acc[e][h][0] = acc[e][h][1] = acc[e][h][2] = acc[e][h][3] = 0.f;
    int u = u_begin, part = 0, c = 0;
    // Ring position `ring` as (stage, phase), advanced incrementally per chunk.
    uint32_t stage = ring % kStages, phase = (ring / kStages) & 1;
    ring += (uint32_t)n_chunks;
    for (int j = 0; j < n_chunks; ++j, stage = stage + 1 == kStages ? 0 : stage + 1, phase ^= stage == 0) {
        if (parts == 1 && c == 0 && u >= c_next) {
            // New store (CTA-uniform): rebuild the codebook replica once every warp
            // is past the previous store's gathers.
            consumers_sync();
            cur = store_of(P, u);
            c_next = cur + 1 < count ? P.st[cur + 1].unit0 : INT_MAX;
            build_replica<kBf16>(P.st[cur], rep, 0, cb_stage);
            consumers_sync();
        }
        const int sidx = parts == 2 ? part : cur;
        const int ng = P.st[sidx].ng;
        const uint32_t lanebase = lane16 | (uint32_t)((parts == 2 ? part : 0) << 7);
        const int g0 = c * kChunkGroups;
        const int ngc = min(kChunkGroups, ng - g0);
        mbar_wait(B.full + 8 * stage, phase);
        const uint32_t sdst = stage0 + stage * kStageBytes;
        {
            // this warp's tiles of the chunk: groups warp, warp + kConsumerWarps, ... < ngc
            const int nt = warp < ngc ? min(kTileSets, (ngc - warp + kConsumerWarps - 1) / kConsumerWarps) : 0;
#define EPQ_TILES(T)                                                                                            \
    mma_tiles<kBf16, kNT, kScaleF32, kXSmem, T>(acc, sdst, warp, g0, lanebase, xs0, xs1, xg0, xg1, k_lane, lane, \
                                                xact0, xact1)
            if constexpr (kTileSets >= 4) {
                if (nt == 4) EPQ_TILES(4);
                else if (nt == 3) EPQ_TILES(3);
                else if (nt == 2) EPQ_TILES(2);
                else if (nt == 1) EPQ_TILES(1);
            } else {
                if (nt == 2) EPQ_TILES(2);
                else if (nt == 1) EPQ_TILES(1);
            }
#undef EPQ_TILES
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(B.empty + 8 * stage);   // this warp is done with the stage
        if (++c < cpu) continue;
        c = 0;
        // End of one part of a unit: this warp's partial sums into the unit's slot,
        // laid out [part][warp][m][16 rows].  A slot is reused kSlots units later,
        // once the reducer warp has released it.
        const uint32_t uslot = uc % kSlots;
        if (part == 0 && uc >= (uint32_t)kSlots) mbar_wait(B.slot_free + 8 * uslot, ((uc / kSlots) - 1) & 1);
        {
            float* mine = slots + uslot * P.slot_floats + (part * kConsumerWarps + warp) * 16 * M;
#pragma unroll
            for (int h = 0; h < kNT; ++h) {
                const int m0 = 8 * h + 2 * q;
                float r[4] = {acc[0][h][0], acc[0][h][1], acc[0][h][2], acc[0][h][3]};
#pragma unroll
                for (int e = 1; e < kTileSets; ++e)
#pragma unroll
                    for (int j = 0; j < 4; ++j) r[j] += acc[e][h][j];
                if (m0 < M) {
                    mine[m0 * 16 + gq] = r[0];
                    mine[m0 * 16 + gq + 8] = r[2];
                }
                if (m0 + 1 < M) {
                    mine[(m0 + 1) * 16 + gq] = r[1];
                    mine[(m0 + 1) * 16 + gq + 8] = r[3];
                }
#pragma unroll
                for (int e = 0; e < kTileSets; ++e) acc[e][h][0] = acc[e][h][1] = acc[e][h][2] = acc[e][h][3] = 0.f;
            }
        }
        if (++part < parts) continue;
        part = 0;
        __syncwarp();   // the warp's partial sums precede lane 0's (releasing) arrival
        if (lane == 0) mbar_arrive(B.slot_full + 8 * uslot);
        ++u;
        ++uc;
    }
}

// Reducer warp: for every unit of [u_begin, u_end), in order, waits until the 16
// consumer warps have dropped their partial sums into its slot, adds them in
// warp order (deterministic), runs the epilogue and releases the slot.
template <bool kBf16, int kNT, bool kProg>
__device__ __forceinline__ void reduce_linear(const MmaParams& P, int u_begin, int u_end, uint8_t* smem,
                                              uint32_t sbase, uint32_t& uc) {
    const Bars B(sbase);
    const float* slots = reinterpret_cast<const float*>(smem + (kHighWin - sbase));
    const int lane = threadIdx.x & 31;
    const int parts = P.parts, count = P.count, M = P.m;
    const int per = 16 * M;   // floats per warp per part
    int cur = parts == 2 ? 0 : store_of(P, u_begin);
    int c_next = (parts == 1 && cur + 1 < count) ? P.st[cur + 1].unit0 : INT_MAX;
    for (int u = u_begin; u < u_end; ++u, ++uc) {
        if (parts == 1 && u >= c_next) {
            cur = store_of(P, u);
            c_next = cur + 1 < count ? P.st[cur + 1].unit0 : INT_MAX;
        }
        const uint32_t uslot = uc % kSlots;
        mbar_wait(B.slot_full + 8 * uslot, (uc / kSlots) & 1);
        const MmaStore& S = P.st[parts == 2 ? 0 : cur];
        const int rowbase = (parts == 2 ? u : u - S.unit0) * 16;
        const float* base = slots + uslot * P.slot_floats;
        const int n_rows = S.n;
        void* const out = S.out;
        const int64_t ldo = S.ldo;
        for (int e = lane; e < per; e += 32) {
            const int rr = e & 15, mm = e >> 4;
            const int row = rowbase + rr;
            float v0 = 0.f, v1 = 0.f;
#pragma unroll
            for (int ww = 0; ww < kConsumerWarps; ++ww) v0 += base[ww * per + e];
            if (parts == 2) {
#pragma unroll
                for (int ww = 0; ww < kConsumerWarps; ++ww) v1 += base[(kConsumerWarps + ww) * per + e];
            }
            if (row < n_rows) {
                const int64_t o = (int64_t)mm * ldo + row;
                if (P.epilogue == EPQ_EPI_RESIDUAL) {
                    const int dt = kBf16 ? EPQ_BF16 : EPQ_F16;
                    store_f(out, dt, o, ld_act<kProg>(out, dt, o) + round_to(v0, dt));
                } else if (P.epilogue == EPQ_EPI_SILU_MUL) {
                    const int dt = kBf16 ? EPQ_BF16 : EPQ_F16;
                    const float gv = round_to(v0, dt), uv = round_to(v1, dt);
                    store_f(out, dt, o, gv / (1.f + expf(-gv)) * uv);
                } else {
                    store_f(out, P.out_dtype, o, v0);
                }
            }
        }
        __syncwarp();   // the slot's reads (and the epilogue's stores) precede the release
        if (lane == 0) mbar_arrive(B.slot_free + 8 * uslot);
    }
}

template <bool kBf16, int kNT, bool kScaleF32, bool kXSmem>
__global__ void __launch_bounds__(kThreads, 1) gemv_mma_kernel(const __grid_constant__ MmaParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    if (sbase + kLowBytes > kRepWin) {   // the layout needs the dynamic block to start low (uniform)
        if (threadIdx.x == 0) atomicExch(&g_mma_wait_timeout, 1);
        return;
    }
    const Bars B(sbase);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int u_begin, u_end;
    unit_range(P.total_units, u_begin, u_end);
    if (threadIdx.x == 0) init_bars(B);
    __syncthreads();

    uint32_t ring = 0, uc = 0;
    if (warp == kProducerWarp) {
        // Weights do not depend on the previous kernel: stream them right away.
        produce_linear<kScaleF32>(P, u_begin, u_end, B.full, B.empty, sbase + kBarBytes, lane, ring);
        pdl_trigger();
        return;
    }
    if (warp == kReducerWarp) {
        pdl_trigger();
        pdl_wait();   // the residual stream belongs to the previous kernel until here
        reduce_linear<kBf16, kNT, false>(P, u_begin, u_end, smem, sbase, uc);
        return;
    }
    uint2* rep = reinterpret_cast<uint2*>(smem + (kRepWin - sbase));
    uint2* cb_stage = reinterpret_cast<uint2*>(smem + kBarBytes + kStages * kStageBytes);
    prepare_linear<kBf16>(P, u_begin, u_end, rep, cb_stage);
    pdl_trigger();
    pdl_wait();   // x (and the output buffers) belong to the previous kernel until here
    run_linear<kBf16, kNT, kScaleF32, kXSmem, false>(P, u_begin, u_end, smem, sbase, ring, uc);
}

// ---------------------------------------------------------------------------
// Decode program: the steps of a whole decode token (every layer's fused packed
// linears and its attention) run by ONE persistent cooperative kernel, one CTA
// per SM.  The producer warp streams the weight chunks of all linear steps back
// to back through the ring -- weights never depend on activations, so HBM keeps
// streaming across step boundaries -- while the consumer warps run the steps in
// order, separated by a grid-wide arrival counter per step (an activation step
// needs every CTA's rows of the previous one).  A CTA rebuilds the codebook
// replica for its next step while it waits for the others.
// ---------------------------------------------------------------------------
constexpr int kStepLinear = 0, kStepAttention = 1;
constexpr int kProgMaxSplits = 16;
constexpr uint32_t kGridSpinLimit = 1u << 23;   // grid-barrier polls (about a second with the naps)

__device__ int g_prog_position_error = 0;

struct AttnStep {
    const uint16_t* q;       // [heads, hd] bf16 (this token's projections)
    const uint16_t* k;       // [kv_heads, hd]
    const uint16_t* v;
    uint16_t* k_cache;       // [max_len, kv_heads, hd]
    uint16_t* v_cache;
    const int64_t* pos;      // device position of this token
    int64_t max_len;
    const float* cos_t;      // [max_len, hd / 2]
    const float* sin_t;
    uint16_t* out;           // [heads, hd]
    int heads, kv_heads, head_dim, qk_norm, splits;
    float eps, scale;
};

struct ProgStep {
    MmaParams lin;
    AttnStep attn;
    int kind;
};

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Consumers wait until every CTA has arrived at `bar` (thread 0 polls with
// acquire loads, bounded; the consumer barrier passes the acquisition on).
__device__ __forceinline__ void grid_wait(const unsigned* bar, unsigned target) {
    if (threadIdx.x == 0) {
        for (uint32_t n = 0; ld_acquire_u32(bar) < target; ++n) {
            if (n == kGridSpinLimit) {
                atomicExch(&g_mma_wait_timeout, 1);
                break;
            }
            __nanosleep(64);
        }
    }
    consumers_sync();
}
// The consumer barrier orders every consumer's writes of the step before thread
// 0's release-add at GPU scope (the cumulative release publishes them).
__device__ __forceinline__ void grid_arrive(unsigned* bar) {
    consumers_sync();
    if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(bar) : "memory");
}

__device__ __forceinline__ float bf16_bits(uint16_t r) { return __uint_as_float((uint32_t)r << 16); }
__device__ __forceinline__ uint16_t to_bf16_bits(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

constexpr int kAttnRows = 64;   // cache positions staged in shared memory per pass

// Stages cache rows [base, base + cnt) of kv head kvh (except position P, which
// comes from registers) into kst / vst with asynchronous 16-byte copies.
template <int kDims>
__device__ __forceinline__ void stage_kv(const AttnStep& A, int kvh, int64_t base, int cnt, int64_t P, uint16_t* kst,
                                         uint16_t* vst) {
    constexpr int hd = kDims * 32, pieces = hd / 8;
    const int KV = A.kv_heads;
    for (int i = threadIdx.x; i < cnt * pieces; i += kConsumers) {
        const int r = i / pieces, c = i - r * pieces;
        const int64_t t = base + r;
        if (t == P) continue;
        const int64_t off = (t * KV + kvh) * hd + c * 8;
        cp_async16(kst + r * hd + c * 8, A.k_cache + off);
        cp_async16(vst + r * hd + c * 8, A.v_cache + off);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// The first pass of an attention step's K / V rows, issued before the grid
// barrier that precedes the step: the position and the cached rows before it
// come from earlier launches, not from the step before (which only writes q /
// k / v), so their HBM latency overlaps the wait.
template <int kDims>
__device__ void prestage_attention(const AttnStep& A, uint16_t* kst, uint16_t* vst) {
    const int64_t P = A.pos[0];
    if (P < 0 || P >= A.max_len) return;
    const int64_t n = P + 1;
    const int S = (int)min((int64_t)A.splits, (n + kAttnRows - 1) / kAttnRows);
    const int blk = blockIdx.x;
    if (blk >= A.kv_heads * S) return;
    const int kvh = blk / S, split = blk - kvh * S;
    const int64_t chunk = (n + S - 1) / S;
    const int64_t t0 = split * chunk, t1 = min(n, t0 + chunk);
    const int cnt = (int)min((int64_t)kAttnRows, t1 - t0);
    if (cnt > 0) stage_kv<kDims>(A, kvh, t0, cnt, P, kst, vst);
}


// Attention step.  The positions 0..P are split over S CTAs per kv head, S the
// fewest splits (at most A.splits) that keep a CTA's range within kAttnRows, so
// a short context needs no cross-CTA merge.  A CTA stages its K / V rows in
// shared memory with asynchronous copies issued first, then applies (q/k
// RMSNorm and) RoPE to q and to this position's k meanwhile; split 0 writes k, v
// into the caches.  The kGroup query heads of the kv head share the 16 consumer
// warps (16 / group per head, every (16 / group)-th position each, four
// positions per step of the loop); per-warp online softmax, merged per head in
// the CTA; with S > 1 one record per (split, head) goes to global memory and
// the last CTA of the kv head merges them in split order.  Same arithmetic as
// the epq_attn_rope_decode kernels (their split merge order aside).
// `prestaged`: prestage_attention has issued the first pass already.
template <int kDims>
__device__ void prog_attention(const AttnStep& A, float* scr, uint16_t* kst, uint16_t* vst, float* recs,
                               unsigned* counters, bool prestaged) {
    constexpr int hd = kDims * 32, kRec = hd + 2;
    const int KV = A.kv_heads, group = A.heads / KV;
    const int blk = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t P = A.pos[0];
    if (P < 0 || P >= A.max_len) {   // every CTA sees the same position
        if (blk < KV) {
            for (int e = threadIdx.x; e < group * hd; e += kConsumers) A.out[(int64_t)blk * group * hd + e] = 0;
            if (threadIdx.x == 0) atomicExch(&g_prog_position_error, 1);
        }
        return;
    }
    const int64_t n = P + 1;
    const int S = (int)min((int64_t)A.splits, (n + kAttnRows - 1) / kAttnRows);
    if (blk >= KV * S) return;
    const int kvh = blk / S, split = blk - kvh * S;
    const int wpg = kConsumerWarps / group;
    const int g = warp / wpg, wsub = warp - g * wpg;
    const int64_t chunk = (n + S - 1) / S;
    const int64_t t0 = split * chunk, t1 = min(n, t0 + chunk);
    int64_t base = t0;
    int cnt = (int)min((int64_t)kAttnRows, t1 - base);
    if (cnt > 0 && !prestaged) stage_kv<kDims>(A, kvh, base, cnt, P, kst, vst);

    const int qh = kvh * group + g;
    float qv[kDims], acc[kDims], kc[kDims], vc[kDims];
#pragma unroll
    for (int d = 0; d < kDims; ++d) {
        qv[d] = bf16_bits(__ldcg(A.q + (int64_t)qh * hd + lane * kDims + d));
        kc[d] = bf16_bits(__ldcg(A.k + (int64_t)kvh * hd + lane * kDims + d));
        vc[d] = bf16_bits(__ldcg(A.v + (int64_t)kvh * hd + lane * kDims + d));
        acc[d] = 0.f;
    }
    rope_head<kDims>(qv, lane, P, A.cos_t, A.sin_t, A.qk_norm, A.eps);
    rope_head<kDims>(kc, lane, P, A.cos_t, A.sin_t, A.qk_norm, A.eps);
    if (split == 0 && warp == 0) {
        const int64_t cb = (P * KV + kvh) * hd + lane * kDims;
#pragma unroll
        for (int d = 0; d < kDims; ++d) {
            A.k_cache[cb + d] = to_bf16_bits(kc[d]);
            A.v_cache[cb + d] = to_bf16_bits(vc[d]);
        }
    }
    float m = -INFINITY, l = 0.f;
    while (cnt > 0) {
        cp_async_wait_all();
        if (warp == 0 && P >= base && P < base + cnt) {   // this position from registers
#pragma unroll
            for (int d = 0; d < kDims; ++d) {
                kst[(P - base) * hd + lane * kDims + d] = to_bf16_bits(kc[d]);
                vst[(P - base) * hd + lane * kDims + d] = to_bf16_bits(vc[d]);
            }
        }
        consumers_sync();
        for (int j0 = wsub; j0 < cnt; j0 += 4 * wpg) {
            float sc[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int j = j0 + u * wpg;
                float s = 0.f;
                if (j < cnt) {
#pragma unroll
                    for (int d = 0; d < kDims; ++d) s += qv[d] * bf16_bits(kst[j * hd + lane * kDims + d]);
                }
                sc[u] = s;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int u = 0; u < 4; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], o);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int j = j0 + u * wpg;
                if (j >= cnt) break;
                const float s = sc[u] * A.scale;
                const float mn = fmaxf(m, s);
                const float corr = expf(m - mn), pw = expf(s - mn);
                l = l * corr + pw;
#pragma unroll
                for (int d = 0; d < kDims; ++d) acc[d] = acc[d] * corr + pw * bf16_bits(vst[j * hd + lane * kDims + d]);
                m = mn;
            }
        }
        base += cnt;
        cnt = (int)min((int64_t)kAttnRows, t1 - base);
        consumers_sync();   // every warp is done with the staged rows
        if (cnt > 0) stage_kv<kDims>(A, kvh, base, cnt, P, kst, vst);
    }
    if (lane == 0) {
        scr[warp * kRec + hd] = m;
        scr[warp * kRec + hd + 1] = l;
    }
#pragma unroll
    for (int d = 0; d < kDims; ++d) scr[warp * kRec + lane * kDims + d] = acc[d];
    consumers_sync();
    float* rec = recs + ((int64_t)(kvh * S + split) * group) * kRec;
    for (int e = threadIdx.x; e < group * hd; e += kConsumers) {
        const int gg = e / hd, d = e - gg * hd;
        float mx = -INFINITY;
        for (int w = gg * wpg; w < (gg + 1) * wpg; ++w) mx = fmaxf(mx, scr[w * kRec + hd]);
        float num = 0.f, den = 0.f;
        for (int w = gg * wpg; w < (gg + 1) * wpg; ++w) {
            if (scr[w * kRec + hd] == -INFINITY) continue;   // a warp that saw no position
            const float f = expf(scr[w * kRec + hd] - mx);
            num += f * scr[w * kRec + d];
            den += f * scr[w * kRec + hd + 1];
        }
        if (S == 1) {
            A.out[(int64_t)(kvh * group + gg) * hd + d] = to_bf16_bits(num / den);
        } else {
            rec[gg * kRec + d] = num;
            if (d == 0) {
                rec[gg * kRec + hd] = mx;
                rec[gg * kRec + hd + 1] = den;
            }
        }
    }
    if (S == 1) return;
    __threadfence();
    consumers_sync();
    int* last = reinterpret_cast<int*>(scr + kConsumerWarps * kRec);
    if (threadIdx.x == 0) *last = atomicAdd(&counters[kvh], 1u) == (unsigned)(S - 1);
    consumers_sync();
    if (!*last) return;
    __threadfence();
    // The S records' (max, sum) first, all loads in flight at once.
    const float* rbase = recs + (int64_t)kvh * S * group * kRec;
    float* ml = scr;   // [S][group][2]; the warp records are consumed
    for (int i = threadIdx.x; i < S * group; i += kConsumers) {
        ml[2 * i] = __ldcg(rbase + i * kRec + hd);
        ml[2 * i + 1] = __ldcg(rbase + i * kRec + hd + 1);
    }
    consumers_sync();
    for (int e = threadIdx.x; e < group * hd; e += kConsumers) {
        const int gg = e / hd, d = e - gg * hd;
        float v[kProgMaxSplits];
#pragma unroll
        for (int sp = 0; sp < kProgMaxSplits; ++sp)
            v[sp] = sp < S ? __ldcg(rbase + (sp * group + gg) * kRec + d) : 0.f;
        float mx = -INFINITY;
        for (int sp = 0; sp < S; ++sp) mx = fmaxf(mx, ml[2 * (sp * group + gg)]);
        float num = 0.f, den = 0.f;
#pragma unroll
        for (int sp = 0; sp < kProgMaxSplits; ++sp) {
            if (sp >= S) break;
            const float rm = ml[2 * (sp * group + gg)];
            if (rm == -INFINITY) continue;   // an empty split
            const float f = expf(rm - mx);
            num += f * v[sp];
            den += f * ml[2 * (sp * group + gg) + 1];
        }
        A.out[(int64_t)(kvh * group + gg) * hd + d] = to_bf16_bits(num / den);
    }
    if (threadIdx.x == 0) counters[kvh] = 0u;
}

template <bool kBf16, bool kScaleF32>
__global__ void __launch_bounds__(kThreads, 1)
    decode_program_kernel(const ProgStep* __restrict__ steps, int n_steps, unsigned* bars, unsigned* attn_counters,
                          float* recs, uint32_t scr_off, uint32_t kv_off) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t sbase = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    if (sbase + kLowBytes > kRepWin) {   // uniform over CTAs: every CTA returns here
        if (threadIdx.x == 0) atomicExch(&g_mma_wait_timeout, 1);
        return;
    }
    const Bars B(sbase);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) init_bars(B);
    __syncthreads();

    uint32_t ring = 0, uc = 0;
    int u_begin, u_end;
    if (warp == kProducerWarp) {
        for (int s = 0; s < n_steps; ++s) {
            if (steps[s].kind != kStepLinear) continue;
            unit_range(steps[s].lin.total_units, u_begin, u_end);
            produce_linear<kScaleF32>(steps[s].lin, u_begin, u_end, B.full, B.empty, sbase + kBarBytes, lane, ring);
        }
        return;
    }
    if (warp == kReducerWarp) {
        // The consumers release a step's units only after the grid barrier before
        // it, and wait for this warp's last release before they arrive at the next.
        for (int s = 0; s < n_steps; ++s) {
            if (steps[s].kind != kStepLinear) continue;
            unit_range(steps[s].lin.total_units, u_begin, u_end);
            reduce_linear<kBf16, 1, true>(steps[s].lin, u_begin, u_end, smem, sbase, uc);
        }
        return;
    }
    uint2* rep = reinterpret_cast<uint2*>(smem + (kRepWin - sbase));
    uint2* cb_stage = reinterpret_cast<uint2*>(smem + kBarBytes + kStages * kStageBytes);
    float* scr = reinterpret_cast<float*>(smem + (scr_off - sbase));
    // the staged K / V rows follow the warp records (16-byte aligned)
    uint16_t* kst = reinterpret_cast<uint16_t*>(smem + (kv_off - sbase));
    if (n_steps > 0 && steps[0].kind == kStepLinear) {
        unit_range(steps[0].lin.total_units, u_begin, u_end);
        prepare_linear<kBf16>(steps[0].lin, u_begin, u_end, rep, cb_stage);
    }
    for (int s = 0; s < n_steps; ++s) {
        const ProgStep& T = steps[s];
        if (T.kind == kStepAttention) {
            if (T.attn.head_dim == 128) prestage_attention<4>(T.attn, kst, kst + kAttnRows * 128);
            else prestage_attention<2>(T.attn, kst, kst + kAttnRows * 64);
        }
        if (s > 0) grid_wait(&bars[s - 1], gridDim.x);
        if (T.kind == kStepLinear) {
            unit_range(T.lin.total_units, u_begin, u_end);
            if (u_begin < u_end) {
                run_linear<kBf16, 1, kScaleF32, true, true>(T.lin, u_begin, u_end, smem, sbase, ring, uc);
                // The step's outputs are complete once the reducer has released its
                // last unit (units are reduced in order).
                if (threadIdx.x == 0) mbar_wait(B.slot_free + 8 * ((uc - 1) % kSlots), ((uc - 1) / kSlots) & 1);
            }
        } else if (T.attn.head_dim == 128) {
            prog_attention<4>(T.attn, scr, kst, kst + kAttnRows * 128, recs, attn_counters, true);
        } else {
            prog_attention<2>(T.attn, scr, kst, kst + kAttnRows * 64, recs, attn_counters, true);
        }
        grid_arrive(&bars[s]);
        if (s + 1 < n_steps && steps[s + 1].kind == kStepLinear) {
            // The next store's codebook does not depend on the other CTAs.
            unit_range(steps[s + 1].lin.total_units, u_begin, u_end);
            prepare_linear<kBf16>(steps[s + 1].lin, u_begin, u_end, rep, cb_stage);
        }
    }
}

}  // namespace

// Bit 0: a bounded wait gave up (GEMV or decode program); bit 1: a decode
// program's position was outside its KV caches.
int mma_read_device_error(int* flag) {
    int w = 0, p = 0;
    if (cudaMemcpyFromSymbol(&w, g_mma_wait_timeout, sizeof(int)) != cudaSuccess ||
        cudaMemcpyFromSymbol(&p, g_prog_position_error, sizeof(int)) != cudaSuccess)
        return check_launch("read gemv_mma error flags");
    *flag = (w ? 1 : 0) | (p ? 2 : 0);
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

// Checks a fused GEMV and fills its parameters (everything but x_off); `fixed`
// = shared bytes below the staged activations, `xbytes` = their size.
static int build_mma_params(const StoreD* s, int count, const void* x, int x_dtype, int64_t m, int64_t ldx,
                            void* const* outs, const int64_t* ldo, int out_dtype, int prologue, int epilogue,
                            float eps, MmaParams& P, int& fixed, int64_t& xbytes) {
    if ((reinterpret_cast<uintptr_t>(x) & 7) || (ldx & 3))
        return set_error(EPQ_EALIGN, "linear: x must be 8-byte aligned with ldx a multiple of 4");
    const bool sf32 = s[0].scale_dtype == EPQ_F32;
    for (int i = 1; i < count; ++i)
        if ((s[i].scale_dtype == EPQ_F32) != sf32)
            return set_error(EPQ_EDTYPE, "linear: fused stores need one scale dtype");
    (void)x_dtype;
    const int parts = epilogue == EPQ_EPI_SILU_MUL ? 2 : 1;
    if (parts == 2 && (count != 2 || s[0].n != s[1].n))
        return set_error(EPQ_ESHAPE, "decode linear: the SiLU epilogue takes two stores of equal rows");
    if (epilogue == EPQ_EPI_RESIDUAL && count != 1)
        return set_error(EPQ_ESHAPE, "decode linear: the residual epilogue takes one store");
    if (epilogue != EPQ_EPI_STORE && out_dtype != x_dtype)
        return set_error(EPQ_EDTYPE, "decode linear: fused epilogues write the activation dtype");
    const int64_t kpad = s[0].ng * 128;
    xbytes = m * kpad * 2;
    const int slot_floats = parts * kConsumerWarps * 16 * (int)m;
    // Requested as if the dynamic block started at window address 0 (it starts a
    // little above, so the request always covers the layout).
    fixed = (int)kHighWin + kSlots * slot_floats * 4;
    P = MmaParams{};
    P.count = count;
    P.x = x;
    P.ldx = ldx;
    P.m = (int)m;
    P.k = (int)s[0].k;
    P.kpad = (int)kpad;
    P.out_dtype = out_dtype;
    P.chunks_per_unit = (int)cdiv(s[0].ng, kChunkGroups);
    P.parts = parts;
    P.prologue = prologue;
    P.epilogue = epilogue;
    P.eps = eps;
    P.slot_floats = slot_floats;
    int64_t units = 0;
    for (int i = 0; i < count; ++i) {
        MmaStore& S = P.st[i];
        const int esz = s[i].scale_dtype == EPQ_F32 ? 4 : 2;
        const int trc = make_tmap_2d_plain(&S.smap, s[i].scale, esz, s[i].rb * 16, s[i].ng, s[i].s_g, 16,
                                           kChunkGroups, "linear");
        if (trc != EPQ_OK) return trc;
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
        S.unit0 = parts == 2 ? 0 : (int)units;
        units += S.rb;
    }
    if (parts == 2) units = s[0].rb;
    if (units >= (int64_t(1) << 30)) return set_error(EPQ_EUNSUPPORTED, "linear: too many rows");
    P.total_units = (int)units;
    return EPQ_OK;
}

int launch_linear_mma_fused(const StoreD* s, int count, const void* x, int x_dtype, int64_t m, int64_t ldx,
                            void* const* outs, const int64_t* ldo, int out_dtype, int prologue, int epilogue,
                            float eps, cudaStream_t st) {
    const bool bf = x_dtype == EPQ_BF16;
    const int nt = m > 8 ? 2 : 1;
    MmaParams P;
    int fixed = 0;
    int64_t xbytes = 0;
    {
        const int rc = build_mma_params(s, count, x, x_dtype, m, ldx, outs, ldo, out_dtype, prologue, epilogue, eps,
                                        P, fixed, xbytes);
        if (rc != EPQ_OK) return rc;
    }
    const bool sf32 = s[0].scale_dtype == EPQ_F32;
    const bool xsm = xbytes <= kMaxXSmem && fixed + xbytes <= kMaxSmem;
    if (prologue == EPQ_PRO_RMSNORM && !xsm)
        return set_error(EPQ_EUNSUPPORTED, "decode linear: RMSNorm prologue needs m*k*2 <= %d bytes", kMaxXSmem);
    if (fixed > kMaxSmem)
        return set_error(EPQ_EUNSUPPORTED, "decode linear: m=%lld needs %d bytes of shared memory", (long long)m,
                         fixed);
    const int smem = fixed + (xsm ? (int)xbytes : 0);
    P.x_off = fixed;
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
    {
        const int arc = set_smem_limit(reinterpret_cast<const void*>(kern), kMaxSmem,
                                       "cudaFuncSetAttribute(gemv_mma_kernel)");
        if (arc != EPQ_OK) return arc;
    }
    int grid = device_sms();
    if (grid > P.total_units) grid = P.total_units;

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

int launch_linear_mma(const StoreD* s, int count, const void* x, int x_dtype, int64_t m, int64_t ldx,
                      void* const* outs, const int64_t* ldo, int out_dtype, cudaStream_t st) {
    return launch_linear_mma_fused(s, count, x, x_dtype, m, ldx, outs, ldo, out_dtype, EPQ_PRO_NONE,
                                   EPQ_EPI_STORE, 0.f, st);
}

}  // namespace epq

using namespace epq;

extern "C" int epq_decode_linear(const epq_store* stores, int32_t count, const void* x, int32_t x_dtype,
                                 int64_t m, int64_t ldx, int32_t prologue, float eps, void* const* outs,
                                 const int64_t* ldo, int32_t epilogue, void* stream) {
    if (!stores || !x || !outs || count < 1 || count > kLutMaxStores || m < 1 || m > 16)
        return set_error(EPQ_EINVAL, "epq_decode_linear: bad arguments");
    if (prologue != EPQ_PRO_NONE && prologue != EPQ_PRO_RMSNORM)
        return set_error(EPQ_EINVAL, "epq_decode_linear: prologue=%d", prologue);
    if (epilogue != EPQ_EPI_STORE && epilogue != EPQ_EPI_RESIDUAL && epilogue != EPQ_EPI_SILU_MUL)
        return set_error(EPQ_EINVAL, "epq_decode_linear: epilogue=%d", epilogue);
    if (x_dtype != EPQ_BF16 && x_dtype != EPQ_F16)
        return set_error(EPQ_EDTYPE, "epq_decode_linear: activations must be bf16 or f16");
    StoreD s[kLutMaxStores];
    for (int i = 0; i < count; ++i) {
        const int rc = make_store(&stores[i], &s[i], "epq_decode_linear");
        if (rc != EPQ_OK) return rc;
        if (!mma_eligible(s[i], m, x_dtype))
            return set_error(EPQ_ELAYOUT,
                             "epq_decode_linear: store %d is not an EPQ_LAYOUT_MMA16 vec-4 group-128 store "
                             "with group-major f16/f32 scales",
                             i);
        if (s[i].k != s[0].k) return set_error(EPQ_ESHAPE, "epq_decode_linear: stores differ in k");
        if (!outs[i]) return set_error(EPQ_EINVAL, "epq_decode_linear: output %d is NULL", i);
        if (ldo && ldo[i] < s[i].n) return set_error(EPQ_ESHAPE, "epq_decode_linear: ldo[%d] < n", i);
    }
    if (ldx < s[0].k) return set_error(EPQ_ESHAPE, "epq_decode_linear: ldx < k");
    return launch_linear_mma_fused(s, count, x, x_dtype, m, ldx, outs, ldo, x_dtype, prologue, epilogue, eps,
                                   static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------------------
// decode program (host side)
// ---------------------------------------------------------------------------
struct epq_program {
    std::vector<ProgStep> steps;
    bool sf32 = false, sf32_set = false, finalized = false;
    int max_xbytes = 0, max_slot_floats = 0;
    int max_kv = 0, max_heads = 0, max_hd = 0;
    int grid = 0, splits = 1;
    int64_t steps_bytes = 0, bars_off = 0, counters_off = 0, recs_off = 0, total_bytes = 0;
    uint8_t* ws = nullptr;
};

namespace epq {
namespace {

int program_layout(epq_program* p) {
    p->grid = device_sms();
    if (p->grid <= 0) return check_launch("decode program: SM count");
    p->splits = 1;
    if (p->max_kv > 0) p->splits = std::max(1, std::min(kProgMaxSplits, p->grid / p->max_kv));
    auto up = [](int64_t v) { return (v + 255) & ~int64_t(255); };
    const int64_t n = (int64_t)p->steps.size();
    p->steps_bytes = up(n * (int64_t)sizeof(ProgStep));
    p->bars_off = p->steps_bytes;
    p->counters_off = p->bars_off + up(std::max<int64_t>(n, 1) * 4);
    p->recs_off = p->counters_off + up(std::max(p->max_kv, 1) * 4);
    p->total_bytes = p->recs_off + up((int64_t)p->splits * std::max(p->max_heads, 1) * (p->max_hd + 2) * 4);
    return EPQ_OK;
}

// Shared bytes: the GEMV layout (replicas, slots), the staged activations of the
// widest step, the attention scratch (16 warp records + a flag), then the
// attention's staged K / V rows.
int program_smem(const epq_program* p, int* x_off, int* scr_off, int* kv_off) {
    const int fixed = (int)kHighWin + kSlots * std::max(p->max_slot_floats, 1) * 4;
    const int hd = std::max(p->max_hd, 64);
    *x_off = fixed;
    *scr_off = fixed + ((p->max_xbytes + 15) & ~15);
    *kv_off = *scr_off + (((kConsumerWarps * (hd + 2) + 4) * 4 + 15) & ~15);
    return *kv_off + (p->max_hd > 0 ? 2 * kAttnRows * hd * 2 : 0);
}

}  // namespace
}  // namespace epq

extern "C" int epq_program_create(epq_program** out) {
    if (!out) return set_error(EPQ_EINVAL, "epq_program_create: out is NULL");
    *out = new (std::nothrow) epq_program();
    if (!*out) return set_error(EPQ_EINVAL, "epq_program_create: out of host memory");
    return EPQ_OK;
}

extern "C" void epq_program_destroy(epq_program* p) { delete p; }

extern "C" int epq_program_add_linear(epq_program* p, const epq_store* stores, int32_t count, const void* x,
                                      int64_t ldx, int32_t prologue, float eps, void* const* outs,
                                      const int64_t* ldo, int32_t epilogue) {
    if (!p || !stores || !x || !outs || count < 1 || count > kLutMaxStores)
        return set_error(EPQ_EINVAL, "epq_program_add_linear: bad arguments");
    if (p->finalized) return set_error(EPQ_EINVAL, "epq_program_add_linear: the program is finalized");
    if (prologue != EPQ_PRO_NONE && prologue != EPQ_PRO_RMSNORM)
        return set_error(EPQ_EINVAL, "epq_program_add_linear: prologue=%d", prologue);
    if (epilogue != EPQ_EPI_STORE && epilogue != EPQ_EPI_RESIDUAL && epilogue != EPQ_EPI_SILU_MUL)
        return set_error(EPQ_EINVAL, "epq_program_add_linear: epilogue=%d", epilogue);
    StoreD s[kLutMaxStores];
    for (int i = 0; i < count; ++i) {
        const int rc = make_store(&stores[i], &s[i], "epq_program_add_linear");
        if (rc != EPQ_OK) return rc;
        if (!mma_eligible(s[i], 1, EPQ_BF16))
            return set_error(EPQ_ELAYOUT,
                             "epq_program_add_linear: store %d is not an EPQ_LAYOUT_MMA16 vec-4 group-128 store "
                             "with group-major f16/f32 scales",
                             i);
        if (s[i].k != s[0].k) return set_error(EPQ_ESHAPE, "epq_program_add_linear: stores differ in k");
        if (!outs[i]) return set_error(EPQ_EINVAL, "epq_program_add_linear: output %d is NULL", i);
        if (ldo && ldo[i] < s[i].n) return set_error(EPQ_ESHAPE, "epq_program_add_linear: ldo[%d] < n", i);
        if ((reinterpret_cast<uintptr_t>(outs[i]) & 1))
            return set_error(EPQ_EALIGN, "epq_program_add_linear: output %d is not 2-byte aligned", i);
    }
    if (ldx < s[0].k) return set_error(EPQ_ESHAPE, "epq_program_add_linear: ldx < k");
    const bool sf32 = s[0].scale_dtype == EPQ_F32;
    if (p->sf32_set && sf32 != p->sf32)
        return set_error(EPQ_EDTYPE, "epq_program_add_linear: every step needs the same scale dtype");
    ProgStep T{};
    T.kind = kStepLinear;
    int fixed = 0;
    int64_t xbytes = 0;
    const int rc = build_mma_params(s, count, x, EPQ_BF16, 1, ldx, outs, ldo, EPQ_BF16, prologue, epilogue, eps,
                                    T.lin, fixed, xbytes);
    if (rc != EPQ_OK) return rc;
    if (xbytes > kMaxXSmem)
        return set_error(EPQ_EUNSUPPORTED, "epq_program_add_linear: k=%lld is wider than %d staged values",
                         (long long)s[0].k, kMaxXSmem / 2);
    p->sf32 = sf32;
    p->sf32_set = true;
    p->max_xbytes = std::max(p->max_xbytes, (int)xbytes);
    p->max_slot_floats = std::max(p->max_slot_floats, T.lin.slot_floats);
    p->steps.push_back(T);
    return EPQ_OK;
}

extern "C" int epq_program_add_attention(epq_program* p, const void* q, const void* k, const void* v,
                                         const int64_t* pos, int32_t heads, int32_t kv_heads, int32_t head_dim,
                                         const float* cos_tab, const float* sin_tab, void* k_cache, void* v_cache,
                                         int64_t max_len, int32_t qk_norm, float eps, float scale, void* out) {
    if (!p || !q || !k || !v || !pos || !cos_tab || !sin_tab || !k_cache || !v_cache || !out)
        return set_error(EPQ_EINVAL, "epq_program_add_attention: NULL pointer");
    if (p->finalized) return set_error(EPQ_EINVAL, "epq_program_add_attention: the program is finalized");
    if (head_dim != 64 && head_dim != 128)
        return set_error(EPQ_EUNSUPPORTED, "epq_program_add_attention: head_dim=%d (64 or 128)", head_dim);
    if (kv_heads < 1 || heads < kv_heads || heads % kv_heads)
        return set_error(EPQ_ESHAPE, "epq_program_add_attention: heads=%d kv_heads=%d", heads, kv_heads);
    const int group = heads / kv_heads;
    if (group > kConsumerWarps || kConsumerWarps % group)
        return set_error(EPQ_EUNSUPPORTED, "epq_program_add_attention: %d query heads per kv head (1, 2, 4, 8, 16)",
                         group);
    if (max_len < 1) return set_error(EPQ_ESHAPE, "epq_program_add_attention: max_len=%lld", (long long)max_len);
    const uintptr_t al = reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
                         reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(k_cache) |
                         reinterpret_cast<uintptr_t>(v_cache) | reinterpret_cast<uintptr_t>(out);
    if (al & 1) return set_error(EPQ_EALIGN, "epq_program_add_attention: bf16 tensors must be 2-byte aligned");
    if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15)
        return set_error(EPQ_EALIGN, "epq_program_add_attention: the KV caches must be 16-byte aligned");
    ProgStep T{};
    T.kind = kStepAttention;
    AttnStep& A = T.attn;
    A.q = static_cast<const uint16_t*>(q);
    A.k = static_cast<const uint16_t*>(k);
    A.v = static_cast<const uint16_t*>(v);
    A.k_cache = static_cast<uint16_t*>(k_cache);
    A.v_cache = static_cast<uint16_t*>(v_cache);
    A.pos = pos;
    A.max_len = max_len;
    A.cos_t = cos_tab;
    A.sin_t = sin_tab;
    A.out = static_cast<uint16_t*>(out);
    A.heads = heads;
    A.kv_heads = kv_heads;
    A.head_dim = head_dim;
    A.qk_norm = qk_norm;
    A.eps = eps;
    A.scale = scale;
    p->max_kv = std::max(p->max_kv, (int)kv_heads);
    p->max_heads = std::max(p->max_heads, (int)heads);
    p->max_hd = std::max(p->max_hd, (int)head_dim);
    p->steps.push_back(T);
    return EPQ_OK;
}

extern "C" int64_t epq_program_workspace_bytes(epq_program* p) {
    if (!p) return set_error(EPQ_EINVAL, "epq_program_workspace_bytes: NULL program");
    const int rc = program_layout(p);
    if (rc != EPQ_OK) return rc;
    return p->total_bytes;
}

extern "C" int epq_program_finalize(epq_program* p, void* workspace, int64_t workspace_bytes, void* stream) {
    if (!p || !workspace) return set_error(EPQ_EINVAL, "epq_program_finalize: NULL argument");
    if (p->steps.empty()) return set_error(EPQ_EINVAL, "epq_program_finalize: the program has no steps");
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
        return set_error(EPQ_EALIGN, "epq_program_finalize: workspace must be 256-byte aligned");
    int rc = program_layout(p);
    if (rc != EPQ_OK) return rc;
    if (workspace_bytes < p->total_bytes)
        return set_error(EPQ_ESHAPE, "epq_program_finalize: workspace of %lld bytes, %lld needed",
                         (long long)workspace_bytes, (long long)p->total_bytes);
    int x_off = 0, scr_off = 0, kv_off = 0;
    if (program_smem(p, &x_off, &scr_off, &kv_off) > kMaxSmem)
        return set_error(EPQ_EUNSUPPORTED, "epq_program_finalize: needs more shared memory than an SM has");
    for (ProgStep& T : p->steps) {
        if (T.kind == kStepLinear) T.lin.x_off = x_off;
        else T.attn.splits = p->splits;
    }
    p->ws = static_cast<uint8_t*>(workspace);
    // The table must outlive the copy: it stays in the program object.
    if (cudaMemcpyAsync(p->ws, p->steps.data(), p->steps.size() * sizeof(ProgStep), cudaMemcpyHostToDevice,
                        static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return check_launch("epq_program_finalize: step table copy");
    if (cudaMemsetAsync(p->ws + p->counters_off, 0, p->recs_off - p->counters_off,
                        static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return check_launch("epq_program_finalize: counters");
    if (cudaStreamSynchronize(static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return check_launch("epq_program_finalize");
    p->finalized = true;
    return EPQ_OK;
}

extern "C" int epq_program_run(epq_program* p, void* stream) {
    if (!p) return set_error(EPQ_EINVAL, "epq_program_run: NULL program");
    if (!p->finalized) return set_error(EPQ_EINVAL, "epq_program_run: finalize the program first");
    if (device_sms() != p->grid)
        return set_error(EPQ_EINVAL, "epq_program_run: the program was finalized for another device");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int x_off = 0, scr_off = 0, kv_off = 0;
    const int smem = program_smem(p, &x_off, &scr_off, &kv_off);
    using KernT = void (*)(const ProgStep*, int, unsigned*, unsigned*, float*, uint32_t, uint32_t);
    static const KernT kernels[2] = {decode_program_kernel<true, false>, decode_program_kernel<true, true>};
    const KernT kern = kernels[p->sf32 ? 1 : 0];
    {
        const int arc = set_smem_limit(reinterpret_cast<const void*>(kern), kMaxSmem,
                                       "cudaFuncSetAttribute(decode_program_kernel)");
        if (arc != EPQ_OK) return arc;
    }
    // Step counters start from zero every token (one memset node in a graph).
    if (cudaMemsetAsync(p->ws + p->bars_off, 0, p->counters_off - p->bars_off, st) != cudaSuccess)
        return check_launch("epq_program_run: step counters");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p->grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;   // every CTA resident: the step counters are grid barriers
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const ProgStep* steps = reinterpret_cast<const ProgStep*>(p->ws);
    unsigned* bars = reinterpret_cast<unsigned*>(p->ws + p->bars_off);
    unsigned* counters = reinterpret_cast<unsigned*>(p->ws + p->counters_off);
    float* recs = reinterpret_cast<float*>(p->ws + p->recs_off);
    if (cudaLaunchKernelEx(&cfg, kern, steps, (int)p->steps.size(), bars, counters, recs, (uint32_t)scr_off,
                           (uint32_t)kv_off) != cudaSuccess)
        return check_launch("decode_program_kernel");
    return check_launch("decode_program_kernel");
}
