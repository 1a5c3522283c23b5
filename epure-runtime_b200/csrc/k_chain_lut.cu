// Persistent chain kernel: a whole sequence of batch-1 packed linears (one
// decode token through a decoder's packed linears) in ONE cooperative launch.
//
// Reference op per step: epure/kernels/_triton.py:56-107 (the table-mode fused
// dequant-matmul), applied in sequence as PackedLinear.forward calls
// (epure/runtime.py:98-126) where each step's input is an earlier step's output.
//
// Why one launch.  At batch 1 the packed weights of one linear are 1-30 MB; a
// kernel that streams that much spends a fixed ~3 us filling and draining the
// memory pipeline, which for 128 dependent launches per token costs more than
// the whole HBM roofline.  Here a producer warp per SM streams the weights of
// every step through a 3-stage TMA ring (cp.async.bulk + mbarriers, each copy to
// this CTA only) without ever waiting for activations -- weights are static -- so
// HBM keeps streaming across step boundaries; only the consumers wait for their
// inputs from the previous step (see "Synchronisation" below).
//
// Inner loop (per index byte: one PRMT, one LDS.32, one FADD).  For one scale
// group (32 index positions) the consumers build an activation table
// T[e][j] = dot(cb[e, 0:4], x[4j : 4j+4]) in shared memory (fp32, 256 B per
// entry e: 2 slots x 32 positions), so a row's group sum is sum_j T[idx[r, j]][j]
// and the scale multiplies it once.  Indices arrive in EPQ_LAYOUT_TILED order
// (16 rows x 32 positions per 512-byte tile); a team of 8 lanes owns a tile,
// each lane 4 positions (rotated per team: the 32 lanes of a warp always hit 32
// different banks), and a 3-step butterfly leaves each lane with 2 row sums.
//
// Synchronisation without a grid barrier on the critical path.  Partial sums
// are written as 8-byte (value, step tag) elements into a ring of three
// buffers; a consumer polls exactly the partials its input slice needs until
// they carry the previous step's tag (an aligned 8-byte access is single-copy
// atomic), so a step starts as soon as its own inputs exist.  A per-step
// arrival counter, bumped (relaxed) when a CTA has consumed its inputs, is
// checked only before a CTA first writes a buffer again, two steps later.
//
// Split over k without a reduction tail.  A step's tiles are ordered (store,
// group, row block) and each CTA takes a contiguous range, chosen on the host
// to balance tiles against table builds (a CTA whose range crosses a group
// boundary builds one table more), so it covers about one group of many rows
// and writes scaled group sums to a partial buffer [group][row].  Nobody reduces them in that step: the NEXT
// step's consumers add the partials of exactly the input columns they need
// while staging their activation slice (deterministic order), and after the
// last step all CTAs reduce the final output rows.  Partial buffers ping-pong
// between steps.
//
// Safety: every mbarrier wait, tag poll and counter spin is bounded; a wait
// that gives up sets g_chain_error (read by epq_device_error) and the kernel
// runs to completion.  The launch is cooperative, so all CTAs are co-resident.
#include <climits>
#include <cstring>
#include <vector>

#include <mutex>

#include "epq_common.cuh"

namespace epq {

struct ChainStoreD {
    const uint8_t* idx;   // EPQ_LAYOUT_TILED
    const void* scale;    // group-major, rows padded to 16: scale(r, g) at g * s_g + r
    const void* cb;
    int64_t s_g;
    int64_t part_off;     // offset (floats) of this store's partials in a partial buffer
    int cb_dtype, scale_f32, levels, n;
    int rb, ng, tile0, pad;
};

struct ChainStepD {
    ChainStoreD st[kLutMaxStores];
    int count, feed, k, kpos;
    int total_tiles;
    int remote;           // tensor parallel: this step's input is summed over every rank
    int64_t range_off;    // workspace offset of int32 [grid + 1]: CTA c takes tiles [r[c], r[c+1])
};

constexpr int kMaxTp = 8;

struct ChainHeaderD {
    int n_steps, grid;
    int64_t part_floats;              // elements per partial buffer (8 bytes each: value, tag)
    int64_t steps_off, ctr_off, part_off0, part_off1, part_off2;   // byte offsets in the workspace
    int64_t xred_off, xred_elems;     // 3 buffers of per-rank input-slice sums (tensor parallel)
    int64_t xfin_off, xfin_elems;     // per-rank sums of the final output rows (tensor parallel)
    int tp_world, tp_rank;            // 1, 0 without tensor parallelism
    int final_remote, pad;
    int64_t peer_ws[kMaxTp];          // every rank's workspace as mapped in this process
};

namespace {

constexpr int kConsumerWarps = 16;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;
constexpr int kRing = 3;
constexpr int kChunkTiles = 64;                                    // one tile per 8-lane team
constexpr uint32_t kStageIdx = kChunkTiles * 512;                  // 32 KB of index tiles
constexpr uint32_t kStageBytes = kStageIdx + kChunkTiles * 64;     // + scales (<= fp32)
constexpr int kXGroups = kConsumerWarps / 2;     // activation staging: parts (warp pairs)
static_assert(kConsumerWarps == 16, "staging: 2 column halves x 8 parts of warps");
// Shared-window addresses (the dynamic block starts at a small offset `base`).
constexpr uint32_t kXsOff = 8192;      // from base: 2 x codebook [1024] fp32 below, then
                                       // 2 x activation slice sums [kXGroups][128] fp32
constexpr uint32_t kBarOff = kXsOff + 2 * kXGroups * 512;  // from base: full[kRing], empty[kRing]
constexpr uint32_t kMiscOff = kBarOff + 128;               // from base: broadcast words
constexpr uint32_t kDescOff = kMiscOff + 64;               // from base: 3 step descriptors (ring)
constexpr uint32_t kLowStages = 26624; // window address of stage 0
constexpr uint32_t kTBase = 65536;     // window address of T (low 16 bits zero for the PRMT trick)
constexpr uint32_t kHighStages = 131072;   // window address of stages 1..2
constexpr uint32_t kWindowEnd = kHighStages + 2 * kStageBytes;
static_assert(kLowStages + kStageBytes <= kTBase, "stage 0 must end below the table");
constexpr int kDynSmem = (int)kWindowEnd;
constexpr uint32_t kWaitLimit = 1u << 22;   // mbarrier polls
constexpr uint32_t kSpinLimit = 1u << 22;   // grid-barrier polls

// from base: per-rank slice sums of a tensor-parallel step [kMaxTp][128] fp32
constexpr uint32_t kXrOff = kDescOff + 3 * (uint32_t)sizeof(ChainStepD);
static_assert(kXrOff % 16 == 0, "rank slice buffer alignment");

__device__ int g_chain_error = 0;

__device__ __forceinline__ uint32_t stage_addr(int s) {
    return s == 0 ? kLowStages : kHighStages + (s - 1) * kStageBytes;
}

__device__ __forceinline__ float lds_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ float4 lds_f32x4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr));
    return v;
}
__device__ __forceinline__ void sts_f32(uint32_t addr, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr));
    return v;
}
__device__ __forceinline__ float lds_scale(uint32_t addr, bool f32) {
    if (f32) return lds_f32(addr);
    unsigned short h;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(addr));
    return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
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
// Bounded wait; once any wait in the kernel has given up, later waits return at once.
__device__ __forceinline__ void mbar_wait(uint32_t bar, uint32_t parity) {
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return;
        if ((i & 1023u) == 1023u && *reinterpret_cast<volatile int*>(&g_chain_error)) return;
    }
    atomicExch(&g_chain_error, 1);
}
// The weight stream is read once per token: evict-first in L2, so that it does not
// push the split-k partial sums (rewritten every token) out to DRAM.
__device__ __forceinline__ uint64_t evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void bulk_g2s_stream(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar,
                                                uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(pol)
        : "memory");
}
// Partial sums travel as 8-byte elements (fp32 value, 32-bit step tag); an aligned
// 8-byte access is single-copy atomic, so a reader that sees the expected tag sees
// the value written with it.
__device__ __forceinline__ uint64_t tagged(float v, uint32_t tag) {
    return (uint64_t)__float_as_uint(v) | ((uint64_t)tag << 32);
}
__device__ __forceinline__ ulonglong2 ldcg_u64x2(const uint64_t* p) {
    ulonglong2 v;
    asm volatile("ld.global.cg.v2.u64 {%0,%1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t ldcg_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.global.cg.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void stg_u64x2(uint64_t* p, uint64_t a, uint64_t b) {
    asm volatile("st.global.v2.u64 [%0], {%1,%2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
// Split-k partial sums are re-read by the next step and rewritten a few steps
// later: evict-last in L2, so they stay there instead of being written back.
__device__ __forceinline__ uint64_t evict_last_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void stg_u64x2_keep(uint64_t* p, uint64_t a, uint64_t b, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.v2.u64 [%0], {%1,%2}, %3;" ::"l"(p), "l"(a), "l"(b), "l"(pol) : "memory");
}
__device__ __forceinline__ ulonglong2 ldsys_u64x2(const uint64_t* p) {   // peer or own memory, no caching
    ulonglong2 v;
    asm volatile("ld.volatile.global.v2.u64 {%0,%1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint64_t ldsys_u64(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_sys_add(unsigned* p, unsigned v) {
    asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t tag_of(uint64_t v) { return (uint32_t)(v >> 32); }
__device__ __forceinline__ float val_of(uint64_t v) { return __uint_as_float((uint32_t)v); }
constexpr uint32_t kTagSpinLimit = 1u << 22;   // polls of one not-yet-written partial

__device__ __forceinline__ void consumers_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumers) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// Grid barrier: until every CTA has counted step `c` for this run (bounded).
__device__ __forceinline__ void grid_wait(const unsigned* c, unsigned target) {
    for (uint32_t it = 0; it < kSpinLimit; ++it) {
        if ((int)(ld_acquire(c) - target) >= 0) return;
        if ((it & 255u) == 255u && *reinterpret_cast<volatile int*>(&g_chain_error)) return;
    }
    atomicExch(&g_chain_error, 1);
}

// Chunk iterator over a CTA's tile range of one step (identical in producer and
// consumers).  Tiles run (store, group, row block); a chunk never crosses a
// (store, group) boundary.  The position is kept incrementally (one division
// per step, at the start).
struct ChunkIt {
    int t, t_end, si, g, rb;
    __device__ void start(const ChainStepD& S, int t0, int t1) {
        t = t0;
        t_end = t1;
        si = 0;
        while (si + 1 < S.count && t0 >= S.st[si + 1].tile0) ++si;
        const int local = t0 - S.st[si].tile0;
        g = local / S.st[si].rb;
        rb = local - g * S.st[si].rb;
    }
    __device__ bool next(const ChainStepD& S, int& csi, int& cg, int& rb0, int& nt) {
        if (t >= t_end) return false;
        const int crb = S.st[si].rb;
        csi = si;
        cg = g;
        rb0 = rb;
        nt = min(kChunkTiles, min(t_end - t, crb - rb));
        t += nt;
        rb += nt;
        if (rb == crb) {
            rb = 0;
            if (++g == S.st[si].ng) {
                g = 0;
                ++si;
            }
        }
        return true;
    }
};

__global__ void __launch_bounds__(kThreads, 1) chain_kernel(const uint8_t* __restrict__ ws, const void* x0,
                                                            int x_dtype, void* out, int out_dtype) {
    extern __shared__ __align__(128) uint8_t smem[];
    const uint32_t base = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    if (base + kXrOff + kMaxTp * 512u > kLowStages ||
        (int)gridDim.x != reinterpret_cast<const int*>(ws)[1]) {
        // placement the addresses below rely on, or a grid other than the one
        // the descriptors were built for
        if (threadIdx.x == 0) atomicExch(&g_chain_error, 2);
        return;
    }
    const ChainHeaderD& H = *reinterpret_cast<const ChainHeaderD*>(ws);
    const ChainStepD* steps = reinterpret_cast<const ChainStepD*>(ws + H.steps_off);
    unsigned* ctr = reinterpret_cast<unsigned*>(const_cast<uint8_t*>(ws) + H.ctr_off);  // [n_steps] + done + gen
    uint64_t* part[3] = {reinterpret_cast<uint64_t*>(const_cast<uint8_t*>(ws) + H.part_off0),
                         reinterpret_cast<uint64_t*>(const_cast<uint8_t*>(ws) + H.part_off1),
                         reinterpret_cast<uint64_t*>(const_cast<uint8_t*>(ws) + H.part_off2)};
    const int n_steps = H.n_steps;
    const int G = gridDim.x;
    const uint32_t bar_full = base + kBarOff, bar_empty = bar_full + 8 * kRing;
    unsigned* misc = reinterpret_cast<unsigned*>(smem + kMiscOff);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kRing; ++s) {
            mbar_init(bar_full + 8 * s, 1);
            mbar_init(bar_empty + 8 * s, kConsumerWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        misc[0] = *reinterpret_cast<volatile unsigned*>(&ctr[n_steps + 1]);   // run generation
    }
    __syncthreads();
    const int world = H.tp_world, my_rank = H.tp_rank;
    const unsigned target = (misc[0] + 1u) * (unsigned)G * (unsigned)world;
    // Step j's partials carry tag gen * n_steps + j + 1 (never 0: buffers start zeroed).
    const unsigned tag_base = misc[0] * (unsigned)n_steps + 1u;

    if (warp == kConsumerWarps) {
        // ---------------- producer: stream every step's tiles into the ring ----------------
        const uint64_t pol = evict_first_policy();
        int i = 0;
        for (int j = 0; j < n_steps; ++j) {
            const ChainStepD& S = steps[j];
            const int* rg = reinterpret_cast<const int*>(ws + S.range_off);
            ChunkIt it;
            it.start(S, rg[blockIdx.x], rg[blockIdx.x + 1]);
            int si, g, rb0, nt;
            while (it.next(S, si, g, rb0, nt)) {
                const int stage = i % kRing;
                if (i >= kRing) mbar_wait(bar_empty + 8 * stage, ((i / kRing) - 1) & 1);
                const ChainStoreD& C = S.st[si];
                const uint32_t esz = C.scale_f32 ? 4u : 2u;
                const uint32_t dst = stage_addr(stage);
                if (lane == 0) {
                    mbar_expect_tx(bar_full + 8 * stage, nt * 512u + nt * 16u * esz);
                    bulk_g2s_stream(dst, C.idx + ((int64_t)g * C.rb + rb0) * 512, nt * 512u, bar_full + 8 * stage,
                                    pol);
                    bulk_g2s_stream(dst + kStageIdx,
                                    static_cast<const char*>(C.scale) + ((int64_t)g * C.s_g + (int64_t)rb0 * 16) * esz,
                                    nt * 16u * esz, bar_full + 8 * stage, pol);
                }
                __syncwarp();
                ++i;
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    const uint64_t keep_pol = evict_last_policy();
    const int team = lane >> 3, tl = lane & 7;
    // Double-buffered staging (parity flips per change), so a new table's inputs
    // can be written while no warp still needs the previous ones.
    float* cbf_buf = reinterpret_cast<float*>(smem);                          // [2][256][4]
    float* xs_buf = reinterpret_cast<float*>(smem + kXsOff);                  // [2][kXGroups][128]
    int cbp = 0, xsp = 0;
    // T ([256][2][32] fp32) lives at window address kTBase and is addressed directly.
    // Codebooks are fetched one step ahead into registers (values 2t, 2t+1 of
    // each store of the step), so building a table never waits on DRAM.
    uint2 cb_raw[kLutMaxStores];
    float2 cb_cur[kLutMaxStores];
    // Step descriptors are read from a 3-slot ring in shared memory (slot j % 3):
    // each is loaded into registers two steps ahead and stored one step ahead, so
    // no consumer waits on the workspace for them.
    const ChainStepD* sdesc = reinterpret_cast<const ChainStepD*>(smem + kDescOff);
    uint32_t* sdw = reinterpret_cast<uint32_t*>(smem + kDescOff);
    constexpr int kDescWords = (int)(sizeof(ChainStepD) / 4);
    static_assert(sizeof(ChainStepD) % 4 == 0 && kDescWords <= kConsumers, "descriptor words");
    const uint32_t* gsteps = reinterpret_cast<const uint32_t*>(steps);
    auto cb_prefetch = [&](int jj) {
#pragma unroll
        for (int q = 0; q < kLutMaxStores; ++q) cb_raw[q] = make_uint2(0u, 0u);
        if (jj >= n_steps) return;
        const ChainStepD& N = sdesc[jj % 3];
        const int e = 2 * threadIdx.x;
#pragma unroll
        for (int q = 0; q < kLutMaxStores; ++q) {
            if (q < N.count && e < N.st[q].levels * 4) {
                const int dt = N.st[q].cb_dtype;
                const uint8_t* p = static_cast<const uint8_t*>(N.st[q].cb) + (int64_t)e * (dt == EPQ_F32 ? 4 : 2);
                if (dt == EPQ_F32)
                    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(cb_raw[q].x), "=r"(cb_raw[q].y) : "l"(p));
                else
                    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(cb_raw[q].x) : "l"(p));
            }
        }
    };
    auto cb_promote = [&](int jj) {
        const ChainStepD& N = sdesc[jj % 3];
#pragma unroll
        for (int q = 0; q < kLutMaxStores; ++q) {
            const int dt = q < N.count ? N.st[q].cb_dtype : EPQ_F32;
            if (dt == EPQ_F32) {
                cb_cur[q] = make_float2(__uint_as_float(cb_raw[q].x), __uint_as_float(cb_raw[q].y));
            } else if (dt == EPQ_F16) {
                const __half2 h = *reinterpret_cast<const __half2*>(&cb_raw[q].x);
                cb_cur[q] = __half22float2(h);
            } else {
                const __nv_bfloat162 h = *reinterpret_cast<const __nv_bfloat162*>(&cb_raw[q].x);
                cb_cur[q] = __bfloat1622float2(h);
            }
        }
    };
    uint32_t dreg = 0;
    if (threadIdx.x < kDescWords) {
        sdw[threadIdx.x] = gsteps[threadIdx.x];
        if (n_steps > 1) sdw[kDescWords + threadIdx.x] = gsteps[kDescWords + threadIdx.x];
        if (n_steps > 2) dreg = __ldg(gsteps + 2 * kDescWords + threadIdx.x);
    }
    consumers_sync();
    cb_prefetch(0);
    // This CTA's tile range of the current and of the next step (loaded a step ahead).
    int rcur0, rcur1, rnext0 = 0, rnext1 = 0;
    {
        const int* rg = reinterpret_cast<const int*>(ws + sdesc[0].range_off);
        rcur0 = __ldg(rg + blockIdx.x);
        rcur1 = __ldg(rg + blockIdx.x + 1);
    }

    int i = 0, slot = 0;
    for (int j = 0; j < n_steps; ++j) {
        const ChainStepD& S = sdesc[j % 3];
        // The step's bookkeeping (codebooks, descriptor ring, next range) runs once,
        // after the first poll round of the step's first input slice has been issued,
        // so that it overlaps that round trip (or at the end for a CTA without tiles).
        bool booked = false;
        auto bookkeeping = [&]() {
            cb_promote(j);
            if (j >= 1 && j + 1 < n_steps && threadIdx.x < kDescWords) {
                // step j+1 into the slot of step j-2 (no longer read); published by the barrier below
                sdw[((j + 1) % 3) * kDescWords + threadIdx.x] = dreg;
                if (j + 2 < n_steps) dreg = __ldg(gsteps + (j + 2) * kDescWords + threadIdx.x);
            }
            if (j > 0) consumers_sync();   // publishes the descriptor slot written above
            cb_prefetch(j + 1);
            if (j + 1 < n_steps) {
                const int* rgn = reinterpret_cast<const int*>(ws + sdesc[(j + 1) % 3].range_off);
                rnext0 = __ldg(rgn + blockIdx.x);
                rnext1 = __ldg(rgn + blockIdx.x + 1);
            }
            booked = true;
        };
        // Input of this step: x0 (step 0) or the partials of step j-1's feed store.
        const ChainStepD* P = j > 0 ? &sdesc[(j - 1) % 3] : nullptr;
        const uint64_t* pin = j > 0 ? part[(j - 1) % 3] + P->st[P->feed].part_off : nullptr;
        const uint32_t want = tag_base + (uint32_t)(j - 1);
        const int64_t pin_stride = j > 0 ? (int64_t)P->st[P->feed].rb * 16 : 0;
        const int pin_ng = j > 0 ? P->st[P->feed].ng : 0;
        uint64_t* pout = part[j % 3];
        const uint32_t tag = tag_base + (uint32_t)j;

        ChunkIt it;
        it.start(S, rcur0, rcur1);
        int si, g, rb0, nt, cur_s = -1, cur_g = -1;
        while (it.next(S, si, g, rb0, nt)) {
            const ChainStoreD& C = S.st[si];
            if (si != cur_s || g != cur_g) {
                // New (store, group): stage the codebook / activation slice, build T.
                // x[128 g + 2 cp .. +2] = sum over the input partial slices.  Warp w
                // covers column pairs 32 (w % 2) .. +31 -- 512 contiguous bytes of a
                // slice per load, every sector fetched once -- for part w / 2; part p
                // adds slices p, p + 8, ... (4 slices in flight per poll round).
                const bool new_g = g != cur_g;
                const int cp = 32 * (warp & 1) + lane;
                const int xpart = warp >> 1;
                const int64_t c = (int64_t)g * 128 + 2 * cp;
                const bool poll = new_g && j > 0 && c < S.k;
                const uint64_t* col = pin + c;
                ulonglong2 a[4];
                auto issue_round = [&](int gp0) {
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int gp = gp0 + kXGroups * q;
                        if (gp < pin_ng) a[q] = ldcg_u64x2(col + gp * pin_stride);
                    }
                };
                if (poll) issue_round(xpart);
                if (!booked) bookkeeping();
                if (si != cur_s) {
                    cbp ^= 1;
                    float* cbf = cbf_buf + cbp * 1024;
                    // codebook values 2t, 2t+1 of store si, loaded during the previous step
                    float2 v = make_float2(0.f, 0.f);
#pragma unroll
                    for (int q = 0; q < kLutMaxStores; ++q)
                        if (q == si) v = cb_cur[q];
                    reinterpret_cast<float2*>(cbf)[threadIdx.x] = v;
                }
                if (new_g) {
                    xsp ^= 1;
                    float* xs = xs_buf + xsp * (kXGroups * 128);
                    // The table build adds the kXGroups part sums (fixed order throughout).
                    float2 v = make_float2(0.f, 0.f);
                    if (c < S.k) {
                        if (j == 0) {
                            if (xpart == 0) v = make_float2(load_f(x0, x_dtype, c), load_f(x0, x_dtype, c + 1));
                        } else {
                            // Each round: wait until the 4 values of each of its slices
                            // carry step j-1's tag (bounded), add them, issue the next.
                            for (int gp0 = xpart; gp0 < pin_ng; gp0 += 4 * kXGroups) {
                                if (gp0 != xpart) issue_round(gp0);
#pragma unroll
                                for (int q = 0; q < 4; ++q) {
                                    const int gp = gp0 + kXGroups * q;
                                    if (gp >= pin_ng) continue;
                                    uint32_t spins = 0;
                                    while ((tag_of(a[q].x) != want) | (tag_of(a[q].y) != want)) {
                                        if (++spins > kTagSpinLimit ||
                                            *reinterpret_cast<volatile int*>(&g_chain_error)) {
                                            atomicExch(&g_chain_error, 1);
                                            break;
                                        }
                                        // a short back-off keeps waiting CTAs' re-polls from
                                        // crowding the L2 that the late producers still use
                                        __nanosleep(100);
                                        a[q] = ldcg_u64x2(col + gp * pin_stride);
                                    }
                                    v.x += val_of(a[q].x);
                                    v.y += val_of(a[q].y);
                                }
                            }
                        }
                    }
                    reinterpret_cast<float2*>(xs)[xpart * 64 + cp] = v;
                }
                // This step overwrites buffer j % 3, last read during step j-2's staging:
                // before the first write, every CTA must have finished step j-2.
                if (cur_s < 0 && j >= 3 && threadIdx.x == 0) grid_wait(&ctr[j - 2], target);
                cur_s = si;
                cur_g = g;
                consumers_sync();
                if (j > 0 && S.remote && new_g) {
                    // Tensor parallel: every rank publishes its own sum of the slice (tagged)
                    // in xred and adds all ranks' sums in rank order, so all ranks build the
                    // same table from the same x.  Warp w brings rank w's sum into shared
                    // memory (warp my_rank: its own, after publishing it), so the peers'
                    // NVLink round trips overlap instead of following each other.
                    float* xsl = xs_buf + xsp * (kXGroups * 128);
                    float4* xr = reinterpret_cast<float4*>(smem + kXrOff);      // [kMaxTp][32]
                    const int64_t e0 = (int64_t)((j - 1) % 3) * H.xred_elems + (int64_t)g * 128 + 4 * lane;
                    if (warp == my_rank) {
                        const float4* x4 = reinterpret_cast<const float4*>(xsl);
                        float4 loc = x4[lane];
#pragma unroll
                        for (int h = 1; h < kXGroups; ++h) {
                            const float4 u = x4[h * 32 + lane];
                            loc.x += u.x;
                            loc.y += u.y;
                            loc.z += u.z;
                            loc.w += u.w;
                        }
                        uint64_t* mine = reinterpret_cast<uint64_t*>(const_cast<uint8_t*>(ws) + H.xred_off) + e0;
                        stg_u64x2(mine, tagged(loc.x, want), tagged(loc.y, want));
                        stg_u64x2(mine + 2, tagged(loc.z, want), tagged(loc.w, want));
                        xr[warp * 32 + lane] = loc;
                    } else if (warp < world) {
                        const uint64_t* src = reinterpret_cast<const uint64_t*>(H.peer_ws[warp] + H.xred_off) + e0;
                        ulonglong2 a = ldsys_u64x2(src), b = ldsys_u64x2(src + 2);
                        uint32_t spins = 0;
                        while ((tag_of(a.x) != want) | (tag_of(a.y) != want) | (tag_of(b.x) != want) |
                               (tag_of(b.y) != want)) {
                            if (++spins > kTagSpinLimit || *reinterpret_cast<volatile int*>(&g_chain_error)) {
                                atomicExch(&g_chain_error, 1);
                                break;
                            }
                            a = ldsys_u64x2(src);
                            b = ldsys_u64x2(src + 2);
                        }
                        xr[warp * 32 + lane] = make_float4(val_of(a.x), val_of(a.y), val_of(b.x), val_of(b.y));
                    }
                    consumers_sync();
                    if (warp == 0) {
                        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
                        for (int rk = 0; rk < world; ++rk) {
                            const float4 r4 = xr[rk * 32 + lane];
                            x.x += r4.x;
                            x.y += r4.y;
                            x.z += r4.z;
                            x.w += r4.w;
                        }
                        float4* xw = reinterpret_cast<float4*>(xsl);
                        xw[lane] = x;
#pragma unroll
                        for (int h = 1; h < kXGroups; ++h) xw[h * 32 + lane] = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                    consumers_sync();
                }
                {
                    const float* xs = xs_buf + xsp * (kXGroups * 128);
                    float4 xv = reinterpret_cast<const float4*>(xs)[lane];
#pragma unroll
                    for (int h = 1; h < kXGroups; ++h) {
                        const float4 u = reinterpret_cast<const float4*>(xs)[h * 32 + lane];
                        xv.x += u.x;
                        xv.y += u.y;
                        xv.z += u.z;
                        xv.w += u.w;
                    }
                    const float x0v = xv.x, x1v = xv.y, x2v = xv.z, x3v = xv.w;
                    // The warp's 16 codebook entries are loaded before any table store:
                    // the loads cannot be reordered past stores to the same shared
                    // window, so interleaving them would serialise 16 load->store chains.
                    const uint32_t cb_addr = base + cbp * 4096u + 16u * warp;
                    const uint32_t t_addr = kTBase + 4u * ((slot ^ 1) * 32 + lane) + 256u * warp;
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        float4 cv[8];
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            cv[q] = lds_f32x4(cb_addr + 16u * kConsumerWarps * (8 * h + q));
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            float v = cv[q].x * x0v;
                            v = fmaf(cv[q].y, x1v, v);
                            v = fmaf(cv[q].z, x2v, v);
                            v = fmaf(cv[q].w, x3v, v);
                            sts_f32(t_addr + 256u * kConsumerWarps * (8 * h + q), v);
                        }
                    }
                }
                slot ^= 1;
                consumers_sync();
            }
            const int stage = i % kRing;
            mbar_wait(bar_full + 8 * stage, (i / kRing) & 1);
            const uint32_t sdst = stage_addr(stage);
            const int tile = warp * 4 + team;
            float acc[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) acc[r] = 0.f;
            if (tile < nt) {
                const uint32_t tb = sdst + tile * 512;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int pos = tl + 8 * ((q + team) & 3);
                    const uint4 w = lds128(tb + pos * 16);
                    const uint32_t tbase = kTBase | (uint32_t)(slot * 128 + 4 * pos);
                    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int wi = 0; wi < 4; ++wi)
#pragma unroll
                        for (int b = 0; b < 4; ++b)
                            acc[wi * 4 + b] += lds_f32(__byte_perm(ww[wi], tbase, 0x7604 | (b << 4)));
                }
            }
            // Butterfly over the 8 lanes of the team: lane tl ends with rows 2tl, 2tl+1.
            const bool b2 = tl & 4, b1 = tl & 2, b0 = tl & 1;
            float a1[8], a2[4], a3[2];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float send = b2 ? acc[q] : acc[q + 8];
                const float keep = b2 ? acc[q + 8] : acc[q];
                a1[q] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float send = b1 ? a1[q] : a1[q + 4];
                const float keep = b1 ? a1[q + 4] : a1[q];
                a2[q] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
            }
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const float send = b0 ? a2[q] : a2[q + 2];
                const float keep = b0 ? a2[q + 2] : a2[q];
                a3[q] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
            }
            if (tile < nt) {
                const bool f32 = C.scale_f32 != 0;
                const uint32_t esz = f32 ? 4u : 2u;
                const uint32_t sa = sdst + kStageIdx + tile * 16 * esz + 2 * tl * esz;
                const float s0 = lds_scale(sa, f32), s1 = lds_scale(sa + esz, f32);
                const int64_t row = (int64_t)(rb0 + tile) * 16 + 2 * tl;
                stg_u64x2_keep(pout + C.part_off + (int64_t)g * C.rb * 16 + row, tagged(a3[0] * s0, tag),
                               tagged(a3[1] * s1, tag), keep_pol);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_empty + 8 * stage);
            ++i;
        }
        if (!booked) bookkeeping();
        rcur0 = rnext0;
        rcur1 = rnext1;
        consumers_sync();                  // all of this CTA's partials for step j are written
        // This CTA is done reading step j-1's partials (their values have been
        // consumed before the barrier above); no fence is needed for that.
        if (threadIdx.x == 0) {
            if (world == 1) {
                atomicAdd(&ctr[j], 1u);
            } else {
                for (int rk = 0; rk < world; ++rk)
                    red_sys_add(reinterpret_cast<unsigned*>(H.peer_ws[rk] + H.ctr_off) + j, 1u);
            }
        }
    }

    // Final output: the last step's feed store, rows split over the CTAs (each
    // partial polled until it carries the last step's tag).
    {
        const ChainStepD& L = steps[n_steps - 1];
        const ChainStoreD& F = L.st[L.feed];
        const uint64_t* pl = part[(n_steps - 1) % 3] + F.part_off;
        const uint32_t want = tag_base + (uint32_t)(n_steps - 1);
        const int64_t stride = (int64_t)F.rb * 16;
        const int r0 = (int)((int64_t)F.n * blockIdx.x / G), r1 = (int)((int64_t)F.n * (blockIdx.x + 1) / G);
        // 8 lanes per row, each adding every 8th slice; a 3-step shuffle combines them.
        const int sub8 = lane & 7;
        for (int rbase = r0; rbase < r1; rbase += kConsumers / 8) {
            const int r = rbase + (threadIdx.x >> 3);
            float v = 0.f;
            if (r < r1) {
                for (int gg = sub8; gg < F.ng; gg += 8) {
                    uint64_t e = ldcg_u64(pl + gg * stride + r);
                    uint32_t spins = 0;
                    while (tag_of(e) != want) {
                        if (++spins > kTagSpinLimit || *reinterpret_cast<volatile int*>(&g_chain_error)) {
                            atomicExch(&g_chain_error, 1);
                            break;
                        }
                        e = ldcg_u64(pl + gg * stride + r);
                    }
                    v += val_of(e);
                }
            }
            v += __shfl_xor_sync(0xffffffffu, v, 1);
            v += __shfl_xor_sync(0xffffffffu, v, 2);
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            if (world > 1 && H.final_remote) {
                // Sum over ranks: lane sub8 of the row's 8 brings rank sub8's row sum (its
                // own after publishing it), then every lane adds them in rank order.
                const uint32_t tfin = tag_base + (uint32_t)n_steps;
                float rv = 0.f;
                if (r < r1 && sub8 < world) {
                    if (sub8 == my_rank) {
                        uint64_t* mine = reinterpret_cast<uint64_t*>(const_cast<uint8_t*>(ws) + H.xfin_off) + r;
                        asm volatile("st.global.u64 [%0], %1;" ::"l"(mine), "l"(tagged(v, tfin)) : "memory");
                        rv = v;
                    } else {
                        const uint64_t* src = reinterpret_cast<const uint64_t*>(H.peer_ws[sub8] + H.xfin_off) + r;
                        uint64_t e = ldsys_u64(src);
                        uint32_t spins = 0;
                        while (tag_of(e) != tfin) {
                            if (++spins > kTagSpinLimit || *reinterpret_cast<volatile int*>(&g_chain_error)) {
                                atomicExch(&g_chain_error, 1);
                                break;
                            }
                            e = ldsys_u64(src);
                        }
                        rv = val_of(e);
                    }
                }
                float x = 0.f;
                for (int rk = 0; rk < world; ++rk) x += __shfl_sync(0xffffffffu, rv, (lane & ~7) + rk);
                v = x;
            }
            if (r < r1 && sub8 == 0) store_f(out, out_dtype, r, v);
        }
    }
    consumers_sync();
    if (threadIdx.x == 0) {
        __threadfence();
        // The last CTA to finish advances the run generation for the next launch.
        if (atomicAdd(&ctr[n_steps], 1u) == (misc[0] + 1u) * (unsigned)G - 1u) atomicAdd(&ctr[n_steps + 1], 1u);
    }
}

int g_chain_sms[64] = {0};
bool g_chain_attr[64] = {false};

}  // namespace

int chain_read_device_error(int* flag) {
    if (cudaMemcpyFromSymbol(flag, g_chain_error, sizeof(int)) != cudaSuccess)
        return check_launch("read chain error flag");
    return EPQ_OK;
}

static int64_t al256(int64_t v) { return (v + 255) & ~int64_t(255); }

// Tile ranges of one step over `grid` CTAs.  A CTA's time is about its tiles
// plus one table build (activation slice staging + LUT build) per (store, group)
// segment it enters; a build costs about kTableTiles tiles of chunk work, so a
// range that straddles a segment boundary is much dearer than its tile count.
// The ranges stay contiguous in (store, group, row block) order and minimise the
// largest per-CTA cost (binary search on the cost; greedy packing); CTAs left
// over get empty ranges.
constexpr int kTableTiles = 160;

static int pack_ranges(const std::vector<int>& seg, int64_t cap, std::vector<int>* starts) {
    int ctas = 0;
    int64_t cost = 0, t = 0;
    bool open = false;
    if (starts) starts->clear();
    for (const int z : seg) {
        int64_t rem = z;
        bool entered = false;          // has the open CTA paid for this segment's table?
        while (rem > 0) {
            if (!open) {
                open = true;
                entered = false;
                ++ctas;
                cost = 0;
                if (starts) starts->push_back((int)t);
            }
            const int64_t room = cap - cost - (entered ? 0 : kTableTiles);
            if (room <= 0) {
                open = false;
                continue;
            }
            const int64_t take = rem < room ? rem : room;
            cost += take + (entered ? 0 : kTableTiles);
            entered = true;
            rem -= take;
            t += take;
            if (cost >= cap) open = false;
        }
    }
    return ctas;
}

static void balance_ranges(const std::vector<int>& seg, int grid, std::vector<int>* r) {
    int64_t total = 0;
    for (const int z : seg) total += z;
    int64_t lo = kTableTiles + 1, hi = kTableTiles + total + 1;
    while (lo < hi) {
        const int64_t mid = lo + (hi - lo) / 2;
        if (pack_ranges(seg, mid, nullptr) <= grid) hi = mid;
        else lo = mid + 1;
    }
    std::vector<int> starts;
    pack_ranges(seg, lo, &starts);
    r->assign(grid + 1, (int)total);
    for (size_t c = 0; c < starts.size() && (int)c < grid; ++c) (*r)[c] = starts[c];
    (*r)[0] = 0;
}

// Host-side description of a chain (validated) and its workspace layout.
struct StoreArr {
    StoreD s[kLutMaxStores];
};

int chain_layout(const StoreArr* st, const int* counts, const int* feeds, int n_steps,
                 int grid, std::vector<ChainStepD>* out_steps, ChainHeaderD* hdr, int64_t* ws_bytes,
                 std::vector<int>* out_ranges) {
    if (n_steps < 1) return set_error(EPQ_EINVAL, "chain: n_steps=%d", n_steps);
    std::vector<ChainStepD> steps(n_steps);
    int64_t part_floats = 0;
    for (int j = 0; j < n_steps; ++j) {
        ChainStepD& D = steps[j];
        memset(&D, 0, sizeof(D));
        D.count = counts[j];
        D.feed = feeds[j];
        if (D.count < 1 || D.count > kLutMaxStores || D.feed < 0 || D.feed >= D.count)
            return set_error(EPQ_EINVAL, "chain: step %d has count=%d feed=%d", j, D.count, D.feed);
        int64_t tiles = 0, floats = 0;
        for (int i = 0; i < D.count; ++i) {
            const StoreD& s = st[j].s[i];
            if (!lut_eligible(s))
                return set_error(EPQ_EUNSUPPORTED, "chain: step %d store %d is not an EPQ_LAYOUT_TILED "
                                 "vector store (vec 4, 8-bit, group 128)", j, i);
            if (s.k != st[j].s[0].k) return set_error(EPQ_ESHAPE, "chain: step %d stores differ in k", j);
            const int64_t esz = s.scale_dtype == EPQ_F32 ? 4 : 2;
            if ((s.scale_dtype != EPQ_F16 && s.scale_dtype != EPQ_F32) || s.s_n != 1 || s.s_g % 16 ||
                s.s_g < s.rb * 16 || (reinterpret_cast<uintptr_t>(s.scale) % (16 * esz)) ||
                (reinterpret_cast<uintptr_t>(s.idx) & 15))
                return set_error(EPQ_ELAYOUT, "chain: step %d store %d needs group-major f16/f32 scales "
                                 "with a row stride padded to 16 and 16-byte aligned buffers", j, i);
            ChainStoreD& C = D.st[i];
            C.idx = s.idx;
            C.scale = s.scale;
            C.cb = s.cb;
            C.s_g = s.s_g;
            C.cb_dtype = s.cb_dtype;
            C.scale_f32 = s.scale_dtype == EPQ_F32;
            C.levels = s.levels;
            C.n = (int)s.n;
            C.rb = (int)s.rb;
            C.ng = (int)s.ng;
            C.tile0 = (int)tiles;
            C.part_off = floats;
            tiles += s.ng * s.rb;
            floats += s.ng * s.rb * 16;
        }
        if (tiles >= (int64_t(1) << 30)) return set_error(EPQ_EUNSUPPORTED, "chain: step %d too large", j);
        D.k = (int)st[j].s[0].k;
        D.kpos = (int)(st[j].s[0].k / 4);
        D.total_tiles = (int)tiles;
        if (j > 0 && st[j - 1].s[feeds[j - 1]].n != st[j].s[0].k)
            return set_error(EPQ_ESHAPE, "chain: step %d input width %lld != step %d feed output %lld", j,
                             (long long)st[j].s[0].k, j - 1, (long long)st[j - 1].s[feeds[j - 1]].n);
        part_floats = floats > part_floats ? floats : part_floats;
    }
    ChainHeaderD H{};
    H.n_steps = n_steps;
    H.grid = grid;
    H.part_floats = part_floats;
    H.steps_off = 256;
    const int64_t ranges_off = al256(H.steps_off + (int64_t)sizeof(ChainStepD) * n_steps);
    for (int j = 0; j < n_steps; ++j) steps[j].range_off = ranges_off + 4 * (int64_t)(grid + 1) * j;
    if (out_ranges) {
        out_ranges->clear();
        for (int j = 0; j < n_steps; ++j) {
            std::vector<int> seg, r;
            for (int i = 0; i < steps[j].count; ++i)
                for (int g = 0; g < steps[j].st[i].ng; ++g) seg.push_back(steps[j].st[i].rb);
            balance_ranges(seg, grid, &r);
            out_ranges->insert(out_ranges->end(), r.begin(), r.end());
        }
    }
    H.ctr_off = al256(ranges_off + 4 * (int64_t)(grid + 1) * n_steps);
    H.part_off0 = al256(H.ctr_off + 4 * (n_steps + 2));
    H.part_off1 = al256(H.part_off0 + 8 * part_floats);
    H.part_off2 = al256(H.part_off1 + 8 * part_floats);
    int64_t kmax = 0;
    for (int j = 0; j < n_steps; ++j) kmax = steps[j].k > kmax ? steps[j].k : kmax;
    H.xred_elems = al256(kmax);
    H.xred_off = al256(H.part_off2 + 8 * part_floats);
    H.xfin_elems = st[n_steps - 1].s[feeds[n_steps - 1]].n;
    H.xfin_off = al256(H.xred_off + 3 * 8 * H.xred_elems);
    H.tp_world = 1;
    H.tp_rank = 0;
    *ws_bytes = al256(H.xfin_off + 8 * H.xfin_elems);
    *hdr = H;
    if (out_steps) *out_steps = std::move(steps);
    return EPQ_OK;
}

int chain_grid(int* grid) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return set_error(EPQ_EUNSUPPORTED, "chain: no usable current device");
    {
        static std::mutex mu;
        std::lock_guard<std::mutex> lock(mu);
        if (!g_chain_attr[dev]) {
            if (cudaFuncSetAttribute(chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmem) !=
                cudaSuccess)
                return check_launch("cudaFuncSetAttribute(chain_kernel)");
            int per_sm = 0, sms = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, chain_kernel, kThreads, kDynSmem) !=
                    cudaSuccess ||
                cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
                return check_launch("chain occupancy");
            if (per_sm < 1) return set_error(EPQ_EUNSUPPORTED, "chain: kernel does not fit on an SM");
            g_chain_sms[dev] = sms;
            g_chain_attr[dev] = true;
        }
    }
    *grid = g_chain_sms[dev];
    return EPQ_OK;
}

int chain_write(const std::vector<ChainStepD>& steps, const std::vector<int>& ranges, const ChainHeaderD& H,
                void* ws, cudaStream_t st) {
    std::vector<uint8_t> host(H.part_off0, 0);
    memcpy(host.data(), &H, sizeof(H));
    memcpy(host.data() + H.steps_off, steps.data(), sizeof(ChainStepD) * steps.size());
    if (!steps.empty())
        memcpy(host.data() + steps[0].range_off, ranges.data(), sizeof(int) * ranges.size());
    // counters (and the run generation) start at zero
    if (cudaMemcpyAsync(ws, host.data(), host.size(), cudaMemcpyHostToDevice, st) != cudaSuccess)
        return check_launch("chain: write descriptors");
    // partial and exchange buffers start with tag 0, which no step uses
    const int64_t part_end = al256(H.xfin_off + 8 * H.xfin_elems);
    if (cudaMemsetAsync(static_cast<uint8_t*>(ws) + H.part_off0, 0, part_end - H.part_off0, st) != cudaSuccess)
        return check_launch("chain: clear partial buffers");
    if (cudaStreamSynchronize(st) != cudaSuccess) return check_launch("chain: write descriptors");
    return EPQ_OK;
}

int chain_launch(const void* ws, const void* x, int x_dtype, void* out, int out_dtype, int grid,
                 cudaStream_t st) {
    const uint8_t* wsp = static_cast<const uint8_t*>(ws);
    void* args[] = {(void*)&wsp, (void*)&x, (void*)&x_dtype, (void*)&out, (void*)&out_dtype};
    if (cudaLaunchCooperativeKernel((void*)chain_kernel, dim3(grid), dim3(kThreads), args, kDynSmem, st) !=
        cudaSuccess)
        return check_launch("chain_kernel");
    return check_launch("chain_kernel");
}

}  // namespace epq

using namespace epq;

extern "C" {

static int chain_collect(const epq_chain_step* steps, int32_t n_steps, StoreArr* st,
                         int* counts, int* feeds) {
    for (int j = 0; j < n_steps; ++j) {
        counts[j] = steps[j].count;
        feeds[j] = steps[j].feed;
        if (counts[j] < 1 || counts[j] > kLutMaxStores)
            return set_error(EPQ_EINVAL, "chain: step %d count=%d (1..%d)", j, counts[j], kLutMaxStores);
        for (int i = 0; i < counts[j]; ++i) {
            int rc = make_store(&steps[j].stores[i], &st[j].s[i], "chain");
            if (rc) return rc;
        }
    }
    return EPQ_OK;
}

int epq_chain_workspace_bytes(const epq_chain_step* steps, int32_t n_steps, int64_t* bytes) {
    if (!steps || !bytes || n_steps < 1 || n_steps > 4096)
        return set_error(EPQ_EINVAL, "chain_workspace_bytes: steps/bytes NULL or n_steps=%d", n_steps);
    std::vector<StoreArr> st(n_steps);
    std::vector<int> counts(n_steps), feeds(n_steps);
    int rc = chain_collect(steps, n_steps, st.data(), counts.data(), feeds.data());
    if (rc) return rc;
    int grid = 0;
    rc = chain_grid(&grid);
    if (rc) return rc;
    ChainHeaderD H;
    return chain_layout(st.data(), counts.data(), feeds.data(), n_steps, grid, nullptr, &H, bytes, nullptr);
}

int epq_chain_prepare(const epq_chain_step* steps, int32_t n_steps, void* workspace,
                      int64_t workspace_bytes, void* stream) {
    if (!steps || !workspace || n_steps < 1 || n_steps > 4096)
        return set_error(EPQ_EINVAL, "chain_prepare: steps/workspace NULL or n_steps=%d", n_steps);
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
        return set_error(EPQ_EALIGN, "chain_prepare: workspace must be 256-byte aligned");
    std::vector<StoreArr> st(n_steps);
    std::vector<int> counts(n_steps), feeds(n_steps);
    int rc = chain_collect(steps, n_steps, st.data(), counts.data(), feeds.data());
    if (rc) return rc;
    int grid = 0;
    rc = chain_grid(&grid);
    if (rc) return rc;
    std::vector<ChainStepD> desc;
    std::vector<int> ranges;
    ChainHeaderD H;
    int64_t need = 0;
    rc = chain_layout(st.data(), counts.data(), feeds.data(), n_steps, grid, &desc, &H, &need, &ranges);
    if (rc) return rc;
    if (workspace_bytes < need)
        return set_error(EPQ_EWORKSPACE, "chain_prepare: workspace of %lld bytes needed, %lld given",
                         (long long)need, (long long)workspace_bytes);
    return chain_write(desc, ranges, H, workspace, static_cast<cudaStream_t>(stream));
}

int epq_chain_set_tp(void* workspace, int32_t rank, int32_t world, const void* const* peer_workspaces,
                     const uint8_t* remote_input, int32_t n_flags, void* stream) {
    if (!workspace || world < 1 || world > kMaxTp || rank < 0 || rank >= world || (world > 1 && !peer_workspaces))
        return set_error(EPQ_EINVAL, "chain_set_tp: rank=%d world=%d (1..%d) / NULL peers", rank, world, kMaxTp);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    ChainHeaderD H;
    if (cudaMemcpyAsync(&H, workspace, sizeof(H), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return check_launch("chain_set_tp: read header");
    if (H.n_steps < 1 || H.n_steps > 4096 || H.steps_off != 256)
        return set_error(EPQ_EINVAL, "chain_set_tp: workspace not prepared by epq_chain_prepare");
    if (!remote_input || n_flags != H.n_steps + 1)
        return set_error(EPQ_EINVAL, "chain_set_tp: %d flags given, n_steps + 1 = %d needed", n_flags,
                         H.n_steps + 1);
    if (remote_input[0])
        return set_error(EPQ_EINVAL, "chain_set_tp: the first step reads the caller's x, not partial sums");
    std::vector<ChainStepD> steps(H.n_steps);
    if (cudaMemcpyAsync(steps.data(), static_cast<uint8_t*>(workspace) + H.steps_off,
                        sizeof(ChainStepD) * H.n_steps, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return check_launch("chain_set_tp: read steps");
    for (int j = 0; j < H.n_steps; ++j) steps[j].remote = world > 1 && remote_input[j];
    H.tp_world = world;
    H.tp_rank = rank;
    H.final_remote = world > 1 && remote_input[H.n_steps];
    for (int r = 0; r < kMaxTp; ++r)
        H.peer_ws[r] = r < world ? reinterpret_cast<int64_t>(world > 1 ? peer_workspaces[r] : workspace) : 0;
    if (world > 1 && peer_workspaces[rank] != workspace)
        return set_error(EPQ_EINVAL, "chain_set_tp: peer_workspaces[rank] must be this workspace");
    if (cudaMemcpyAsync(workspace, &H, sizeof(H), cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(static_cast<uint8_t*>(workspace) + H.steps_off, steps.data(),
                        sizeof(ChainStepD) * H.n_steps, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
        return check_launch("chain_set_tp: write");
    return EPQ_OK;
}

int epq_chain_run(const void* workspace, const void* x, int32_t x_dtype, void* out, int32_t out_dtype,
                  void* stream) {
    if (!workspace || !x || !out) return set_error(EPQ_EINVAL, "chain_run: NULL pointer");
    if (!dtype_ok(x_dtype) || !dtype_ok(out_dtype))
        return set_error(EPQ_EDTYPE, "chain_run: x/out dtype must be f32, f16 or bf16");
    int grid = 0;
    int rc = chain_grid(&grid);
    if (rc) return rc;
    return chain_launch(workspace, x, x_dtype, out, out_dtype, grid, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
