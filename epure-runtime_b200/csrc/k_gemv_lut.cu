// Batch-1 dequant-GEMV for 4-weight vector codebooks: out[r] = sum_c x[c] W[r, c]
// with W[r, 4j+p] = cb[idx[r, j], p] * scale[r, g(j)].  HBM-bound: the index
// stream (1 byte per 4 weights) is ~94% of the bytes the op must move.
//
// Reference op: epure/kernels/_triton.py:56-107 (_dequant_matmul, table mode),
// which gathers cb[idx] per weight and multiplies by the scale in registers.
//
// Design (B200, sm_100a):
// * Activation LUT.  For one scale group (32 index positions j) the kernel
//   first builds T[e][j] = dot(cb[e, 0:4], x[4j : 4j+4]) in fp32 shared
//   memory for all 256 entries e.  A row's group sum is then
//   sum_j T[idx[r, j]][j]: one 4-byte shared load and one add per index,
//   instead of an 8-byte codebook gather plus 4 conversions and 4 FMAs.  The
//   scale multiplies the group sum once.  The table is built once per
//   (group, CTA) and reused by every row the CTA streams.
// * Conflict-free lookups.  T is stored row-major by entry, 256 B per entry
//   (2 slots x 32 positions x 4 B), so position j always falls in bank j; the
//   index layout (EPQ_LAYOUT_TILED: 16 rows x 32 positions per 512-byte tile)
//   makes every lane read one fixed position for 16 rows with a single
//   128-bit load.  The lookup address is one PRMT: the index byte becomes
//   address bits 8..15, the lane's position and the table base fill the rest.
// * Teams of 8 lanes.  Each team owns one 16-row tile; a lane covers 4 of
//   the 32 positions (position blocks permuted per team, block i ^ team, so
//   the 32 lanes of a warp always hit 32 different banks), then a 3-step
//   butterfly leaves every lane with the sums of 2 rows.  The four blocks are
//   added as (b0 + b1) + (b2 + b3) whatever the permutation, so a tile's sums
//   are the same bits in every launch shape (fused stores, split grids).
// * Split over k with a deterministic reduction.  The grid is one CTA per SM;
//   CTA c streams a contiguous range of tiles in (store, group, row-block)
//   order.  Each finished tile writes its 16 scaled group sums to
//   partials[g][row]; a per-row-block counter picks the last arriving team,
//   which adds the partials in group order and writes the output row-block,
//   then resets the counter to zero for the next call.
#include <mutex>

#include "epq_common.cuh"

namespace epq {
namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr uint32_t kTBase = 65536;   // shared-window offset of T: low 16 bits must be 0
constexpr uint32_t kTBytes = 65536;  // 256 entries x 256 B
constexpr int kDynSmem = 131072;     // covers [dynamic base, kTBase + kTBytes)
constexpr int kListOffset = 8192;    // finished-row-block list (below T, after the codebook)
constexpr int kListCap = 8192;       // entries (32 KB)

struct LutStore {
    const uint8_t* idx;
    const void* scale;
    int64_t s_n, s_g;
    const void* cb;
    void* out;
    float* partials;     // [ng][rb * 16]
    unsigned* counters;  // [rb]
    int scale_dtype, cb_dtype, levels;
    int n, rb, ng, kpos;
    int tile0;           // global index of this store's first tile
};

struct LutParams {
    LutStore st[kLutMaxStores];
    const void* x;
    int count, x_dtype, out_dtype;
    int total_tiles, tiles_per_cta;
    int dyn_smem;
};

// Set by the kernel when the shared-memory placement it relies on does not
// hold (the kernel then writes nothing); read by epq_device_error().
__device__ int g_lut_layout_error = 0;

__device__ __forceinline__ float lds_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint4 ldg_stream(const uint8_t* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Adds the 16 T entries selected by the 16 index bytes of `v` into acc.
__device__ __forceinline__ void lookup16(const uint4 v, uint32_t base, float (&acc)[16]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int wi = 0; wi < 4; ++wi) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t addr = __byte_perm(w[wi], base, 0x7604 | (q << 4));
            acc[wi * 4 + q] += lds_f32(addr);
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1) gemv_lut_kernel(const __grid_constant__ LutParams P) {
    extern __shared__ __align__(16) uint8_t smem[];
    const uint32_t smem_base = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    if (smem_base + kListOffset + 4u * kListCap > kTBase ||
        smem_base + (uint32_t)P.dyn_smem < kTBase + kTBytes) {
        if (threadIdx.x == 0) atomicExch(&g_lut_layout_error, 1);
        return;
    }
    float* cbf = reinterpret_cast<float*>(smem);                 // [256][4] fp32
    float* T = reinterpret_cast<float*>(smem + (kTBase - smem_base));  // [256][2][32]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int team = lane >> 3, tl = lane & 7;

    const int t_begin = blockIdx.x * P.tiles_per_cta;
    int t = t_begin;
    const int t_end = min(t + P.tiles_per_cta, P.total_tiles);
    int cur_store = -1, slot = 0;
    bool wrote = false;

    while (t < t_end) {
        int si = 0;
        while (si + 1 < P.count && t >= P.st[si + 1].tile0) ++si;
        const LutStore& S = P.st[si];
        const int local = t - S.tile0;
        const int g = local / S.rb;
        const int rb0 = local - g * S.rb;
        const int seg_end = min(t_end, S.tile0 + (g + 1) * S.rb);
        const int seg_tiles = seg_end - t;
        const int n_quads = (seg_tiles + 3) >> 2;

        // First quad of this warp: issue its loads before building the table.
        int q = warp;
        uint4 cur[4];
        const uint8_t* tile_base = S.idx + ((int64_t)g * S.rb) * 512;
        auto load_quad = [&](int qq, uint4 (&dst)[4]) {
            const int tile = 4 * qq + team;
            if (qq < n_quads && tile < seg_tiles) {
                const uint8_t* tp = tile_base + (int64_t)(rb0 + tile) * 512;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int pos = tl + 8 * (i ^ team);
                    dst[i] = ldg_stream(tp + pos * 16);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 4; ++i) dst[i] = make_uint4(0, 0, 0, 0);
            }
        };
        load_quad(q, cur);
        auto load_scales = [&](int qq, float& s0, float& s1) {
            const int tile = 4 * qq + team;
            s0 = s1 = 0.f;
            if (qq < n_quads && tile < seg_tiles) {
                const int row = (rb0 + tile) * 16 + 2 * tl;
                if (row < S.n) s0 = load_f(S.scale, S.scale_dtype, row * S.s_n + (int64_t)g * S.s_g);
                if (row + 1 < S.n)
                    s1 = load_f(S.scale, S.scale_dtype, (row + 1) * S.s_n + (int64_t)g * S.s_g);
            }
        };
        float cs0, cs1;
        load_scales(q, cs0, cs1);

        if (si != cur_store) {
            // Codebook -> fp32 shared, zero-padded to 256 entries.
            for (int i = threadIdx.x; i < 1024; i += kThreads)
                cbf[i] = (i < S.levels * 4) ? load_f(S.cb, S.cb_dtype, i) : 0.f;
            cur_store = si;
            __syncthreads();
        }
        // Build T[e][slot][pos] for the 32 positions of group g.
        {
            const int j = g * 32 + lane;
            float x0 = 0.f, x1 = 0.f, x2 = 0.f, x3 = 0.f;
            if (j < S.kpos) {
                const int64_t c = (int64_t)j * 4;
                x0 = load_f(P.x, P.x_dtype, c);
                x1 = load_f(P.x, P.x_dtype, c + 1);
                x2 = load_f(P.x, P.x_dtype, c + 2);
                x3 = load_f(P.x, P.x_dtype, c + 3);
            }
            const float4* cb4 = reinterpret_cast<const float4*>(cbf);
#pragma unroll 4
            for (int i = 0; i < 256 / kWarps; ++i) {
                const int e = warp + kWarps * i;
                const float4 c = cb4[e];
                float v = c.x * x0;
                v = fmaf(c.y, x1, v);
                v = fmaf(c.z, x2, v);
                v = fmaf(c.w, x3, v);
                T[e * 64 + slot * 32 + lane] = v;
            }
        }
        __syncthreads();

        uint32_t base[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
            base[i] = kTBase | (uint32_t)(slot * 128 + 4 * (tl + 8 * (i ^ team)));

        const int n16 = S.rb * 16;
        for (; q < n_quads; q += kWarps) {
            uint4 nxt[4];
            float ns0, ns1;
            load_quad(q + kWarps, nxt);
            load_scales(q + kWarps, ns0, ns1);
            // Position blocks {0, 1} and {2, 3} are summed apart and then added: the
            // blocks a lane holds are permuted by team (i ^ team), but the pairs are
            // the same sets for every team, so a tile's sums do not depend on which
            // team (and so which launch shape) processed it.
            float acc[16], acc2[16];
#pragma unroll
            for (int r = 0; r < 16; ++r) acc[r] = acc2[r] = 0.f;
            lookup16(cur[0], base[0], acc);
            lookup16(cur[1], base[1], acc);
            lookup16(cur[2], base[2], acc2);
            lookup16(cur[3], base[3], acc2);
#pragma unroll
            for (int r = 0; r < 16; ++r) acc[r] += acc2[r];

            // Butterfly over the 8 lanes of the team: lane tl ends with rows 2tl, 2tl+1.
            const bool b2 = tl & 4, b1 = tl & 2, b0 = tl & 1;
            float a1[8], a2[4], a3[2];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float send = b2 ? acc[i] : acc[i + 8];
                const float keep = b2 ? acc[i + 8] : acc[i];
                a1[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float send = b1 ? a1[i] : a1[i + 4];
                const float keep = b1 ? a1[i + 4] : a1[i];
                a2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
            }
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const float send = b0 ? a2[i] : a2[i + 2];
                const float keep = b0 ? a2[i + 2] : a2[i];
                a3[i] = keep + __shfl_xor_sync(0xffffffffu, send, 1);
            }

            // Scaled group sums of this tile -> partials[g][row]; nothing waits here.
            const int tile = 4 * q + team;
            if (tile < seg_tiles) {
                const int row = (rb0 + tile) * 16 + 2 * tl;
                *reinterpret_cast<float2*>(S.partials + (int64_t)g * n16 + row) =
                    make_float2(a3[0] * cs0, a3[1] * cs1);
                wrote = true;
            }
            cs0 = ns0;
            cs1 = ns1;
#pragma unroll
            for (int i = 0; i < 4; ++i) cur[i] = nxt[i];
        }
        slot ^= 1;
        t = seg_end;
    }

    // Completion: one counter increment per tile of this CTA; the CTA whose
    // increment completes a row block (all ng groups written) reduces it.
    if (wrote) __threadfence();
    int* finish = reinterpret_cast<int*>(smem + kListOffset);   // (store << 24) | rb
    int* n_finish = reinterpret_cast<int*>(smem + kListOffset - 16);
    if (threadIdx.x == 0) *n_finish = 0;
    __syncthreads();
    for (int tt = t_begin + threadIdx.x; tt < t_end; tt += kThreads) {
        int si = 0;
        while (si + 1 < P.count && tt >= P.st[si + 1].tile0) ++si;
        const LutStore& S = P.st[si];
        const int rb = (tt - S.tile0) % S.rb;
        if (atomicAdd(&S.counters[rb], 1u) == (unsigned)(S.ng - 1)) {
            __threadfence();
            const int slot_i = atomicAdd(n_finish, 1);
            if (slot_i < kListCap) {
                finish[slot_i] = (si << 24) | rb;
            } else {  // list full: reduce this row block here (rare)
                // Same order as the list path below (even groups, odd groups, then
                // their sum), so the result does not depend on which path ran.
                for (int r = 0; r < 16; ++r) {
                    const int row = rb * 16 + r;
                    float even = 0.f, odd = 0.f;
                    for (int gg = 0; gg < S.ng; gg += 2) even += __ldcg(S.partials + (int64_t)gg * S.rb * 16 + row);
                    for (int gg = 1; gg < S.ng; gg += 2) odd += __ldcg(S.partials + (int64_t)gg * S.rb * 16 + row);
                    if (row < S.n) store_f(S.out, P.out_dtype, row, even + odd);
                }
                S.counters[rb] = 0u;
            }
        }
    }
    __syncthreads();
    const int nf = min(*n_finish, kListCap);
    for (int f = warp; f < nf; f += kWarps) {
        const int si = finish[f] >> 24, rb = finish[f] & 0xFFFFFF;
        const LutStore& S = P.st[si];
        const int row = rb * 16 + (lane & 15);
        const int64_t n16 = (int64_t)S.rb * 16;
        float sum = 0.f;
        for (int gg = lane >> 4; gg < S.ng; gg += 2) sum += __ldcg(S.partials + gg * n16 + row);
        sum += __shfl_xor_sync(0xffffffffu, sum, 16);
        if (lane < 16 && row < S.n) store_f(S.out, P.out_dtype, row, sum);
        if (lane == 0) S.counters[rb] = 0u;
    }
}

int num_sms() { return device_sms(); }

}  // namespace

bool lut_eligible(const StoreD& s) {
    return s.layout == EPQ_LAYOUT_TILED && s.bits == 8 && s.vec == 4 && s.group == 128 &&
           s.levels <= 256 && s.n <= (1 << 30) && s.k <= (1 << 30) && s.n > 0 && s.k > 0;
}

static int64_t align256(int64_t v) { return (v + 255) & ~int64_t(255); }

// Per-row-block completion counters (u32) at the start of the workspace.
constexpr int64_t kCounterRegionBytes = 65536;

bool lut_counters_fit(const StoreD* s, int count) {
    int64_t n = 0;
    for (int i = 0; i < count; ++i) n += s[i].rb;
    return n * 4 <= kCounterRegionBytes;
}

int64_t lut_workspace_bytes(const StoreD* s, int count) {
    int64_t b = kCounterRegionBytes;
    for (int i = 0; i < count; ++i) b += align256(s[i].ng * s[i].rb * 16 * 4);
    return b;
}

int launch_linear_lut(const StoreD* s, int count, const void* x, int x_dtype, void* const* outs,
                      int out_dtype, void* ws, int64_t ws_bytes, cudaStream_t st) {
    const int64_t need = lut_workspace_bytes(s, count);
    if (ws == nullptr || ws_bytes < need)
        return set_error(EPQ_EWORKSPACE, "linear: workspace of %lld bytes needed, %lld given",
                         (long long)need, (long long)ws_bytes);
    if ((reinterpret_cast<uintptr_t>(ws) & 255) != 0)
        return set_error(EPQ_EALIGN, "linear: workspace must be 256-byte aligned");
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return set_error(EPQ_EUNSUPPORTED, "device ordinal %d", dev);
    {
        const int arc = set_smem_limit(reinterpret_cast<const void*>(gemv_lut_kernel), kDynSmem,
                                       "cudaFuncSetAttribute(gemv_lut_kernel)");
        if (arc != EPQ_OK) return arc;
    }
    LutParams P{};
    P.count = count;
    P.x = x;
    P.x_dtype = x_dtype;
    P.out_dtype = out_dtype;
    P.dyn_smem = kDynSmem;
    // Counters live in a fixed region at the start of every workspace, so no
    // call ever uses bytes another call wrote partial sums into as counters.
    int64_t n_counters = 0;
    for (int i = 0; i < count; ++i) n_counters += s[i].rb;
    if (n_counters * 4 > kCounterRegionBytes)
        return set_error(EPQ_EUNSUPPORTED, "linear: %lld row blocks exceed the %lld counters of "
                         "the batch-1 kernel", (long long)n_counters,
                         (long long)(kCounterRegionBytes / 4));
    unsigned* counters = static_cast<unsigned*>(ws);
    uint8_t* wp = static_cast<uint8_t*>(ws) + kCounterRegionBytes;
    int64_t total = 0;
    for (int i = 0; i < count; ++i) {
        LutStore& L = P.st[i];
        L.idx = s[i].idx;
        L.scale = s[i].scale;
        L.s_n = s[i].s_n;
        L.s_g = s[i].s_g;
        L.cb = s[i].cb;
        L.out = outs[i];
        L.scale_dtype = s[i].scale_dtype;
        L.cb_dtype = s[i].cb_dtype;
        L.levels = s[i].levels;
        L.n = (int)s[i].n;
        L.rb = (int)s[i].rb;
        L.ng = (int)s[i].ng;
        L.kpos = (int)s[i].kpos;
        L.tile0 = (int)total;
        L.counters = counters;
        counters += s[i].rb;
        total += s[i].ng * s[i].rb;
    }
    for (int i = 0; i < count; ++i) {
        P.st[i].partials = reinterpret_cast<float*>(wp);
        wp += align256(s[i].ng * s[i].rb * 16 * 4);
    }
    if (total >= (int64_t(1) << 31)) return set_error(EPQ_EUNSUPPORTED, "linear: too many tiles");
    P.total_tiles = (int)total;
    const int sms = num_sms();
    int per = (int)cdiv(total, sms);
    if (per < 8) per = 8;
    P.tiles_per_cta = per;
    const int grid = (int)cdiv(total, per);
    gemv_lut_kernel<<<grid, kThreads, kDynSmem, st>>>(P);
    return check_launch("gemv_lut_kernel");
}

int lut_read_device_error(int* flag) {
    if (cudaMemcpyFromSymbol(flag, g_lut_layout_error, sizeof(int)) != cudaSuccess)
        return check_launch("read gemv_lut error flag");
    return EPQ_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of the batch-1 LUT GEMV.
//
// Some callers cannot call cudaMalloc (or any allocating routine) at the point
// where they run the op: a plugin loaded into a serving engine whose memory
// manager reserves the whole device up front and forbids side allocations, or
// a latency-critical loop where an allocation could block or fail.  For them
// the workspace of the LUT kernel (completion counters + partial sums) lives
// in this file-scope device array instead of a caller buffer.  Every GPU that
// loads the library holds it until the process exits.
// ---------------------------------------------------------------------------
constexpr int64_t kStaticScratchBytes = 4 << 20;   // 4 MiB: counters + partial sums
static __device__ __align__(256) unsigned char g_lut_static_scratch[kStaticScratchBytes];

namespace {
std::mutex g_static_mu;
void* g_static_ptr[64] = {nullptr};
}  // namespace

int64_t lut_static_scratch_bytes() { return kStaticScratchBytes; }

int launch_linear_lut_static(const StoreD* s, int count, const void* x, int x_dtype,
                             void* const* outs, int out_dtype, cudaStream_t st) {
    const int64_t need = lut_workspace_bytes(s, count);
    if (need > kStaticScratchBytes)
        return set_error(EPQ_EWORKSPACE,
                         "linear_noalloc: these stores need %lld bytes of scratch; the static "
                         "scratch holds %lld (use epq_linear_multi with a workspace)",
                         (long long)need, (long long)kStaticScratchBytes);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return set_error(EPQ_EUNSUPPORTED, "linear_noalloc: no usable current device");
    void* ptr = nullptr;
    {
        // First call on a device: resolve the device address of the array with
        // that device current (the host-side symbol is not a device address).
        std::lock_guard<std::mutex> lock(g_static_mu);
        if (g_static_ptr[dev] == nullptr) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_lut_static_scratch);
            if (e != cudaSuccess || p == nullptr)
                return set_error(EPQ_ELAUNCH, "linear_noalloc: cudaGetSymbolAddress failed: %s",
                                 cudaGetErrorString(e));
            g_static_ptr[dev] = p;
        }
        ptr = g_static_ptr[dev];
    }
    // The completion counters must start at zero; clear the ones this call uses
    // (partial sums are written before they are read).  Stores with more row
    // blocks than the counter region holds are refused before anything is cleared.
    int64_t n_counters = 0;
    for (int i = 0; i < count; ++i) n_counters += s[i].rb;
    if (!lut_counters_fit(s, count))
        return set_error(EPQ_EUNSUPPORTED, "linear_noalloc: %lld row blocks exceed the %lld counters of the "
                         "batch-1 kernel", (long long)n_counters, (long long)(kCounterRegionBytes / 4));
    if (cudaMemsetAsync(ptr, 0, n_counters * 4, st) != cudaSuccess)
        return check_launch("linear_noalloc: clear counters");
    return launch_linear_lut(s, count, x, x_dtype, outs, out_dtype, ptr, kStaticScratchBytes, st);
}

}  // namespace epq
