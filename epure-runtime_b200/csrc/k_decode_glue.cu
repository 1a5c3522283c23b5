// Decode-step glue around the packed linears: the non-linear parts of a
// Llama-3 / Qwen3 block for one token, each one small launch instead of the
// dozen elementwise torch kernels it replaces, so that a whole-token CUDA graph
// is dominated by the packed linears and the lm_head.
//
// Reference counterpart: the reference leaves these to the Hugging Face model
// around its PackedLinear modules (epure/runtime.py:214-305 swaps only the
// linears); the arithmetic follows that model's (fp32 math, results rounded to
// the activation dtype where the model's tensors are in that dtype):
//
//   epq_add_rmsnorm  h = x + add (rounded), y = h * rsqrt(mean(h^2) + eps) (weight 1)
//   epq_rope_kv      optional per-head RMSNorm of q and k (Qwen3), rotate-half RoPE
//                    at a device-resident position, k / v written into the caches
//   epq_attn_decode  one query row per head against cache positions 0..pos
//                    (grouped-query attention, fp32 online softmax)
//   epq_silu_mul     silu(g) * u
//
// All four read positions from device memory, so a decode step captured in a
// CUDA graph replays at any position.
#include "epq_common.cuh"
#include "epq_decode.h"
#include "epq_rope.cuh"

namespace epq {
namespace {

// Set when a decode position is at or past the KV cache's capacity (max_len):
// the kernel then writes nothing to the cache and zeros to its output.
__device__ int g_glue_position_error = 0;

// Programmatic dependent launch: every glue kernel is launched allowed to start
// while the previous kernel in the stream is still running; it lets its own
// dependents launch at once and waits for the previous grid's completion (and
// memory) before reading anything that grid wrote.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <typename... KArgs, typename... Args>
int launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, unsigned cluster_x, size_t smem,
                       cudaStream_t st, const char* what, Args... args) {
    if (smem > 0) {
        const int rc = set_smem_limit(reinterpret_cast<const void*>(kern), (int)smem, what);
        if (rc != EPQ_OK) return rc;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
    return check_launch(what);
}

template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, const char* what,
               Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
    return check_launch(what);
}

template <int kThreads>
__device__ __forceinline__ float block_sum(float v, float* red) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (kThreads > 32) {
        if (l == 0) red[w] = v;
        __syncthreads();
        v = l < kThreads / 32 ? red[l] : 0.f;
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        __syncthreads();
    }
    return v;
}

constexpr int kNormThreads = 512;

// One CTA per row.  h is kept in shared memory between the two passes.
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(
    const void* __restrict__ x, const void* __restrict__ add, void* __restrict__ h_out,
    void* __restrict__ y, int64_t n, float eps, int dtype) {
    pdl_enter();
    extern __shared__ float hs[];
    __shared__ float red[32];
    const int64_t row = blockIdx.x;
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < n; i += kNormThreads) {
        float h = load_f(x, dtype, row * n + i);
        if (add) h = round_to(h + load_f(add, dtype, row * n + i), dtype);
        hs[i] = h;
        ss += h * h;
    }
    ss = block_sum<kNormThreads>(ss, red);
    const float r = rsqrtf(ss / (float)n + eps);
    for (int64_t i = threadIdx.x; i < n; i += kNormThreads) {
        const float h = hs[i];
        if (h_out) store_f(h_out, dtype, row * n + i, h);
        store_f(y, dtype, row * n + i, h * r);
    }
}

// One CTA of head_dim / 2 threads per (row, head); heads [0, H) are q heads,
// [H, H + KV) k heads (their v rows are copied alongside).
__global__ void __launch_bounds__(128) rope_kv_kernel(
    void* __restrict__ q, const void* __restrict__ k, const void* __restrict__ v,
    const int64_t* __restrict__ pos, int H, int KV, int hd, const float* __restrict__ cos_t,
    const float* __restrict__ sin_t, void* __restrict__ k_cache, void* __restrict__ v_cache,
    int qk_norm, float eps, int dtype, int64_t max_len) {
    pdl_enter();
    __shared__ float red[32];
    const int64_t row = blockIdx.x;
    const int head = blockIdx.y;
    const int half = hd / 2, i = threadIdx.x;
    const bool is_q = head < H;
    const int kh = head - H;
    const int64_t p = pos[row];
    if (p < 0 || p >= max_len) {   // uniform per CTA: nothing is written
        if (i == 0) atomicExch(&g_glue_position_error, 1);
        return;
    }
    const void* src = is_q ? static_cast<const void*>(q) : k;
    const int64_t base = is_q ? (row * H + head) * hd : (row * KV + kh) * hd;
    float x1 = load_f(src, dtype, base + i), x2 = load_f(src, dtype, base + i + half);
    if (qk_norm) {
        float ss = x1 * x1 + x2 * x2;
        if (half == 32) ss = block_sum<32>(ss, red);
        else if (half == 64) ss = block_sum<64>(ss, red);
        else ss = block_sum<128>(ss, red);
        const float r = rsqrtf(ss / (float)hd + eps);
        x1 = round_to(x1 * r, dtype);
        x2 = round_to(x2 * r, dtype);
    }
    const float c = cos_t[p * half + i], s = sin_t[p * half + i];
    const float o1 = x1 * c - x2 * s, o2 = x2 * c + x1 * s;
    if (is_q) {
        store_f(q, dtype, base + i, o1);
        store_f(q, dtype, base + i + half, o2);
    } else {
        const int64_t dst = (p * KV + kh) * hd;
        store_f(k_cache, dtype, dst + i, o1);
        store_f(k_cache, dtype, dst + i + half, o2);
        store_f(v_cache, dtype, dst + i, load_f(v, dtype, base + i));
        store_f(v_cache, dtype, dst + i + half, load_f(v, dtype, base + i + half));
    }
}

// bf16 rows of n = 8 * blockDim.x values: one 16-byte load per thread, values kept
// in registers between the sum of squares and the scaling.
__global__ void __launch_bounds__(1024) add_rmsnorm_bf16x8_kernel(
    const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ add,
    __nv_bfloat16* __restrict__ h_out, __nv_bfloat16* __restrict__ y, int64_t n, float eps) {
    pdl_enter();
    __shared__ float red[32];
    const int64_t off = blockIdx.x * n + 8 * threadIdx.x;
    const uint4 xr = *reinterpret_cast<const uint4*>(x + off);
    const __nv_bfloat16* xv = reinterpret_cast<const __nv_bfloat16*>(&xr);
    float h[8];
    if (add) {
        const uint4 ar = *reinterpret_cast<const uint4*>(add + off);
        const __nv_bfloat16* av = reinterpret_cast<const __nv_bfloat16*>(&ar);
#pragma unroll
        for (int e = 0; e < 8; ++e)
            h[e] = __bfloat162float(__float2bfloat16_rn(__bfloat162float(xv[e]) + __bfloat162float(av[e])));
    } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) h[e] = __bfloat162float(xv[e]);
    }
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += h[e] * h[e];
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31, nw = blockDim.x >> 5;
    if (l == 0) red[w] = ss;
    __syncthreads();
    ss = l < nw ? red[l] : 0.f;
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / (float)n + eps);
    uint4 hr, yr;
    __nv_bfloat16* hv = reinterpret_cast<__nv_bfloat16*>(&hr);
    __nv_bfloat16* yv = reinterpret_cast<__nv_bfloat16*>(&yr);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        hv[e] = __float2bfloat16_rn(h[e]);
        yv[e] = __float2bfloat16_rn(h[e] * r);
    }
    if (h_out) *reinterpret_cast<uint4*>(h_out + off) = hr;
    *reinterpret_cast<uint4*>(y + off) = yr;
}

// Split decode attention: CTA (kv head, split) takes a contiguous range of the
// positions 0..pos[0] for the kGroup query heads that read that kv head (each K/V
// row is loaded once for all of them); warp w takes every 8th position of the
// range, softmax is online per (warp, head); the CTA writes (max, sum, acc) per
// head to the workspace, and the last CTA of the kv head to finish (counter)
// merges the splits in split order and resets the counter.
constexpr int kAttnSplits = 16;
constexpr int kAttnWarps = 8;

template <int kDims, int kGroup>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_split_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k_cache,
    const __nv_bfloat16* __restrict__ v_cache, const int64_t* __restrict__ pos, int KV, float scale,
    __nv_bfloat16* __restrict__ out, float* __restrict__ ws, unsigned* __restrict__ counters, int64_t max_len) {
    pdl_enter();
    constexpr int hd = kDims * 32;
    constexpr int kRec = hd + 2;                       // acc[hd], max, sum
    __shared__ float wm[kAttnWarps][kGroup], wl[kAttnWarps][kGroup];
    __shared__ float wacc[kAttnWarps][kGroup][hd];
    __shared__ bool last;
    const int kvh = blockIdx.x, split = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (pos[0] < 0 || pos[0] >= max_len) {   // every CTA sees the same position: all return here
        if (split == 0) {
            for (int e = threadIdx.x; e < kGroup * hd; e += kAttnWarps * 32)
                out[(int64_t)kvh * kGroup * hd + e] = __float2bfloat16_rn(0.f);
            if (threadIdx.x == 0) atomicExch(&g_glue_position_error, 1);
        }
        return;
    }
    const int64_t n = pos[0] + 1;
    const int64_t chunk = (n + kAttnSplits - 1) / kAttnSplits;
    const int64_t t0 = split * chunk, t1 = min(n, t0 + chunk);
    float qv[kGroup][kDims], acc[kGroup][kDims], m[kGroup], l[kGroup];
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int d = 0; d < kDims; ++d) {
            qv[g][d] = __bfloat162float(q[(int64_t)(kvh * kGroup + g) * hd + lane * kDims + d]);
            acc[g][d] = 0.f;
        }
    }
    for (int64_t t = t0 + warp; t < t1; t += kAttnWarps) {
        const int64_t kb = (t * KV + kvh) * hd + lane * kDims;
        float kr[kDims], vr[kDims];
#pragma unroll
        for (int d = 0; d < kDims; ++d) {
            kr[d] = __bfloat162float(k_cache[kb + d]);
            vr[d] = __bfloat162float(v_cache[kb + d]);
        }
#pragma unroll
        for (int g = 0; g < kGroup; ++g) {
            float s = 0.f;
#pragma unroll
            for (int d = 0; d < kDims; ++d) s += qv[g][d] * kr[d];
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            s *= scale;
            const float mn = fmaxf(m[g], s);
            const float corr = expf(m[g] - mn), pw = expf(s - mn);
            l[g] = l[g] * corr + pw;
#pragma unroll
            for (int d = 0; d < kDims; ++d) acc[g][d] = acc[g][d] * corr + pw * vr[d];
            m[g] = mn;
        }
    }
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
        if (lane == 0) {
            wm[warp][g] = m[g];
            wl[warp][g] = l[g];
        }
#pragma unroll
        for (int d = 0; d < kDims; ++d) wacc[warp][g][lane * kDims + d] = acc[g][d];
    }
    __syncthreads();
    float* rec = ws + ((int64_t)(kvh * kAttnSplits + split) * kGroup) * kRec;
    for (int e = threadIdx.x; e < kGroup * hd; e += kAttnWarps * 32) {
        const int g = e / hd, d = e - g * hd;
        float mx = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, wm[w][g]);
        float num = 0.f, den = 0.f;
        for (int w = 0; w < kAttnWarps; ++w) {
            if (wm[w][g] == -INFINITY) continue;   // a warp that saw no position
            const float f = expf(wm[w][g] - mx);
            num += f * wacc[w][g][d];
            den += f * wl[w][g];
        }
        rec[g * kRec + d] = num;
        if (d == 0) {
            rec[g * kRec + hd] = mx;
            rec[g * kRec + hd + 1] = den;
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(&counters[kvh], 1u) == kAttnSplits - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    const float* base = ws + (int64_t)kvh * kAttnSplits * kGroup * kRec;
    for (int e = threadIdx.x; e < kGroup * hd; e += kAttnWarps * 32) {
        const int g = e / hd, d = e - g * hd;
        float mx = -INFINITY;
        for (int sp = 0; sp < kAttnSplits; ++sp) mx = fmaxf(mx, base[(sp * kGroup + g) * kRec + hd]);
        float num = 0.f, den = 0.f;
        for (int sp = 0; sp < kAttnSplits; ++sp) {
            const float* r = base + (sp * kGroup + g) * kRec;
            if (r[hd] == -INFINITY) continue;      // an empty split
            const float f = expf(r[hd] - mx);
            num += f * r[d];
            den += f * r[hd + 1];
        }
        out[(int64_t)(kvh * kGroup + g) * hd + d] = __float2bfloat16_rn(num / den);
    }
    if (threadIdx.x == 0) counters[kvh] = 0u;
}

// Decode attention with the q/k/v projections of the current token as inputs: the
// kernel applies (q/k RMSNorm and) RoPE to q and to this position's k itself, uses
// this position's k / v straight from registers, and split 0 writes them into the
// caches for later tokens (other CTAs only read earlier positions).  Otherwise as
// attn_split_kernel; replaces an epq_rope_kv + epq_attn_decode pair.
template <int kDims, int kGroup>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_rope_split_kernel(
    const __nv_bfloat16* __restrict__ q_in, const __nv_bfloat16* __restrict__ k_in,
    const __nv_bfloat16* __restrict__ v_in, __nv_bfloat16* __restrict__ k_cache,
    __nv_bfloat16* __restrict__ v_cache, const int64_t* __restrict__ pos, int KV,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, int qk_norm, float eps, float scale,
    __nv_bfloat16* __restrict__ out, float* __restrict__ ws, unsigned* __restrict__ counters, int64_t max_len) {
    pdl_enter();
    constexpr int hd = kDims * 32;
    constexpr int kRec = hd + 2;
    __shared__ float wm[kAttnWarps][kGroup], wl[kAttnWarps][kGroup];
    __shared__ float wacc[kAttnWarps][kGroup][hd];
    __shared__ bool last;
    const int kvh = blockIdx.x, split = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t P = pos[0];
    if (P < 0 || P >= max_len) {   // every CTA sees the same position: all return here
        if (split == 0) {
            for (int e = threadIdx.x; e < kGroup * hd; e += kAttnWarps * 32)
                out[(int64_t)kvh * kGroup * hd + e] = __float2bfloat16_rn(0.f);
            if (threadIdx.x == 0) atomicExch(&g_glue_position_error, 1);
        }
        return;
    }
    const int64_t n = P + 1;
    const int64_t chunk = (n + kAttnSplits - 1) / kAttnSplits;
    const int64_t t0 = split * chunk, t1 = min(n, t0 + chunk);
    float qv[kGroup][kDims], acc[kGroup][kDims], m[kGroup], l[kGroup];
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int d = 0; d < kDims; ++d) {
            qv[g][d] = __bfloat162float(q_in[(int64_t)(kvh * kGroup + g) * hd + lane * kDims + d]);
            acc[g][d] = 0.f;
        }
        rope_head<kDims>(qv[g], lane, P, cos_t, sin_t, qk_norm, eps);
    }
    float kc[kDims], vc[kDims];
#pragma unroll
    for (int d = 0; d < kDims; ++d) {
        kc[d] = __bfloat162float(k_in[(int64_t)kvh * hd + lane * kDims + d]);
        vc[d] = __bfloat162float(v_in[(int64_t)kvh * hd + lane * kDims + d]);
    }
    rope_head<kDims>(kc, lane, P, cos_t, sin_t, qk_norm, eps);
    if (split == 0 && warp == 0) {
        const int64_t cb = (P * KV + kvh) * hd + lane * kDims;
#pragma unroll
        for (int d = 0; d < kDims; ++d) {
            k_cache[cb + d] = __float2bfloat16_rn(kc[d]);
            v_cache[cb + d] = __float2bfloat16_rn(vc[d]);
        }
    }
    for (int64_t t = t0 + warp; t < t1; t += kAttnWarps) {
        float kr[kDims], vr[kDims];
        if (t == P) {
#pragma unroll
            for (int d = 0; d < kDims; ++d) {
                kr[d] = kc[d];
                vr[d] = vc[d];
            }
        } else {
            const int64_t kb = (t * KV + kvh) * hd + lane * kDims;
#pragma unroll
            for (int d = 0; d < kDims; ++d) {
                kr[d] = __bfloat162float(k_cache[kb + d]);
                vr[d] = __bfloat162float(v_cache[kb + d]);
            }
        }
#pragma unroll
        for (int g = 0; g < kGroup; ++g) {
            float s = 0.f;
#pragma unroll
            for (int d = 0; d < kDims; ++d) s += qv[g][d] * kr[d];
            for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
            s *= scale;
            const float mn = fmaxf(m[g], s);
            const float corr = expf(m[g] - mn), pw = expf(s - mn);
            l[g] = l[g] * corr + pw;
#pragma unroll
            for (int d = 0; d < kDims; ++d) acc[g][d] = acc[g][d] * corr + pw * vr[d];
            m[g] = mn;
        }
    }
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
        if (lane == 0) {
            wm[warp][g] = m[g];
            wl[warp][g] = l[g];
        }
#pragma unroll
        for (int d = 0; d < kDims; ++d) wacc[warp][g][lane * kDims + d] = acc[g][d];
    }
    __syncthreads();
    float* rec = ws + ((int64_t)(kvh * kAttnSplits + split) * kGroup) * kRec;
    for (int e = threadIdx.x; e < kGroup * hd; e += kAttnWarps * 32) {
        const int g = e / hd, d = e - g * hd;
        float mx = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, wm[w][g]);
        float num = 0.f, den = 0.f;
        for (int w = 0; w < kAttnWarps; ++w) {
            if (wm[w][g] == -INFINITY) continue;
            const float f = expf(wm[w][g] - mx);
            num += f * wacc[w][g][d];
            den += f * wl[w][g];
        }
        rec[g * kRec + d] = num;
        if (d == 0) {
            rec[g * kRec + hd] = mx;
            rec[g * kRec + hd + 1] = den;
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(&counters[kvh], 1u) == kAttnSplits - 1;
    __syncthreads();
    if (!last) return;
    __threadfence();
    const float* base = ws + (int64_t)kvh * kAttnSplits * kGroup * kRec;
    for (int e = threadIdx.x; e < kGroup * hd; e += kAttnWarps * 32) {
        const int g = e / hd, d = e - g * hd;
        float mx = -INFINITY;
        for (int sp = 0; sp < kAttnSplits; ++sp) mx = fmaxf(mx, base[(sp * kGroup + g) * kRec + hd]);
        float num = 0.f, den = 0.f;
        for (int sp = 0; sp < kAttnSplits; ++sp) {
            const float* r = base + (sp * kGroup + g) * kRec;
            if (r[hd] == -INFINITY) continue;
            const float f = expf(r[hd] - mx);
            num += f * r[d];
            den += f * r[hd + 1];
        }
        out[(int64_t)(kvh * kGroup + g) * hd + d] = __float2bfloat16_rn(num / den);
    }
    if (threadIdx.x == 0) counters[kvh] = 0u;
}

// Decode attention as thread-block clusters: the kClusterSplits CTAs of one
// cluster split the positions of one kv head, and their partial softmax
// records are merged over distributed shared memory, each CTA merging one slice
// of the kv head's outputs
// (no workspace round trip, fence or completion counter).  Otherwise as
// attn_rope_split_kernel: (q/k RMSNorm and) RoPE inside, this position's k / v
// from registers and written into the caches by rank 0; each warp prefetches
// the K / V rows of its next position while it scores the current one.
constexpr int kClusterSplits = 8;

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_cluster_f32(const float* local, uint32_t rank) {
    uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(local)), r;
    float v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(r) : "memory");
    return v;
}

// Cached rows a CTA stages in shared memory per pass.
constexpr int kClusterRows = 64;

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gsrc) : "memory");
}

// Rows [base, base + cnt) of kv head kvh except position P into kst / vst, as
// asynchronous 16-byte copies.
template <int kDims>
__device__ __forceinline__ void stage_rows(const __nv_bfloat16* k_cache, const __nv_bfloat16* v_cache, int KV,
                                           int kvh, int64_t base, int cnt, int64_t P, __nv_bfloat16* kst,
                                           __nv_bfloat16* vst) {
    constexpr int hd = kDims * 32, pieces = hd / 8;
    for (int i = threadIdx.x; i < cnt * pieces; i += kAttnWarps * 32) {
        const int r = i / pieces, c = i - r * pieces;
        const int64_t t = base + r;
        if (t == P) continue;
        const int64_t off = (t * KV + kvh) * hd + c * 8;
        cp_async16(kst + r * hd + c * 8, k_cache + off);
        cp_async16(vst + r * hd + c * 8, v_cache + off);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int kDims, int kGroup>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_rope_cluster_kernel(
    const __nv_bfloat16* __restrict__ q_in, const __nv_bfloat16* __restrict__ k_in,
    const __nv_bfloat16* __restrict__ v_in, __nv_bfloat16* __restrict__ k_cache,
    __nv_bfloat16* __restrict__ v_cache, const int64_t* __restrict__ pos, int KV,
    const float* __restrict__ cos_t, const float* __restrict__ sin_t, int qk_norm, float eps, float scale,
    __nv_bfloat16* __restrict__ out, int64_t max_len) {
    constexpr int hd = kDims * 32;
    constexpr int kRec = hd + 2;                   // merged acc[hd], max, sum of one head
    __shared__ float wm[kAttnWarps][kGroup], wl[kAttnWarps][kGroup];
    __shared__ float wacc[kAttnWarps][kGroup][hd];
    __shared__ float rec[kGroup * kRec];            // this CTA's record, read by the whole cluster
    extern __shared__ __align__(16) uint8_t dyn[];  // the staged K / V rows
    __nv_bfloat16* kst = reinterpret_cast<__nv_bfloat16*>(dyn);
    __nv_bfloat16* vst = kst + kClusterRows * hd;
    const int split = blockIdx.x, kvh = blockIdx.y;   // the cluster spans the splits of one kv head
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // The position and the cached rows before it were written by launches that
    // completed before this grid's predecessor started (the previous token's
    // position update and attention), so they are read before the dependency
    // wait: the first pass of K / V rows streams in while the q / k / v
    // projection that precedes this kernel is still finishing.
    const int64_t P = pos[0];
    const bool valid = P >= 0 && P < max_len;
    const int64_t n = P + 1;
    const int64_t chunk = (n + kClusterSplits - 1) / kClusterSplits;
    const int64_t t0 = split * chunk, t1 = valid ? min(n, t0 + chunk) : t0;
    int64_t base = t0;
    int cnt = (int)min((int64_t)kClusterRows, t1 - base);
    if (cnt > 0) stage_rows<kDims>(k_cache, v_cache, KV, kvh, base, cnt, P, kst, vst);
    pdl_enter();
    if (!valid) {   // the same position for every CTA: the whole cluster returns here
        asm volatile("cp.async.wait_all;" ::: "memory");
        if (split == 0) {
            for (int e = threadIdx.x; e < kGroup * hd; e += kAttnWarps * 32)
                out[(int64_t)kvh * kGroup * hd + e] = __float2bfloat16_rn(0.f);
            if (threadIdx.x == 0) atomicExch(&g_glue_position_error, 1);
        }
        return;
    }
    float qv[kGroup][kDims], acc[kGroup][kDims], m[kGroup], l[kGroup];
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int d = 0; d < kDims; ++d) {
            qv[g][d] = __bfloat162float(q_in[(int64_t)(kvh * kGroup + g) * hd + lane * kDims + d]);
            acc[g][d] = 0.f;
        }
        rope_head<kDims>(qv[g], lane, P, cos_t, sin_t, qk_norm, eps);
    }
    float kc[kDims], vc[kDims];
#pragma unroll
    for (int d = 0; d < kDims; ++d) {
        kc[d] = __bfloat162float(k_in[(int64_t)kvh * hd + lane * kDims + d]);
        vc[d] = __bfloat162float(v_in[(int64_t)kvh * hd + lane * kDims + d]);
    }
    rope_head<kDims>(kc, lane, P, cos_t, sin_t, qk_norm, eps);
    if (split == 0 && warp == 0) {
        const int64_t cb = (P * KV + kvh) * hd + lane * kDims;
#pragma unroll
        for (int d = 0; d < kDims; ++d) {
            k_cache[cb + d] = __float2bfloat16_rn(kc[d]);
            v_cache[cb + d] = __float2bfloat16_rn(vc[d]);
        }
    }
    while (cnt > 0) {
        asm volatile("cp.async.wait_all;" ::: "memory");
        if (warp == 0 && P >= base && P < base + cnt) {   // this position from registers
#pragma unroll
            for (int d = 0; d < kDims; ++d) {
                kst[(P - base) * hd + lane * kDims + d] = __float2bfloat16_rn(kc[d]);
                vst[(P - base) * hd + lane * kDims + d] = __float2bfloat16_rn(vc[d]);
            }
        }
        __syncthreads();
        // each warp scores every kAttnWarps-th staged row, four at a time
        for (int j0 = warp; j0 < cnt; j0 += 4 * kAttnWarps) {
            float kr[4][kDims];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int j = min(j0 + u * kAttnWarps, cnt - 1);
#pragma unroll
                for (int d = 0; d < kDims; ++d) kr[u][d] = __bfloat162float(kst[j * hd + lane * kDims + d]);
            }
#pragma unroll
            for (int g = 0; g < kGroup; ++g) {
                float sc[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    float a = 0.f;
#pragma unroll
                    for (int d = 0; d < kDims; ++d) a += qv[g][d] * kr[u][d];
                    sc[u] = a;
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                    for (int u = 0; u < 4; ++u) sc[u] += __shfl_xor_sync(0xffffffffu, sc[u], o);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int j = j0 + u * kAttnWarps;
                    if (j >= cnt) break;
                    const float s = sc[u] * scale;
                    const float mn = fmaxf(m[g], s);
                    const float corr = expf(m[g] - mn), pw = expf(s - mn);
                    l[g] = l[g] * corr + pw;
#pragma unroll
                    for (int d = 0; d < kDims; ++d)
                        acc[g][d] = acc[g][d] * corr + pw * __bfloat162float(vst[j * hd + lane * kDims + d]);
                    m[g] = mn;
                }
            }
        }
        base += cnt;
        cnt = (int)min((int64_t)kClusterRows, t1 - base);
        __syncthreads();   // every warp is done with the staged rows
        if (cnt > 0) stage_rows<kDims>(k_cache, v_cache, KV, kvh, base, cnt, P, kst, vst);
    }
#pragma unroll
    for (int g = 0; g < kGroup; ++g) {
        if (lane == 0) {
            wm[warp][g] = m[g];
            wl[warp][g] = l[g];
        }
#pragma unroll
        for (int d = 0; d < kDims; ++d) wacc[warp][g][lane * kDims + d] = acc[g][d];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < kGroup * hd; e += kAttnWarps * 32) {
        const int g = e / hd, d = e - g * hd;
        float mx = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, wm[w][g]);
        float num = 0.f, den = 0.f;
        for (int w = 0; w < kAttnWarps; ++w) {
            if (wm[w][g] == -INFINITY) continue;
            const float f = expf(wm[w][g] - mx);
            num += f * wacc[w][g][d];
            den += f * wl[w][g];
        }
        rec[g * kRec + d] = num;
        if (d == 0) {
            rec[g * kRec + hd] = mx;
            rec[g * kRec + hd + 1] = den;
        }
    }
    cluster_sync_all();   // every split's record is in its shared memory
    {
        // Every CTA of the cluster merges one slice of the kv head's outputs, so the
        // merge's dependent remote loads run once per thread (rank 0 alone took two turns).
        constexpr int kSlice = (kGroup * hd + kClusterSplits - 1) / kClusterSplits;
        const int e_end = min(kGroup * hd, (split + 1) * kSlice);
        for (int e = split * kSlice + threadIdx.x; e < e_end; e += kAttnWarps * 32) {
            const int g = e / hd, d = e - g * hd;
            float mxs[kClusterSplits];
            float mx = -INFINITY;
#pragma unroll
            for (int r = 0; r < kClusterSplits; ++r) {
                mxs[r] = ld_cluster_f32(&rec[g * kRec + hd], (uint32_t)r);
                mx = fmaxf(mx, mxs[r]);
            }
            float num = 0.f, den = 0.f;
#pragma unroll
            for (int r = 0; r < kClusterSplits; ++r) {
                if (mxs[r] == -INFINITY) continue;   // a split that saw no position
                const float f = expf(mxs[r] - mx);
                num += f * ld_cluster_f32(&rec[g * kRec + d], (uint32_t)r);
                den += f * ld_cluster_f32(&rec[g * kRec + hd + 1], (uint32_t)r);
            }
            out[(int64_t)(kvh * kGroup + g) * hd + d] = __float2bfloat16_rn(num / den);
        }
    }
    cluster_sync_all();   // no CTA leaves while another still reads its record
}

// Arg-max of n floats (first index of the maximum, as torch.argmax): every CTA
// reduces a strided share, the last CTA to finish merges the per-CTA results.
constexpr int kArgBlocks = 64;

__global__ void __launch_bounds__(256) argmax_kernel(const float* __restrict__ x, int64_t n,
                                                     int64_t* __restrict__ out, float* __restrict__ wv,
                                                     int64_t* __restrict__ wi, unsigned* __restrict__ counter) {
    pdl_enter();
    __shared__ float sv[256];
    __shared__ int64_t si[256];
    __shared__ bool last;
    float bv = -INFINITY;
    int64_t bi = n;
    for (int64_t i = blockIdx.x * 256 + threadIdx.x; i < n; i += (int64_t)gridDim.x * 256) {
        const float v = x[i];
        if (v > bv) {                                   // strided order: indices increase
            bv = v;
            bi = i;
        }
    }
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (int s2 = 128; s2 > 0; s2 >>= 1) {
        if (threadIdx.x < s2) {
            const float ov = sv[threadIdx.x + s2];
            const int64_t oi = si[threadIdx.x + s2];
            if (ov > sv[threadIdx.x] || (ov == sv[threadIdx.x] && oi < si[threadIdx.x])) {
                sv[threadIdx.x] = ov;
                si[threadIdx.x] = oi;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        wv[blockIdx.x] = sv[0];
        wi[blockIdx.x] = si[0];
        __threadfence();
        last = atomicAdd(counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    __threadfence();
    float v = wv[0];
    int64_t id = wi[0];
    for (unsigned b = 1; b < gridDim.x; ++b) {
        const float ov = wv[b];
        const int64_t oi = wi[b];
        if (ov > v || (ov == v && oi < id)) {
            v = ov;
            id = oi;
        }
    }
    *out = id;
    *counter = 0u;
}

// One CTA per query head.  Warp w takes positions w, w + 8, ...: a lane holds
// hd / 32 dimensions, the score is a warp sum, softmax is online per warp and
// the warps are merged at the end (fixed order).
template <int kDims>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_decode_kernel(
    const void* __restrict__ q, const void* __restrict__ k_cache, const void* __restrict__ v_cache,
    const int64_t* __restrict__ pos, int H, int KV, float scale, void* __restrict__ out, int dtype,
    int64_t max_len) {
    pdl_enter();
    constexpr int hd = kDims * 32;
    __shared__ float wm[kAttnWarps], wl[kAttnWarps];
    __shared__ float wacc[kAttnWarps][hd];
    const int head = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kvh = head / (H / KV);
    const int64_t P = pos[0];
    if (P < 0 || P >= max_len) {
        for (int e = threadIdx.x; e < hd; e += kAttnWarps * 32) store_f(out, dtype, (int64_t)head * hd + e, 0.f);
        if (threadIdx.x == 0) atomicExch(&g_glue_position_error, 1);
        return;
    }
    float qv[kDims];
#pragma unroll
    for (int d = 0; d < kDims; ++d) qv[d] = load_f(q, dtype, (int64_t)head * hd + lane * kDims + d);
    float m = -INFINITY, l = 0.f, acc[kDims];
#pragma unroll
    for (int d = 0; d < kDims; ++d) acc[d] = 0.f;
    for (int64_t t = warp; t <= P; t += kAttnWarps) {
        const int64_t kb = (t * KV + kvh) * hd + lane * kDims;
        float s = 0.f;
#pragma unroll
        for (int d = 0; d < kDims; ++d) s += qv[d] * load_f(k_cache, dtype, kb + d);
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        s *= scale;
        const float mn = fmaxf(m, s);
        const float corr = expf(m - mn), pw = expf(s - mn);
        l = l * corr + pw;
#pragma unroll
        for (int d = 0; d < kDims; ++d) acc[d] = acc[d] * corr + pw * load_f(v_cache, dtype, kb + d);
        m = mn;
    }
    if (lane == 0) {
        wm[warp] = m;
        wl[warp] = l;
    }
#pragma unroll
    for (int d = 0; d < kDims; ++d) wacc[warp][lane * kDims + d] = acc[d];
    __syncthreads();
    for (int d = threadIdx.x; d < hd; d += kAttnWarps * 32) {
        float mx = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) mx = fmaxf(mx, wm[w]);
        float num = 0.f, den = 0.f;
        for (int w = 0; w < kAttnWarps; ++w) {
            if (wm[w] == -INFINITY) continue;      // a warp that saw no position
            const float f = expf(wm[w] - mx);
            num += f * wacc[w][d];
            den += f * wl[w];
        }
        store_f(out, dtype, (int64_t)head * hd + d, num / den);
    }
}

__global__ void silu_mul_kernel(const void* __restrict__ g, const void* __restrict__ u,
                                void* __restrict__ out, int64_t n, int dtype) {
    pdl_enter();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float gv = load_f(g, dtype, i);
        store_f(out, dtype, i, gv / (1.f + expf(-gv)) * load_f(u, dtype, i));
    }
}

bool glue_dtype_ok(int d) { return d == EPQ_F32 || d == EPQ_F16 || d == EPQ_BF16; }

}  // namespace

int glue_read_device_error(int* flag) {
    if (cudaMemcpyFromSymbol(flag, g_glue_position_error, sizeof(int)) != cudaSuccess)
        return check_launch("read decode glue error flag");
    return EPQ_OK;
}

}  // namespace epq

using namespace epq;

extern "C" {

int epq_add_rmsnorm(const void* x, const void* add, void* h_out, void* y, int64_t m, int64_t n,
                    float eps, int32_t dtype, void* stream) {
    if (!x || !y || m < 0 || n <= 0) return set_error(EPQ_EINVAL, "epq_add_rmsnorm: bad arguments");
    if (!glue_dtype_ok(dtype)) return set_error(EPQ_EDTYPE, "epq_add_rmsnorm: dtype %d", dtype);
    if (n > 12288) return set_error(EPQ_EUNSUPPORTED, "epq_add_rmsnorm: n=%lld > 12288", (long long)n);
    if (m == 0) return EPQ_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const bool aligned = ((uintptr_t)x | (uintptr_t)add | (uintptr_t)h_out | (uintptr_t)y) % 16 == 0;
    if (dtype == EPQ_BF16 && aligned && n % 256 == 0 && n / 8 <= 1024) {
        return launch_pdl(add_rmsnorm_bf16x8_kernel, dim3((unsigned)m), dim3((unsigned)(n / 8)), 0, st,
                          "epq_add_rmsnorm", static_cast<const __nv_bfloat16*>(x),
                          static_cast<const __nv_bfloat16*>(add), static_cast<__nv_bfloat16*>(h_out),
                          static_cast<__nv_bfloat16*>(y), n, eps);
    }
    return launch_pdl(add_rmsnorm_kernel, dim3((unsigned)m), dim3(kNormThreads), n * sizeof(float), st,
                      "epq_add_rmsnorm", x, add, h_out, y, n, eps, (int)dtype);
}

int epq_rope_kv(void* q, const void* k, const void* v, const int64_t* pos, int64_t m, int32_t heads,
                int32_t kv_heads, int32_t head_dim, const float* cos_tab, const float* sin_tab,
                void* k_cache, void* v_cache, int64_t max_len, int32_t qk_norm, float eps, int32_t dtype,
                void* stream) {
    if (!q || !k || !v || !pos || !cos_tab || !sin_tab || !k_cache || !v_cache || m < 0 || max_len <= 0)
        return set_error(EPQ_EINVAL, "epq_rope_kv: bad arguments");
    if (!glue_dtype_ok(dtype)) return set_error(EPQ_EDTYPE, "epq_rope_kv: dtype %d", dtype);
    if ((head_dim != 64 && head_dim != 128 && head_dim != 256) || heads <= 0 || kv_heads <= 0 ||
        heads % kv_heads)
        return set_error(EPQ_EUNSUPPORTED, "epq_rope_kv: head_dim=%d (64, 128 or 256), heads=%d, kv_heads=%d",
                         head_dim, heads, kv_heads);
    if (m == 0) return EPQ_OK;
    return launch_pdl(rope_kv_kernel, dim3((unsigned)m, heads + kv_heads), dim3(head_dim / 2), 0,
                      static_cast<cudaStream_t>(stream), "epq_rope_kv", q, k, v, pos, (int)heads,
                      (int)kv_heads, (int)head_dim, cos_tab, sin_tab, k_cache, v_cache, (int)qk_norm, eps,
                      (int)dtype, max_len);
}

int64_t epq_attn_decode_workspace_bytes(int32_t heads, int32_t kv_heads, int32_t head_dim) {
    if (heads <= 0 || kv_heads <= 0 || heads % kv_heads || head_dim <= 0) return 0;
    return 256 + (int64_t)kv_heads * kAttnSplits * (heads / kv_heads) * (head_dim + 2) * 4;
}

int epq_attn_decode(const void* q, const void* k_cache, const void* v_cache, const int64_t* pos,
                    int64_t max_len, int32_t heads, int32_t kv_heads, int32_t head_dim, float scale, void* out,
                    int32_t dtype, void* workspace, int64_t workspace_bytes, void* stream) {
    if (!q || !k_cache || !v_cache || !pos || !out || heads <= 0 || kv_heads <= 0 || heads % kv_heads ||
        max_len <= 0)
        return set_error(EPQ_EINVAL, "epq_attn_decode: bad arguments");
    if (!glue_dtype_ok(dtype)) return set_error(EPQ_EDTYPE, "epq_attn_decode: dtype %d", dtype);
    if (head_dim != 64 && head_dim != 128)
        return set_error(EPQ_EUNSUPPORTED, "epq_attn_decode: head_dim=%d (64 or 128)", head_dim);
    if (kv_heads > 256) return set_error(EPQ_EUNSUPPORTED, "epq_attn_decode: kv_heads=%d > 256", kv_heads);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int group = heads / kv_heads;
    const bool split = dtype == EPQ_BF16 && workspace &&
                       (group == 1 || group == 2 || group == 4 || group == 8);
    if (split) {
        if (workspace_bytes < epq_attn_decode_workspace_bytes(heads, kv_heads, head_dim) ||
            (uintptr_t)workspace % 256)
            return set_error(EPQ_EWORKSPACE, "epq_attn_decode: workspace of %lld bytes (need %lld, 256-aligned)",
                             (long long)workspace_bytes,
                             (long long)epq_attn_decode_workspace_bytes(heads, kv_heads, head_dim));
        unsigned* ctr = static_cast<unsigned*>(workspace);
        float* ws = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 256);
        const auto* qb = static_cast<const __nv_bfloat16*>(q);
        const auto* kb = static_cast<const __nv_bfloat16*>(k_cache);
        const auto* vb = static_cast<const __nv_bfloat16*>(v_cache);
        auto* ob = static_cast<__nv_bfloat16*>(out);
        const dim3 grid(kv_heads, kAttnSplits);
#define EPQ_ATTN_SPLIT(D, G) return launch_pdl(attn_split_kernel<D, G>, grid, dim3(kAttnWarps * 32), 0, st, \
                                             "epq_attn_decode", qb, kb, vb, pos, (int)kv_heads, scale, ob, ws, ctr, max_len)
        if (head_dim == 128) {
            if (group == 1) EPQ_ATTN_SPLIT(4, 1);
            else if (group == 2) EPQ_ATTN_SPLIT(4, 2);
            else if (group == 4) EPQ_ATTN_SPLIT(4, 4);
            else EPQ_ATTN_SPLIT(4, 8);
        } else {
            if (group == 1) EPQ_ATTN_SPLIT(2, 1);
            else if (group == 2) EPQ_ATTN_SPLIT(2, 2);
            else if (group == 4) EPQ_ATTN_SPLIT(2, 4);
            else EPQ_ATTN_SPLIT(2, 8);
        }
#undef EPQ_ATTN_SPLIT
    } else if (head_dim == 128) {
        return launch_pdl(attn_decode_kernel<4>, dim3(heads), dim3(kAttnWarps * 32), 0, st, "epq_attn_decode",
                          q, k_cache, v_cache, pos, (int)heads, (int)kv_heads, scale, out, (int)dtype, max_len);
    } else {
        return launch_pdl(attn_decode_kernel<2>, dim3(heads), dim3(kAttnWarps * 32), 0, st, "epq_attn_decode",
                          q, k_cache, v_cache, pos, (int)heads, (int)kv_heads, scale, out, (int)dtype, max_len);
    }
    return check_launch("epq_attn_decode");
}

int epq_attn_rope_decode(const void* q, const void* k, const void* v, const int64_t* pos, int32_t heads,
                         int32_t kv_heads, int32_t head_dim, const float* cos_tab, const float* sin_tab,
                         void* k_cache, void* v_cache, int64_t max_len, int32_t qk_norm, float eps, float scale,
                         void* out, int32_t dtype, void* workspace, int64_t workspace_bytes, void* stream) {
    if (!q || !k || !v || !pos || !cos_tab || !sin_tab || !k_cache || !v_cache || !out || !workspace ||
        heads <= 0 || kv_heads <= 0 || heads % kv_heads || max_len <= 0)
        return set_error(EPQ_EINVAL, "epq_attn_rope_decode: bad arguments");
    const int group = heads / kv_heads;
    if (dtype != EPQ_BF16 || (head_dim != 64 && head_dim != 128) ||
        !(group == 1 || group == 2 || group == 4 || group == 8))
        return set_error(EPQ_EUNSUPPORTED, "epq_attn_rope_decode: bf16, head_dim 64/128, heads/kv_heads 1/2/4/8 "
                         "(got dtype %d, head_dim %d, %d/%d)", dtype, head_dim, heads, kv_heads);
    if (workspace_bytes < epq_attn_decode_workspace_bytes(heads, kv_heads, head_dim) || (uintptr_t)workspace % 256)
        return set_error(EPQ_EWORKSPACE, "epq_attn_rope_decode: workspace of %lld bytes (need %lld, 256-aligned)",
                         (long long)workspace_bytes,
                         (long long)epq_attn_decode_workspace_bytes(heads, kv_heads, head_dim));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const auto* qb = static_cast<const __nv_bfloat16*>(q);
    const auto* kb = static_cast<const __nv_bfloat16*>(k);
    const auto* vb = static_cast<const __nv_bfloat16*>(v);
    auto* kcb = static_cast<__nv_bfloat16*>(k_cache);
    auto* vcb = static_cast<__nv_bfloat16*>(v_cache);
    auto* ob = static_cast<__nv_bfloat16*>(out);
    const dim3 grid(kClusterSplits, kv_heads);
#define EPQ_ATTN_ROPE(D, G)                                                                                     \
    return launch_pdl_cluster(attn_rope_cluster_kernel<D, G>, grid, dim3(kAttnWarps * 32), kClusterSplits,     \
                              (size_t)(2 * kClusterRows * D * 32 * 2), st,                                     \
                              "epq_attn_rope_decode", qb, kb, vb, kcb, vcb, pos, (int)kv_heads, cos_tab, sin_tab,  \
                              (int)qk_norm, eps, scale, ob, max_len)
    if (head_dim == 128) {
        if (group == 1) EPQ_ATTN_ROPE(4, 1);
        if (group == 2) EPQ_ATTN_ROPE(4, 2);
        if (group == 4) EPQ_ATTN_ROPE(4, 4);
        EPQ_ATTN_ROPE(4, 8);
    }
    if (group == 1) EPQ_ATTN_ROPE(2, 1);
    if (group == 2) EPQ_ATTN_ROPE(2, 2);
    if (group == 4) EPQ_ATTN_ROPE(2, 4);
    EPQ_ATTN_ROPE(2, 8);
#undef EPQ_ATTN_ROPE
}

int64_t epq_argmax_workspace_bytes(void) { return 256 + kArgBlocks * (4 + 8); }

int epq_argmax(const float* x, int64_t n, int64_t* out, void* workspace, int64_t workspace_bytes,
               void* stream) {
    if (!x || !out || n <= 0 || !workspace) return set_error(EPQ_EINVAL, "epq_argmax: bad arguments");
    if (workspace_bytes < epq_argmax_workspace_bytes() || (uintptr_t)workspace % 256)
        return set_error(EPQ_EWORKSPACE, "epq_argmax: workspace of %lld bytes (need %lld, 256-aligned)",
                         (long long)workspace_bytes, (long long)epq_argmax_workspace_bytes());
    uint8_t* w = static_cast<uint8_t*>(workspace);
    return launch_pdl(argmax_kernel, dim3(kArgBlocks), dim3(256), 0, static_cast<cudaStream_t>(stream),
                      "epq_argmax", x, n, out, reinterpret_cast<float*>(w + 256),
                      reinterpret_cast<int64_t*>(w + 256 + kArgBlocks * 4), reinterpret_cast<unsigned*>(w));
}

int epq_silu_mul(const void* g, const void* u, void* out, int64_t n, int32_t dtype, void* stream) {
    if (!g || !u || !out || n < 0) return set_error(EPQ_EINVAL, "epq_silu_mul: bad arguments");
    if (!glue_dtype_ok(dtype)) return set_error(EPQ_EDTYPE, "epq_silu_mul: dtype %d", dtype);
    if (n == 0) return EPQ_OK;
    const int64_t blocks = (n + 255) / 256;
    return launch_pdl(silu_mul_kernel, dim3((unsigned)(blocks < 1184 ? blocks : 1184)), dim3(256), 0,
                      static_cast<cudaStream_t>(stream), "epq_silu_mul", g, u, out, n, (int)dtype);
}

}  // extern "C"
