// Per-head RoPE shared by the decode glue kernels and the decode program.
#pragma once

#include <cuda_bf16.h>

namespace epq {

// RoPE (rotate-half) of a head vector held kDims dims per lane: lane l holds dims
// kDims*l .. +kDims-1; dim i pairs with i + hd/2, held by lane l ^ 16.  Optional
// per-head RMSNorm first (rounded to bf16, as the q/k tensors of the model are),
// result rounded to bf16.
template <int kDims>
__device__ __forceinline__ void rope_head(float (&v)[kDims], int lane, int64_t p, const float* cos_t,
                                          const float* sin_t, int qk_norm, float eps) {
    constexpr int hd = kDims * 32, half = hd / 2;
    if (qk_norm) {
        float ss = 0.f;
#pragma unroll
        for (int d = 0; d < kDims; ++d) ss += v[d] * v[d];
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        const float r = rsqrtf(ss / (float)hd + eps);
#pragma unroll
        for (int d = 0; d < kDims; ++d) v[d] = __bfloat162float(__float2bfloat16_rn(v[d] * r));
    }
    const bool lo = lane < 16;
#pragma unroll
    for (int d = 0; d < kDims; ++d) {
        const float other = __shfl_xor_sync(0xffffffffu, v[d], 16);
        const int i = (kDims * lane + d) & (half - 1);
        const float c = cos_t[p * half + i], s = sin_t[p * half + i];
        const float x1 = lo ? v[d] : other, x2 = lo ? other : v[d];
        const float o = lo ? x1 * c - x2 * s : x2 * c + x1 * s;
        v[d] = __bfloat162float(__float2bfloat16_rn(o));
    }
}

}  // namespace epq
