// Shared device helpers for the epq kernels: element loads in any of the three
// float types, index lookups in both layouts, and the host-side error state.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

#include "epq.h"

namespace epq {

// ---------------------------------------------------------------------------
// element access
// ---------------------------------------------------------------------------
__device__ __forceinline__ float load_f(const void* p, int dtype, int64_t i) {
    switch (dtype) {
        case EPQ_F16: return __half2float(static_cast<const __half*>(p)[i]);
        case EPQ_BF16: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
        default: return static_cast<const float*>(p)[i];
    }
}

__device__ __forceinline__ void store_f(void* p, int dtype, int64_t i, float v) {
    switch (dtype) {
        case EPQ_F16: static_cast<__half*>(p)[i] = __float2half_rn(v); break;
        case EPQ_BF16: static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
        default: static_cast<float*>(p)[i] = v; break;
    }
}

// Round a float to the nearest value of `dtype` (ties to even), as torch's
// dtype casts do; used where the reference rounds intermediate values.
__device__ __forceinline__ float round_to(float v, int dtype) {
    switch (dtype) {
        case EPQ_F16: return __half2float(__float2half_rn(v));
        case EPQ_BF16: return __bfloat162float(__float2bfloat16_rn(v));
        default: return v;
    }
}

// Device copy of the store description, with derived sizes.
struct StoreD {
    const uint8_t* idx;
    int layout, bits, vec, levels, group;
    int cb_dtype, scale_dtype;
    const void* cb;
    const void* scale;
    int64_t s_n, s_g;
    int64_t n, k;
    int64_t ng;   // groups along k
    int64_t rb;   // 16-row blocks (tiled layout)
    int64_t p;    // index positions per group (tiled layout)
    int64_t kpos; // index positions per row = k / vec
};

// Codebook index of weight (r, c); c is the weight column.
__device__ __forceinline__ int index_at(const StoreD& s, int64_t r, int64_t c) {
    if (s.layout == EPQ_LAYOUT_TILED) {
        const int64_t j = c / s.vec;
        const int64_t g = j / s.p, l = j - g * s.p;
        const int64_t b = r >> 4, rr = r & 15;
        return s.idx[((g * s.rb + b) * s.p + l) * 16 + rr];
    }
    if (s.layout == EPQ_LAYOUT_MMA16) {   // P = 32: lane 4*(r%8) + j%4, byte 8*((r%16)/8) + (j%32)/4
        const int64_t j = c / s.vec;
        const int64_t g = j >> 5, jj = j & 31;
        const int64_t b = r >> 4, lane = 4 * (r & 7) + (jj & 3);
        return s.idx[((b * s.ng + g) * 32 + lane) * 16 + 8 * ((r >> 3) & 1) + (jj >> 2)];
    }
    if (s.vec == 4) return s.idx[r * s.kpos + (c >> 2)];
    const int64_t f = r * s.k + c;  // flat position in the _pack4 stream
    if (s.bits == 4) {
        const uint8_t byte = s.idx[f >> 1];
        return (f & 1) ? (byte >> 4) : (byte & 0x0F);
    }
    return s.idx[f];
}

__device__ __forceinline__ float scale_at(const StoreD& s, int64_t r, int64_t g) {
    return load_f(s.scale, s.scale_dtype, r * s.s_n + g * s.s_g);
}

// ---------------------------------------------------------------------------
// host-side helpers
// ---------------------------------------------------------------------------
int set_error(int code, const char* fmt, ...);
// Raises kernel `fn`'s dynamic shared-memory limit to `bytes` on the current
// device, once per (kernel, device, bytes); thread-safe (epq_capi.cu).
int set_smem_limit(const void* fn, int bytes, const char* who);
// The current device's SM count, cached per device; thread-safe.
int device_sms();
int check_launch(const char* what);
int make_store(const epq_store* in, StoreD* out, const char* who);

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

inline int dtype_size(int dtype) { return dtype == EPQ_F32 ? 4 : 2; }

inline bool dtype_ok(int dtype) {
    return dtype == EPQ_F32 || dtype == EPQ_F16 || dtype == EPQ_BF16;
}

// Kernel launchers (defined in the .cu files).
int launch_linear_generic(const StoreD& s, const void* x, int x_dtype, int64_t m, int64_t ldx,
                          void* out, int64_t ldo, int out_dtype, cudaStream_t st);
int launch_bwd_generic(const StoreD& s, const void* x, int64_t ldx, const void* dy, int64_t ldy,
                       int act_dtype, int64_t m, void* dx, int64_t lddx, int dx_dtype,
                       float* dscale, float* dcb, cudaStream_t st);
int launch_materialize(const StoreD& s, void* w, int64_t ldw, int out_dtype, cudaStream_t st);
int64_t layout_bytes(int layout, int64_t n, int64_t k, int vec, int group);
int launch_relayout(const uint8_t* src, int layout, int64_t n, int64_t k, int vec, int group,
                    uint8_t* dst, cudaStream_t st);

// Persistent chain kernel (k_chain_lut.cu).
struct ChainStepD;
struct ChainHeaderD;
int chain_grid(int* grid);
int chain_read_device_error(int* flag);
int launch_embedding(const StoreD& s, const int64_t* ids, int64_t n_ids, void* out, int64_t ldo,
                     int out_dtype, cudaStream_t st);
int embed_read_device_error(int* flag);

// Small-batch tensor-core GEMV over EPQ_LAYOUT_MMA16 stores (k_gemv_mma.cu).
bool mma_eligible(const StoreD& s, int64_t m, int x_dtype);
int launch_linear_mma(const StoreD* s, int count, const void* x, int x_dtype, int64_t m, int64_t ldx,
                      void* const* outs, const int64_t* ldo, int out_dtype, cudaStream_t st);

// Tensor-core dequant-GEMM for M > 16 over EPQ_LAYOUT_MMA16 / EPQ_LAYOUT_TILED stores (k_gemm_tc.cu).
bool tc_eligible(const StoreD& s, int64_t m, int x_dtype);
int launch_linear_tc(const StoreD* s, int count, const void* x, int x_dtype, int64_t m, int64_t ldx,
                     void* const* outs, const int64_t* ldo, int out_dtype, cudaStream_t st);
int tc_read_device_error(int* flag);

// Tensor-core compressed-state backward: dscale / dcb from dY^T X tiles (k_bwd_tc.cu).
bool bwd_tc_eligible(const StoreD& s, int64_t m, int act_dtype, const void* x, int64_t ldx,
                     const void* dy, int64_t ldy);
int launch_bwd_dw_tc(const StoreD& s, const void* x, int64_t ldx, const void* dy, int64_t ldy,
                     int act_dtype, int64_t m, float* dscale, float* dcb, cudaStream_t st);
int bwd_tc_read_device_error(int* flag);
// Tensor-core dX = dY W with W decoded along its rows (k_bwd_dx_tc.cu).
bool dx_tc_eligible(const StoreD& s, int64_t m, int act_dtype, const void* dy, int64_t ldy);
int launch_bwd_dx_tc(const StoreD& s, const void* dy, int64_t ldy, int act_dtype, int64_t m, void* dx,
                     int64_t lddx, int dx_dtype, cudaStream_t st);
int dx_tc_read_device_error(int* flag);

// Batch-1 LUT kernel over up to 4 stores sharing x.
constexpr int kLutMaxStores = 4;
bool lut_eligible(const StoreD& s);
bool lut_counters_fit(const StoreD* s, int count);
int64_t lut_workspace_bytes(const StoreD* s, int count);
int launch_linear_lut(const StoreD* s, int count, const void* x, int x_dtype, void* const* outs,
                      int out_dtype, void* ws, int64_t ws_bytes, cudaStream_t st);
int64_t lut_static_scratch_bytes();
int launch_linear_lut_static(const StoreD* s, int count, const void* x, int x_dtype,
                             void* const* outs, int out_dtype, cudaStream_t st);

}  // namespace epq
