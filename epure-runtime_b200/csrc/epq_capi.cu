// The C ABI of libepq.so: argument validation, dispatch to the kernels, and
// error reporting.  Declarations and the reference interfaces each entry
// point replaces are in include/epq.h.
#include <stdarg.h>
#include <stdio.h>

#include <mutex>
#include <set>
#include <tuple>

#include "epq_common.cuh"

namespace epq {

namespace {
std::mutex g_attr_mutex;
std::set<std::tuple<const void*, int, int>> g_attr_done;   // (kernel, device, bytes)
int g_dev_sms[64] = {0};
}  // namespace

int set_smem_limit(const void* fn, int bytes, const char* who) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return check_launch(who);
    std::lock_guard<std::mutex> lock(g_attr_mutex);
    const auto key = std::make_tuple(fn, dev, bytes);
    if (g_attr_done.count(key)) return EPQ_OK;
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
        return check_launch(who);
    g_attr_done.insert(key);
    return EPQ_OK;
}

int device_sms() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(g_attr_mutex);
    if (g_dev_sms[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        g_dev_sms[dev] = v;
    }
    return g_dev_sms[dev];
}

static thread_local char g_err[512] = "";

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

int check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return set_error(EPQ_ELAUNCH, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
    return EPQ_OK;
}

int make_store(const epq_store* in, StoreD* s, const char* who) {
    if (!in) return set_error(EPQ_EINVAL, "%s: store is NULL", who);
    if (in->n < 0 || in->k < 0) return set_error(EPQ_EINVAL, "%s: negative shape", who);
    if (in->vec != 1 && in->vec != 4)
        return set_error(EPQ_EUNSUPPORTED, "%s: vec=%d (1 or 4 supported)", who, in->vec);
    if (in->bits != 4 && in->bits != 8)
        return set_error(EPQ_EUNSUPPORTED, "%s: bits=%d (4 or 8 supported)", who, in->bits);
    if (in->bits == 4 && in->vec != 1)
        return set_error(EPQ_EUNSUPPORTED, "%s: 4-bit indices need vec=1", who);
    const int max_levels = in->bits == 4 ? 16 : 256;
    if (in->levels <= 0 || in->levels > max_levels)
        return set_error(EPQ_EINVAL, "%s: levels=%d outside 1..%d for %d-bit indices", who,
                         in->levels, max_levels, in->bits);
    if (in->group <= 0) return set_error(EPQ_EINVAL, "%s: group=%d", who, in->group);
    if (in->vec == 4 && (in->k % 4) != 0)
        return set_error(EPQ_ESHAPE, "%s: k=%lld not a multiple of vec=4", who, (long long)in->k);
    if (in->group % in->vec != 0)
        return set_error(EPQ_ESHAPE, "%s: group=%d not a multiple of vec=%d", who, in->group, in->vec);
    if (!dtype_ok(in->cb_dtype) || !dtype_ok(in->scale_dtype))
        return set_error(EPQ_EDTYPE, "%s: cb/scale dtype must be f32, f16 or bf16", who);
    if (in->layout != EPQ_LAYOUT_ROWS && in->layout != EPQ_LAYOUT_TILED &&
        in->layout != EPQ_LAYOUT_MMA16)
        return set_error(EPQ_EINVAL, "%s: layout=%d", who, in->layout);
    if (in->layout != EPQ_LAYOUT_ROWS && in->bits != 8)
        return set_error(EPQ_ELAYOUT, "%s: tiled layouts hold 8-bit indices only", who);
    if (in->layout == EPQ_LAYOUT_MMA16 && in->group / in->vec != 32)
        return set_error(EPQ_ELAYOUT, "%s: EPQ_LAYOUT_MMA16 needs group / vec = 32", who);
    if (in->n > 0 && in->k > 0 && (!in->idx || !in->cb || !in->scale))
        return set_error(EPQ_EINVAL, "%s: idx, cb and scale must be non-NULL", who);
    s->idx = in->idx;
    s->layout = in->layout;
    s->bits = in->bits;
    s->vec = in->vec;
    s->levels = in->levels;
    s->group = in->group;
    s->cb_dtype = in->cb_dtype;
    s->scale_dtype = in->scale_dtype;
    s->cb = in->cb;
    s->scale = in->scale;
    s->s_n = in->scale_stride_n;
    s->s_g = in->scale_stride_g;
    s->n = in->n;
    s->k = in->k;
    s->ng = cdiv(in->k, in->group);
    s->rb = cdiv(in->n, 16);
    s->p = in->group / in->vec;
    s->kpos = in->k / in->vec;
    return EPQ_OK;
}

int lut_read_device_error(int* flag);
int mma_read_device_error(int* flag);
int chain_read_device_error(int* flag);
int glue_read_device_error(int* flag);

static bool x_ok(const void* x, int64_t m, int64_t k, int64_t ldx) {
    return (m == 0 || k == 0) || (x != nullptr && ldx >= k);
}

}  // namespace epq

using namespace epq;

extern "C" {

int epq_abi_version(void) { return EPQ_ABI_VERSION; }

const char* epq_last_error(void) { return g_err; }

int epq_device_error(int* flag) {
    if (!flag) return set_error(EPQ_EINVAL, "epq_device_error: flag is NULL");
    int lut = 0, mma = 0, chain = 0, tc = 0, bwd = 0;
    int rc = lut_read_device_error(&lut);
    if (rc) return rc;
    rc = mma_read_device_error(&mma);
    if (rc) return rc;
    rc = tc_read_device_error(&tc);
    if (rc) return rc;
    rc = bwd_tc_read_device_error(&bwd);
    if (rc) return rc;
    int dxe = 0;
    rc = dx_tc_read_device_error(&dxe);
    if (rc) return rc;
    bwd = bwd || dxe;
    rc = chain_read_device_error(&chain);
    if (rc) return rc;
    int emb = 0;
    rc = embed_read_device_error(&emb);
    if (rc) return rc;
    int glue = 0;
    rc = glue_read_device_error(&glue);
    if (rc) return rc;
    // bit 0: LUT placement check; bit 1: a bounded wait gave up (GEMV, GEMM, backward or chain);
    // bit 2: the chain kernel's placement or grid check failed; bit 3: an embedding id was
    // outside the store's rows; bit 4: a decode position was at or past the KV cache's capacity
    *flag = (lut ? 1 : 0) | (((mma & 1) || tc || bwd || chain == 1) ? 2 : 0) | (chain == 2 ? 4 : 0) |
            (emb ? 8 : 0) | ((glue || (mma & 2)) ? 16 : 0);
    return EPQ_OK;
}

int64_t epq_layout_bytes(int32_t layout, int64_t n, int64_t k, int32_t vec, int32_t group) {
    if (n < 0 || k < 0 || (vec != 1 && vec != 4) || group <= 0 || group % vec || k % vec) return -1;
    if (layout == EPQ_LAYOUT_MMA16 && group / vec != 32) return -1;
    if (layout != EPQ_LAYOUT_TILED && layout != EPQ_LAYOUT_MMA16) return -1;
    return layout_bytes(layout, n, k, vec, group);
}

int epq_relayout(const uint8_t* src_rows, int32_t layout, int64_t n, int64_t k, int32_t vec,
                 int32_t group, uint8_t* dst, void* stream) {
    if (n < 0 || k < 0) return set_error(EPQ_EINVAL, "relayout: negative shape");
    if (vec != 1 && vec != 4) return set_error(EPQ_EUNSUPPORTED, "relayout: vec=%d", vec);
    if (group <= 0 || group % vec) return set_error(EPQ_ESHAPE, "relayout: group=%d vec=%d", group, vec);
    if (k % vec) return set_error(EPQ_ESHAPE, "relayout: k=%lld not a multiple of vec", (long long)k);
    if (layout != EPQ_LAYOUT_TILED && layout != EPQ_LAYOUT_MMA16)
        return set_error(EPQ_ELAYOUT, "relayout: target layout %d", layout);
    if (layout == EPQ_LAYOUT_MMA16 && group / vec != 32)
        return set_error(EPQ_ESHAPE, "relayout: EPQ_LAYOUT_MMA16 needs group / vec = 32");
    if (n * k == 0) return EPQ_OK;
    if (!src_rows || !dst) return set_error(EPQ_EINVAL, "relayout: NULL buffer");
    if (reinterpret_cast<uintptr_t>(dst) & 15)
        return set_error(EPQ_EALIGN, "relayout: destination must be 16-byte aligned");
    return launch_relayout(src_rows, layout, n, k, vec, group, dst, static_cast<cudaStream_t>(stream));
}

int epq_linear_workspace_bytes(const epq_store* stores, int32_t count, int64_t m, int64_t* bytes) {
    if (!bytes) return set_error(EPQ_EINVAL, "workspace_bytes: bytes is NULL");
    *bytes = 0;
    if (count < 1 || count > kLutMaxStores || !stores)
        return set_error(EPQ_EINVAL, "workspace_bytes: count=%d (1..%d)", count, kLutMaxStores);
    StoreD s[kLutMaxStores];
    bool all_lut = (m == 1);
    for (int i = 0; i < count; ++i) {
        int rc = make_store(&stores[i], &s[i], "workspace_bytes");
        if (rc) return rc;
        all_lut = all_lut && lut_eligible(s[i]);
    }
    all_lut = all_lut && lut_counters_fit(s, count);
    *bytes = all_lut ? lut_workspace_bytes(s, count) : 0;
    return EPQ_OK;
}

int epq_linear_multi(const epq_store* stores, int32_t count, const void* x, int32_t x_dtype,
                     int64_t m, int64_t ldx, void* const* outs, const int64_t* ldo,
                     int32_t out_dtype, void* workspace, int64_t workspace_bytes, void* stream) {
    if (count < 1 || count > kLutMaxStores || !stores || !outs)
        return set_error(EPQ_EINVAL, "linear: count=%d (1..%d) / NULL arrays", count, kLutMaxStores);
    if (m < 0) return set_error(EPQ_EINVAL, "linear: m=%lld", (long long)m);
    if (!dtype_ok(x_dtype) || !dtype_ok(out_dtype))
        return set_error(EPQ_EDTYPE, "linear: x/out dtype must be f32, f16 or bf16");
    StoreD s[kLutMaxStores];
    bool all_lut = (m == 1);
    for (int i = 0; i < count; ++i) {
        int rc = make_store(&stores[i], &s[i], "linear");
        if (rc) return rc;
        if (s[i].k != s[0].k)
            return set_error(EPQ_ESHAPE, "linear: stores sharing x must have equal k");
        if (m > 0 && s[i].n > 0 && !outs[i]) return set_error(EPQ_EINVAL, "linear: out[%d] is NULL", i);
        if (ldo && ldo[i] < s[i].n) return set_error(EPQ_ESHAPE, "linear: ldo[%d] < n", i);
        all_lut = all_lut && lut_eligible(s[i]);
    }
    all_lut = all_lut && lut_counters_fit(s, count);
    if (!x_ok(x, m, s[0].k, ldx)) return set_error(EPQ_EINVAL, "linear: x is NULL or ldx < k");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    bool all_mma = true;
    for (int i = 0; i < count; ++i) all_mma = all_mma && mma_eligible(s[i], m, x_dtype);
    if (all_mma) return launch_linear_mma(s, count, x, x_dtype, m, ldx, outs, ldo, out_dtype, st);
    bool all_tc = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && ldx % 8 == 0;
    for (int i = 0; i < count; ++i)
        all_tc = all_tc && tc_eligible(s[i], m, x_dtype) && s[i].layout == s[0].layout;
    if (all_tc) return launch_linear_tc(s, count, x, x_dtype, m, ldx, outs, ldo, out_dtype, st);
    if (all_lut) {
        if (reinterpret_cast<uintptr_t>(x) % dtype_size(x_dtype))
            return set_error(EPQ_EALIGN, "linear: x misaligned");
        return launch_linear_lut(s, count, x, x_dtype, outs, out_dtype, workspace, workspace_bytes, st);
    }
    for (int i = 0; i < count; ++i) {
        int rc = launch_linear_generic(s[i], x, x_dtype, m, ldx, outs[i], ldo ? ldo[i] : s[i].n,
                                       out_dtype, st);
        if (rc) return rc;
    }
    return EPQ_OK;
}

int epq_linear(const epq_store* store, const void* x, int32_t x_dtype, int64_t m, int64_t ldx,
               void* out, int64_t ldo, int32_t out_dtype, void* workspace, int64_t workspace_bytes,
               void* stream) {
    void* outs[1] = {out};
    int64_t ldos[1] = {ldo};
    return epq_linear_multi(store, 1, x, x_dtype, m, ldx, outs, ldos, out_dtype, workspace,
                            workspace_bytes, stream);
}

int epq_linear_noalloc(const epq_store* stores, int32_t count, const void* x, int32_t x_dtype,
                       void* const* outs, int32_t out_dtype, void* stream) {
    if (count < 1 || count > kLutMaxStores || !stores || !outs)
        return set_error(EPQ_EINVAL, "linear_noalloc: count=%d (1..%d) / NULL arrays", count,
                         kLutMaxStores);
    if (!dtype_ok(x_dtype) || !dtype_ok(out_dtype))
        return set_error(EPQ_EDTYPE, "linear_noalloc: x/out dtype must be f32, f16 or bf16");
    StoreD s[kLutMaxStores];
    for (int i = 0; i < count; ++i) {
        int rc = make_store(&stores[i], &s[i], "linear_noalloc");
        if (rc) return rc;
        if (s[i].k != s[0].k)
            return set_error(EPQ_ESHAPE, "linear_noalloc: stores sharing x must have equal k");
        if (!lut_eligible(s[i]))
            return set_error(EPQ_EUNSUPPORTED, "linear_noalloc: store %d is not an EPQ_LAYOUT_TILED "
                             "vector store (vec 4, 8-bit, group 128)", i);
        if (!outs[i]) return set_error(EPQ_EINVAL, "linear_noalloc: out[%d] is NULL", i);
    }
    if (!lut_counters_fit(s, count))
        return set_error(EPQ_EUNSUPPORTED, "linear_noalloc: too many row blocks");
    if (!x || reinterpret_cast<uintptr_t>(x) % dtype_size(x_dtype))
        return set_error(EPQ_EINVAL, "linear_noalloc: x is NULL or misaligned");
    return launch_linear_lut_static(s, count, x, x_dtype, outs, out_dtype,
                                    static_cast<cudaStream_t>(stream));
}

int64_t epq_linear_noalloc_max_scratch(void) { return lut_static_scratch_bytes(); }

int epq_linear_bwd(const epq_store* store, const void* x, int64_t ldx, const void* dy, int64_t ldy,
                   int32_t act_dtype, int64_t m, void* dx, int64_t lddx, int32_t dx_dtype,
                   float* dscale, float* dcb, void* stream) {
    StoreD s;
    int rc = make_store(store, &s, "linear_bwd");
    if (rc) return rc;
    if (m < 0) return set_error(EPQ_EINVAL, "linear_bwd: m=%lld", (long long)m);
    if (!dtype_ok(act_dtype) || (dx && !dtype_ok(dx_dtype)))
        return set_error(EPQ_EDTYPE, "linear_bwd: activation dtypes must be f32, f16 or bf16");
    if (m > 0 && s.n > 0 && (!dy || ldy < s.n)) return set_error(EPQ_EINVAL, "linear_bwd: dy/ldy");
    if ((dscale || dcb) && !x_ok(x, m, s.k, ldx)) return set_error(EPQ_EINVAL, "linear_bwd: x/ldx");
    if (dx && lddx < s.k) return set_error(EPQ_ESHAPE, "linear_bwd: lddx < k");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // dX: tensor cores (W decoded along its rows into TMEM) where eligible
    if (dx && m > 0 && s.k > 0 && dx_tc_eligible(s, m, act_dtype, dy, ldy)) {
        rc = launch_bwd_dx_tc(s, dy, ldy, act_dtype, m, dx, lddx, dx_dtype, st);
        if (rc) return rc;
        dx = nullptr;
    }
    if ((dscale || dcb) && s.n > 0 && bwd_tc_eligible(s, m, act_dtype, x, ldx, dy, ldy)) {
        // dscale / dcb on the tensor cores (dW never stored)
        if (dcb && cudaMemsetAsync(dcb, 0, sizeof(float) * s.levels * s.vec, st) != cudaSuccess)
            return check_launch("memset dcb");
        rc = launch_bwd_dw_tc(s, x, ldx, dy, ldy, act_dtype, m, dscale, dcb, st);
        if (rc) return rc;
        dscale = nullptr;
        dcb = nullptr;
    }
    if (!dx && !dscale && !dcb) return EPQ_OK;
    return launch_bwd_generic(s, x, ldx, dy, ldy, act_dtype, m, dx, lddx, dx_dtype, dscale, dcb, st);
}

int epq_embedding(const epq_store* store, const int64_t* ids, int64_t n_ids, void* out, int64_t ldo,
                  int32_t out_dtype, void* stream) {
    StoreD s;
    int rc = make_store(store, &s, "embedding");
    if (rc) return rc;
    if (!dtype_ok(out_dtype)) return set_error(EPQ_EDTYPE, "embedding: out dtype");
    if (n_ids < 0) return set_error(EPQ_EINVAL, "embedding: n_ids < 0");
    if (n_ids * s.k > 0 && (!ids || !out || ldo < s.k)) return set_error(EPQ_EINVAL, "embedding: ids/out/ldo");
    return launch_embedding(s, ids, n_ids, out, ldo, out_dtype, static_cast<cudaStream_t>(stream));
}

int epq_materialize(const epq_store* store, void* w, int64_t ldw, int32_t out_dtype, void* stream) {
    StoreD s;
    int rc = make_store(store, &s, "materialize");
    if (rc) return rc;
    if (!dtype_ok(out_dtype)) return set_error(EPQ_EDTYPE, "materialize: out dtype");
    if (s.n * s.k > 0 && (!w || ldw < s.k)) return set_error(EPQ_EINVAL, "materialize: w/ldw");
    return launch_materialize(s, w, ldw, out_dtype, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
