/*
 * epq.h -- C ABI of the B200 fused codebook dequant-matmul library (libepq.so).
 *
 * A packed weight ("store") is W[n, k] = cb[idx(n, k)] * scale[n, k / group]:
 *   idx    uint8 codebook indices; one index per `vec` consecutive weights
 *          along k (vec = 1: the reference's scalar codebook; vec = 4: a
 *          4-weight vector codebook).  bits = 4 packs two scalar indices per
 *          byte (even k in the low nibble), bits = 8 is one index per byte.
 *   cb     `levels` entries of `vec` values (f32, f16 or bf16).
 *   scale  one value per output row per group of `group` weights along k
 *          (f16, f32 or bf16), addressed as scale[n * scale_stride_n +
 *          g * scale_stride_g] (element strides).
 *
 * Everything here takes plain device pointers and sizes.  Nothing allocates
 * or frees memory: callers pass output buffers and, where a kernel needs
 * scratch, a workspace sized by the matching *_workspace_bytes query.  Every
 * call is asynchronous on the given stream (a cudaStream_t passed as void*;
 * NULL is the legacy default stream) and returns EPQ_OK or a negative
 * epq_status; epq_last_error() then describes the failure.  The calls are
 * safe to capture in a CUDA graph.
 *
 * Reference interfaces replaced (epure-runtime v0.2.4, paths in that project):
 *   epq_linear / epq_linear_multi
 *       epure/kernels/_triton.py:477  dequant_matmul(x, packed, scale, cb,
 *                                     group, bits, n_out, k_in)  (GPU)
 *       kernel/src/lib.rs:96          dequant_matmul(x, packed, scales, cb,
 *                                     group, four_bit)            (CPU)
 *       epure/kernels/cuda.py:88      linear(x, store)  -- the backend
 *                                     contract; the ABI never declines, it
 *                                     returns an error instead
 *   epq_linear_bwd
 *       the autograd of epure/runtime.py:78-89 (materialize) + F.linear used
 *       by epure/finetune.py:49-102 (make_trainable) -- the reference has no
 *       backward kernel
 *   epq_materialize
 *       epure/runtime.py:78-89        PackedWeight.materialize(dtype)
 *   epq_embedding
 *       epure/runtime.py:129-160      PackedEmbedding.forward(ids)
 *   epq_relayout / epq_layout_bytes
 *       the re-layout step of epure/runtime.py:243-249 (apply_to builds the
 *       store from the container's index stream)
 */
#ifndef EPQ_H
#define EPQ_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EPQ_ABI_VERSION 1

/* Status codes.  0 is success; every failure is negative. */
enum epq_status {
    EPQ_OK = 0,
    EPQ_EINVAL = -1,        /* null pointer, negative size, bad enum value   */
    EPQ_ESHAPE = -2,        /* sizes inconsistent with each other            */
    EPQ_EDTYPE = -3,        /* dtype not supported for this argument         */
    EPQ_EALIGN = -4,        /* pointer or stride alignment not met           */
    EPQ_ELAYOUT = -5,       /* index layout not supported for this call      */
    EPQ_EWORKSPACE = -6,    /* workspace missing or smaller than required    */
    EPQ_ELAUNCH = -7,       /* the CUDA launch failed                        */
    EPQ_EUNSUPPORTED = -8,  /* combination of parameters not implemented     */
    EPQ_ETIMEOUT = -9       /* a bounded device-side wait gave up            */
};

/* Element types. */
enum epq_dtype { EPQ_F32 = 0, EPQ_F16 = 1, EPQ_BF16 = 2 };

/* Index layouts.
 *   EPQ_LAYOUT_ROWS   the reference's layout: the flat stream of runtime.py
 *                     _pack4 over [n, k] (bits = 4: two per byte, even flat
 *                     position low nibble; bits = 8: one per byte), or for
 *                     vec = 4 one byte per vector, [n, k / 4] row-major.
 *   EPQ_LAYOUT_TILED  the kernel-native layout for bits = 8.  With
 *                     P = group / vec index positions per group, RB =
 *                     ceil(n / 16) row blocks and NG = ceil(k / group) groups,
 *                     the index of row r, position j lives at byte
 *                       ((g * RB + rb) * P + l) * 16 + rr,
 *                     g = j / P, l = j % P, rb = r / 16, rr = r % 16.  A
 *                     16-row x P-position tile is contiguous, tiles run
 *                     row-block fastest within a group.  Padding (rows >= n,
 *                     positions >= k / vec) holds index 0.
 *   EPQ_LAYOUT_MMA16  the small-batch tensor-core layout for bits = 8 with
 *                     group / vec = 32 positions per group.  With RB =
 *                     ceil(n / 16) and NG = ceil(k / group), the index of
 *                     row r, position j lives at byte
 *                       ((rb * NG + g) * 32 + t) * 16 + 8 * h + s,
 *                     g = j / 32, rb = r / 16, h = (r % 16) / 8,
 *                     t = 4 * (r % 8) + j % 4, s = (j % 32) / 4: a 512-byte
 *                     tile per (16-row block, group), group fastest, in which
 *                     each of 32 lanes reads one 16-byte word.  Padding holds
 *                     index 0.                                          */
enum epq_layout { EPQ_LAYOUT_ROWS = 0, EPQ_LAYOUT_TILED = 1, EPQ_LAYOUT_MMA16 = 2 };

/* A packed weight, described by plain pointers (all device memory). */
typedef struct epq_store {
    const uint8_t* idx;       /* packed indices, `layout`                      */
    int32_t layout;           /* enum epq_layout                               */
    int32_t bits;             /* 4 or 8                                        */
    int32_t vec;              /* weights per index: 1 or 4                     */
    int32_t levels;           /* codebook entries (<= 16 for bits = 4, <= 256) */
    int32_t group;            /* weights per scale along k (> 0)               */
    int32_t cb_dtype;         /* enum epq_dtype                                */
    const void* cb;           /* [levels * vec]                                */
    int32_t scale_dtype;      /* enum epq_dtype                                */
    int32_t reserved0;
    const void* scale;        /* [n, ceil(k / group)] with the strides below   */
    int64_t scale_stride_n;   /* element stride between rows                   */
    int64_t scale_stride_g;   /* element stride between groups                 */
    int64_t n;                /* output features (rows)                        */
    int64_t k;                /* input features                                */
} epq_store;

/* ABI version of the loaded library (EPQ_ABI_VERSION it was built with). */
int epq_abi_version(void);

/* Human-readable description of the last failure on the calling host thread. */
const char* epq_last_error(void);

/* Reads (synchronously, on the current device) the flags kernels set when an
 * in-kernel check fails: bit 0 -- the batch-1 LUT kernel found its shared
 * memory placement violated and wrote nothing; bit 1 -- a bounded
 * device-side wait gave up (that call's output is invalid); bit 2 -- the
 * chain kernel's placement or grid check failed; bit 3 -- epq_embedding was
 * given an id outside the store's rows (that row of its output is zero); bit
 * 4 -- a decode-glue call (include/epq_decode.h) got a position outside its
 * KV cache (nothing was written to the cache).
 * *flag = 0 means no kernel has reported a failure. */
int epq_device_error(int* flag);

/* Bytes of an index buffer in `layout` (EPQ_LAYOUT_TILED or EPQ_LAYOUT_MMA16)
 * for the given shape, or -1 for an unsupported combination. */
int64_t epq_layout_bytes(int32_t layout, int64_t n, int64_t k, int32_t vec, int32_t group);

/* Re-lay an EPQ_LAYOUT_ROWS index buffer (bits = 8, [n, k / vec] row-major)
 * into `layout`.  `dst` must hold epq_layout_bytes(...) bytes and be 16-byte
 * aligned; padding is written as index 0. */
int epq_relayout(const uint8_t* src_rows, int32_t layout, int64_t n, int64_t k, int32_t vec,
                 int32_t group, uint8_t* dst, void* stream);

/* Scratch needed by epq_linear_multi for these stores at `m` activation rows
 * (0 when the call needs none).  The first 64 KiB of a workspace hold
 * completion counters and the rest partial sums.  Zero-fill a workspace once
 * after allocating it; every call leaves the counters zero again when it
 * completes, so one workspace serves any later call that is ordered after it
 * (same stream, or a dependency), whatever its shapes.  Calls that overlap on
 * the GPU need separate workspaces. */
int epq_linear_workspace_bytes(const epq_store* stores, int32_t count, int64_t m,
                               int64_t* bytes);

/* out[i][m, n_i] = x[m, k] @ W_i[n_i, k]^T for `count` (1..4) stores that share
 * the activation x (same k).  x: [m, k] with row stride ldx (elements),
 * x_dtype f32/f16/bf16; outs[i]: [m, n_i] with row stride ldo[i], out_dtype
 * f32/f16/bf16.  fp32 accumulation.  Calls with 1 <= m <= 16 bf16/f16
 * activations on EPQ_LAYOUT_MMA16 vector stores run the tensor-core GEMV (no
 * workspace; it may overlap the previous kernel on the stream through
 * programmatic dependent launch).  Batch-1 calls on EPQ_LAYOUT_TILED vector
 * stores run the LUT kernel and need the workspace above.  Every other
 * combination runs the general kernel. */
int epq_linear_multi(const epq_store* stores, int32_t count, const void* x,
                     int32_t x_dtype, int64_t m, int64_t ldx, void* const* outs,
                     const int64_t* ldo, int32_t out_dtype, void* workspace,
                     int64_t workspace_bytes, void* stream);

/* Single-store form of epq_linear_multi. */
int epq_linear(const epq_store* store, const void* x, int32_t x_dtype, int64_t m,
               int64_t ldx, void* out, int64_t ldo, int32_t out_dtype, void* workspace,
               int64_t workspace_bytes, void* stream);

/* Batch-1 linear that allocates nothing and takes no workspace: for callers
 * that cannot call cudaMalloc when they run the op (a plugin inside a serving
 * engine that owns all device memory, a loop where an allocation could block
 * or fail).  No counterpart in the reference.
 *   Same math and arguments as epq_linear_multi with m = 1 (x: k values,
 *   outs[i]: n_i values), for EPQ_LAYOUT_TILED vector stores (vec 4, 8-bit,
 *   group 128) only.  Its scratch is a file-scope device array of
 *   epq_linear_noalloc_max_scratch() bytes (4 MiB) that every GPU loading the
 *   library holds until exit; stores needing more are rejected with
 *   EPQ_EWORKSPACE.  The first call on a device resolves the array's address
 *   with that device current -- make that call before any stream capture.
 *   All calls share the array (the counters are cleared on the stream at each
 *   call), so calls that overlap on the GPU race: order them on one stream. */
int epq_linear_noalloc(const epq_store* stores, int32_t count, const void* x, int32_t x_dtype,
                       void* const* outs, int32_t out_dtype, void* stream);

/* Bytes of the static scratch behind epq_linear_noalloc. */
int64_t epq_linear_noalloc_max_scratch(void);

/* Backward of out = x @ W^T with the indices frozen.
 *   dy [m, n] (ldy), x [m, k] (ldx): same dtype, f32/f16/bf16.
 *   dx [m, k] (lddx, dx_dtype) = dy @ W        (skipped when dx is NULL)
 *   dscale [n, ceil(k / group)] f32, dense row-major:
 *       dscale[r, g] = sum_{k in g} dW[r, k] * cb[idx(r, k)]
 *   dcb [levels * vec] f32:
 *       dcb[e * vec + p] = sum over weights with index e, sub-position p of
 *                          dW[r, k] * scale[r, k / group]
 *   with dW = dy^T x never stored.  dscale / dcb are overwritten (skipped
 *   when NULL).  They are reduced with float atomics, so their last bits can
 *   vary from run to run. */
int epq_linear_bwd(const epq_store* store, const void* x, int64_t ldx, const void* dy,
                   int64_t ldy, int32_t act_dtype, int64_t m, void* dx, int64_t lddx,
                   int32_t dx_dtype, float* dscale, float* dcb, void* stream);

/* A chain of batch-1 linears run as ONE persistent kernel: step j multiplies
 * its input vector by each of its stores; the output of store `feed` of step j
 * is the input of step j + 1; the output of store `feed` of the last step is
 * written to `out`.  Replaces a sequence of PackedLinear.forward calls
 * (epure/runtime.py:98-126, each the Triton kernel of kernels/_triton.py:56-107)
 * such as one decode token through a decoder's packed linears.
 * Stores must be EPQ_LAYOUT_TILED vector stores (vec 4, 8-bit, group 128) with
 * group-major f16/f32 scales whose row stride is padded to a multiple of 16
 * (scale_stride_n = 1, scale_stride_g % 16 == 0, >= 16 * ceil(n / 16)) and
 * 16-byte aligned buffers; the stores of a step share k; the feed output width
 * equals the next step's k.  Intermediate outputs are not written. */
typedef struct epq_chain_step {
    epq_store stores[4];
    int32_t count;    /* 1..4 stores sharing the step's input                      */
    int32_t feed;     /* index of the store whose output feeds the next step / out */
} epq_chain_step;

/* Workspace bytes for a chain (descriptors, counters, two partial-sum buffers). */
int epq_chain_workspace_bytes(const epq_chain_step* steps, int32_t n_steps, int64_t* bytes);

/* Writes the chain's descriptors into the workspace (256-byte aligned) and zeroes
 * its counters.  Synchronous; call once per chain, on the device it will run on. */
int epq_chain_prepare(const epq_chain_step* steps, int32_t n_steps, void* workspace,
                      int64_t workspace_bytes, void* stream);

/* Tensor parallelism inside the chain (no reference counterpart: the
 * reference has no multi-GPU path; it replaces, for a sharded model, the
 * per-linear launches + NCCL all-reduce after every row-parallel linear).
 * Each of `world` ranks (one GPU each, one process each) prepares a chain over
 * its shards with identical shapes, maps every rank's workspace into its
 * address space (CUDA IPC), and calls this once: peer_workspaces[r] is rank
 * r's workspace as mapped here (peer_workspaces[rank] == workspace).
 * remote_input[j] = 1 marks step j whose input is the output of a
 * row-parallel step (a sum over ranks); remote_input[n_steps] marks the final
 * output likewise.  Inside the kernel each rank publishes its sum of every
 * input slice it stages and adds the other ranks' over NVLink (plain peer
 * loads of tagged values, bounded polling) -- no collective launch, no
 * barrier.  All ranks must run their chains concurrently (one run per token
 * each).  Synchronous. */
int epq_chain_set_tp(void* workspace, int32_t rank, int32_t world, const void* const* peer_workspaces,
                     const uint8_t* remote_input, int32_t n_flags, void* stream);

/* Runs a prepared chain on x (k0 values) into out.  One cooperative launch;
 * capturable in a CUDA graph.  Runs on one workspace must be ordered (same
 * stream); each run leaves the workspace ready for the next. */
int epq_chain_run(const void* workspace, const void* x, int32_t x_dtype, void* out,
                  int32_t out_dtype, void* stream);

/* Dense W [n, k] (row stride ldw) in out_dtype with PackedWeight.materialize's
 * rounding: cb and scale are first rounded to out_dtype, their product is
 * rounded to out_dtype (runtime.py:85-88). */
int epq_materialize(const epq_store* store, void* w, int64_t ldw, int32_t out_dtype,
                    void* stream);

/* Rows of the dequantised table for a packed embedding: out[i, :] (row stride
 * ldo >= k, out_dtype) = W[ids[i], :] with materialize's rounding, for n_ids
 * device-resident int64 ids; only those rows are decoded.  Replaces
 * PackedEmbedding.forward (runtime.py:129-160: gather cb[idx] for the ids'
 * rows, cast, multiply by the rows' scales).  Any store format.  A negative
 * id counts from the end (id + n), as torch indexing does; an id outside
 * [-n, n) gives a zero row and sets bit 3 of epq_device_error (the reference's
 * indexing raises there -- set EPURE_CHECK_IDS=1 for the same on the host). */
int epq_embedding(const epq_store* store, const int64_t* ids, int64_t n_ids, void* out, int64_t ldo,
                  int32_t out_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* EPQ_H */
