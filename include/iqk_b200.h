/*
 * iqk_b200: C ABI of the B200-native IQ_K routed-expert hot path.
 *
 * One shared library (mlx_iqk_b200/libiqk_b200.so, built for sm_100a)
 * exports the entry points below. They take plain device pointers, sizes and
 * a CUDA stream, return an int status, borrow every pointer and allocate
 * nothing: outputs and workspaces are the caller's.
 *
 * Streams are the reference's k-contiguous relayout, passed as an array of
 * device pointers in the reference's component order
 * (src/mlx_iqk/format.py:352-377):
 *
 *   IQK_IQ2_KS   {qs u32[E,o,n/16], scl u8[E,o,n/64], sch u8[E,o,n/256],
 *                 sex u8[E,o,n/256], dv f16[E,o]}
 *   IQK_IQ2_K    {qs u32[E,o,n/16], scl u8[E,o,n/32], sex u8[E,o,n/128],
 *                 dv f16[E,o,n/256]}
 *   IQK_IQ1_S_R4 {qs u32[E,o,n/32], qh u16[E,o,n/32], dv f16[E,o]}
 *
 * Every entry point is stream-ordered on the caller's stream. Library state
 * is a read-only constant table per device, plus one exception: the
 * writable static scratch array of iqk_gemv_static (one copy per CUDA
 * context). Every other entry point is reentrant; iqk_gemv_static calls that
 * are unordered with each other in one process's context on one device race
 * on that array.
 */
#ifndef IQK_B200_H
#define IQK_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t; NULL is the legacy default stream. */
typedef struct CUstream_st *iqk_stream_t;

/* Members (src/mlx_iqk/format.py:116 MEMBERS) and the dense members
 * (format.py:120 DENSE_MEMBERS), which only the iqk_dense_* entries take. */
enum {
    IQK_IQ2_KS = 0,
    IQK_IQ2_K = 1,
    IQK_IQ1_S_R4 = 2,
    IQK_IQ4_KS = 3,
    IQK_IQ4_K = 4,
    IQK_IQ5_K = 5,
    IQK_IQ6_K = 6
};

/* Element types of activations and outputs. */
enum {
    IQK_F32 = 0,
    IQK_F16 = 1,
    IQK_BF16 = 2
};

/* Status codes. The Python layer maps them onto the reference's exception
 * classes: IqkFormatError (MEMBER), IqkKernelError (WIDTH, GEOMETRY) and
 * IqkRuntimeError (the rest) -- src/mlx_iqk/format.py:265,
 * src/mlx_iqk/kernels.py:86, src/mlx_iqk/nn.py:97. */
enum {
    IQK_OK = 0,
    IQK_ERR_MEMBER = 1,      /* member not one an entry point takes */
    IQK_ERR_WIDTH = 2,       /* in_features not a sized width (2048, 4096; dense 1024-8192) */
    IQK_ERR_GEOMETRY = 3,    /* out_features / experts / row range / pairs */
    IQK_ERR_ARGUMENT = 4,    /* null pointer, bad dtype, negative count */
    IQK_ERR_ALIGNMENT = 5,   /* a pointer lacks the alignment a kernel needs */
    IQK_ERR_WORKSPACE = 6,   /* workspace missing or smaller than required */
    IQK_ERR_CUDA = 7,        /* a CUDA runtime call or launch failed */
    IQK_ERR_DEVICE = 8       /* current device is not compute capability 10.0 */
};

/* Bits of the device-side error word (iqk_read_error). */
enum {
    IQK_DEVERR_EXPERT = 1,   /* an expert index was outside [0, num_experts) */
    IQK_DEVERR_TOKEN = 2,    /* a pair's activation row was outside [0, x_rows) */
    IQK_DEVERR_NONFINITE = 4, /* an activation row held a NaN or infinity */
    IQK_DEVERR_TIMEOUT = 8    /* a kernel's bounded wait on its copy pipeline expired */
};

/* Short description of a status code (static storage). */
const char *iqk_status_string(int status);

/* ABI version of this header: 1. */
int iqk_abi_version(void);

/* IQK_OK when the current device is compute capability 10.0 (sm_100a). */
int iqk_check_device(void);

/*
 * Failure-detection check of the kernels' bounded waits: one warp waits on a
 * shared-memory mbarrier that nothing arrives on, with the same bounded-wait
 * code the decode kernels use and a limit of limit_ns (at most 2 s), then
 * ORs IQK_DEVERR_TIMEOUT into the device word *flags (caller-owned, zeroed
 * by the caller). The kernel returns normally, so the context stays usable.
 * No reference counterpart: the reference's kernels have no bounded waits.
 */
int iqk_check_bounded_wait(int64_t limit_ns, int32_t *flags, iqk_stream_t stream);

/*
 * On-device relayout of ik wire rows into the streams above: wire is
 * [rows, ggml row bytes] (IQ2_KS 2 + 70*n/256, IQ2_K 76*n/256, IQ1_S_R4
 * 2 + 6*n/32 -- for IQ1_S_R4 rows is a multiple of 4, the wire's row groups);
 * streams[i] receives [rows, stream length] in component order, the same
 * bits as the reference's host relayout. in_features a multiple of 256.
 *
 * Replaces format.pack (src/mlx_iqk/format.py:612-678, the numpy relayout
 * the reference runs on the host before load_streams).
 */
int iqk_pack(int member, const void *wire, int64_t rows, int64_t in_features,
             void *const *streams, iqk_stream_t stream);

/*
 * Bit-exact stacked dequantization of out-rows [row_start, row_start + rows)
 * of every expert into dst[E, rows, in_features] (row-major), in float32,
 * float16 or bfloat16 (out_dtype). Every weight is the CPU dequantizer's
 * float32 chain -- d * float(index) then * value, or
 * d * float(2*ls + 1) then * (grid + shift) -- rounded to nearest-even once
 * when out_dtype is 16-bit.
 *
 * Replaces the reference's dequant_kernel / dequant_range_kernel
 * (src/mlx_iqk/kernels.py:631-742, launched at src/mlx_iqk/nn.py:155-201),
 * which emit float16 only and take a power-of-two range.
 */
int iqk_dequant(int member, const void *const *streams, int64_t num_experts,
                int64_t out_features, int64_t in_features, int64_t row_start,
                int64_t rows, int out_dtype, void *dst, iqk_stream_t stream);

/*
 * Address floor of iqk_dequant: the same loads and the same stores with the
 * decode deleted (the loaded words are folded into an integer, and that is
 * what is stored, so nothing can be dropped). Same arguments; dst receives
 * no weights. For the benchmark's "vs own floor" ratio only.
 *
 * Replaces the reference's dequant floor (bench/floors.py:186-220,
 * dequant_floor_source), which prices its dequantization the same way.
 */
int iqk_dequant_floor(int member, const void *const *streams, int64_t num_experts,
                      int64_t out_features, int64_t in_features, int64_t row_start,
                      int64_t rows, int out_dtype, void *dst, iqk_stream_t stream);

/*
 * Workspace bytes iqk_gemv needs for this member, width, activation-row
 * count and pair count (routing tables plus the prepared activations).
 * iqk_gemv_workspace_min_bytes is the smallest workspace the GEMV entries
 * accept (today the same figure). The run kernels keep their
 * work-distribution counters in the workspace header (CTAs claim items from
 * it, the last one done resets it; the prepare zeroes it), so runs over one
 * workspace must be ordered (one stream, or events): two projections that
 * share a preparation run one after the other, or each over its own
 * prepared workspace.
 */
size_t iqk_gemv_workspace_bytes(int member, int64_t in_features, int64_t x_rows,
                                int64_t pairs);
size_t iqk_gemv_workspace_min_bytes(int member, int64_t in_features, int64_t x_rows,
                                    int64_t pairs);

/*
 * Fused dequant + GEMV over token-expert pairs:
 *   y[p, r] = sum_k W[sel[p], r, k] * x[tok[p], k]
 * for p in [0, pairs), r in [0, out_features). x is [x_rows, in_features]
 * (x_dtype), y is [pairs, out_features] (y_dtype). When tok is NULL the pair's
 * activation row is p / (pairs / x_rows): top_k for the gate/up seam
 * ([..., 1, 1, in]) and 1 for the down seam ([..., top_k, 1, in]);
 * pairs % x_rows must then be 0. Pairs may arrive in any order; each expert's
 * weights are streamed once for all pairs that selected it. Pairs whose
 * expert or row index is out of range produce zeros and set the device error
 * word. The per-element result does not depend on the order or grouping of
 * pairs, so a sorted call is bit-identical to the unsorted one after
 * un-permuting. num_experts is at most 4096 (the routing tables live in
 * shared memory).
 *
 * Replaces gemv_kernel, gemv_sorted_kernel and gemv_union_kernel
 * (src/mlx_iqk/kernels.py:332-572, launched at src/mlx_iqk/nn.py:240-333).
 */
int iqk_gemv(int member, const void *x, int x_dtype, int64_t x_rows,
             const void *const *streams, int64_t num_experts, int64_t out_features,
             int64_t in_features, const int32_t *sel, const int32_t *tok,
             int64_t pairs, void *y, int y_dtype, void *workspace,
             size_t workspace_bytes, iqk_stream_t stream);

/*
 * The two halves of iqk_gemv, for callers that share one preparation between
 * several projections of the same activations and routing (a SwitchGLU's
 * gate and up) or schedule them apart.
 *
 * iqk_gemv_prepare: turns each activation row into the kernel's exact
 * integer operand form (power-of-two scale + three int8 digit planes) and
 * buckets the pairs by expert, all into `workspace` (iqk_gemv_workspace_bytes
 * for the same in_features / x_rows / pairs). Member-independent.
 *
 * iqk_gemv_run: streams the selected experts' rows of one projection and
 * writes y; reads only the prepared workspace (x and sel are not needed).
 * Must follow an iqk_gemv_prepare of the same workspace, on the same stream
 * or with an equivalent ordering.
 *
 * Together they replace the reference's single gemv launch
 * (src/mlx_iqk/nn.py:240-271); the split has no reference counterpart.
 */
int iqk_gemv_prepare(const void *x, int x_dtype, int64_t x_rows, int64_t in_features,
                     int64_t num_experts, const int32_t *sel, const int32_t *tok,
                     int64_t pairs, void *workspace, size_t workspace_bytes,
                     iqk_stream_t stream);

int iqk_gemv_run(int member, const void *const *streams, int64_t num_experts,
                 int64_t out_features, int64_t in_features, int64_t x_rows, int64_t pairs,
                 void *y, int y_dtype, const void *workspace, size_t workspace_bytes,
                 iqk_stream_t stream);

/*
 * Address floor of iqk_gemv_run: the same launch, the same copies from HBM
 * into shared memory and the same shared-memory reads of code words and
 * activation planes, with the decode deleted (the words are folded into an
 * integer that reaches y). Same arguments; y receives no projection. For the
 * benchmark's "vs own floor" ratio only.
 *
 * Replaces the reference's GEMV floor (bench/floors.py:60-183,
 * gemv_floor_source).
 */
int iqk_gemv_floor_run(int member, const void *const *streams, int64_t num_experts,
                       int64_t out_features, int64_t in_features, int64_t x_rows,
                       int64_t pairs, void *y, int y_dtype, const void *workspace,
                       size_t workspace_bytes, iqk_stream_t stream);

/*
 * A SwitchGLU's gate and up projections in one launch over a prepared
 * workspace (iqk_gemv_prepare of the layer input): for every routed pair p
 * and row r < out_features,
 *   h[p, r] = silu(gate_p[r]) * up_p[r] * weight[p]     (float32)
 * where gate_p / up_p are the two projections' decode GEMVs of the pair
 * (the same per-element values iqk_gemv_run gives) and weight is the pair's
 * router weight (NULL: 1). Both projections have member `member`; the down
 * projection is linear, so folding the router weight into h makes the
 * layer's output the plain sum over a token's pairs (iqk_pairs_combine).
 * out_features a multiple of 32. Each CTA item covers 32 rows of one pair
 * in both projections, so silu * up happens before anything leaves the SM.
 *
 * iqk_swiglu_rows: the same h from two finished float32 projections
 * [rows, cols] (for a layer whose gate and up members differ).
 *
 * Replaces the caller's seam around the reference's projections
 * (src/mlx_iqk/nn.py:1-22: gate and up IqkSwitchLinear on the token,
 * SiLU(gate) * up, down); the reference runs them as separate dispatches.
 */
int iqk_gemv_glu_run(int member, const void *const *gate_streams,
                     const void *const *up_streams, int64_t num_experts, int64_t out_features,
                     int64_t in_features, int64_t x_rows, int64_t pairs, const float *weight,
                     float *h, const void *workspace, size_t workspace_bytes,
                     iqk_stream_t stream);

int iqk_swiglu_rows(const float *gate, const float *up, const float *weight, int64_t rows,
                    int64_t cols, float *h, iqk_stream_t stream);

/*
 * Copy the device error bits of the last preparation in `workspace` (same
 * in_features / x_rows / pairs) into *flags (IQK_DEVERR_* bits),
 * synchronising the stream. No reference counterpart: the reference's
 * kernels read out-of-range indices unchecked.
 */
int iqk_read_error(const void *workspace, int64_t in_features, int64_t x_rows,
                   int64_t pairs, int32_t *flags, iqk_stream_t stream);

/*
 * Grouped per-expert GEMM for prefill-sized calls (many pairs per expert):
 *   y[p, r] = sum_k W[sel[p], r, k] * x[tok[p], k]
 * with the same argument meaning as iqk_gemv. Pairs are sorted by expert on
 * the device and each expert's weights are read once per tile of up to 128
 * of its pairs, dequantized into tensor memory and multiplied on the tensor
 * cores (f16 operands, f32 accumulation). Members IQK_IQ2_KS and IQK_IQ2_K;
 * out_features a multiple of 16; num_experts at most 4096. IQ2_KS weights
 * reach the tensor cores exactly (integer products, row scale in the
 * epilogue); IQ2_K weights carry two f16 roundings.
 *
 * Replaces the prefill route of IqkSwitchLinear.__call__: dequantized() then
 * mx.gather_mm(..., sorted_indices) (src/mlx_iqk/nn.py:221-238).
 *
 * iqk_grouped_workspace_bytes: workspace size (routing tables plus one f16
 * activation row per pair). iqk_grouped_prepare / iqk_grouped_run split the
 * call like iqk_gemv_prepare / iqk_gemv_run (the split has no reference
 * counterpart); the error word reads back with iqk_grouped_read_error.
 */
size_t iqk_grouped_workspace_bytes(int64_t in_features, int64_t num_experts, int64_t pairs);

int iqk_grouped_gemm(int member, const void *x, int x_dtype, int64_t x_rows,
                     const void *const *streams, int64_t num_experts, int64_t out_features,
                     int64_t in_features, const int32_t *sel, const int32_t *tok,
                     int64_t pairs, void *y, int y_dtype, void *workspace,
                     size_t workspace_bytes, iqk_stream_t stream);

int iqk_grouped_prepare(const void *x, int x_dtype, int64_t x_rows, int64_t in_features,
                        int64_t num_experts, const int32_t *sel, const int32_t *tok,
                        int64_t pairs, void *workspace, size_t workspace_bytes,
                        iqk_stream_t stream);

int iqk_grouped_run(int member, const void *const *streams, int64_t num_experts,
                    int64_t out_features, int64_t in_features, int64_t pairs, void *y,
                    int y_dtype, const void *workspace, size_t workspace_bytes,
                    iqk_stream_t stream);

int iqk_grouped_read_error(const void *workspace, int32_t *flags, iqk_stream_t stream);

/*
 * iqk_grouped_run restricted to output rows [row_start, row_start + rows) of
 * every expert: y is [pairs, rows]. Only those rows' weights are read and
 * multiplied, and each output element is the same dot product as in the
 * whole call, so range outputs concatenated along the feature axis equal
 * iqk_grouped_run's bit for bit.
 *
 * Replaces the reference's bounded-liveness range route,
 * IqkSwitchLinear.sorted_matmul_range (src/mlx_iqk/nn.py:203-217:
 * dequantized_range + gather_mm over one out-row slice).
 */
int iqk_grouped_run_range(int member, const void *const *streams, int64_t num_experts,
                          int64_t out_features, int64_t in_features, int64_t pairs,
                          int64_t row_start, int64_t rows, void *y, int y_dtype,
                          const void *workspace, size_t workspace_bytes, iqk_stream_t stream);

/*
 * Expert-parallel helpers (no reference counterpart: the reference serves a
 * whole layer on one device; these shard its SwitchGLU seam,
 * src/mlx_iqk/nn.py:1-22, over ranks that each hold num_experts local
 * experts and see every rank's pairs).
 *
 * iqk_grouped_prepare_shard: iqk_grouped_prepare, except that a pair whose
 * expert index lies outside [0, num_experts) belongs to another rank: it is
 * skipped without an error, and iqk_grouped_run leaves its output row
 * untouched (an out-of-range row index is still an error).
 *
 * iqk_pairs_swiglu: for every pair q routed by a prepared workspace (same
 * in_features, num_experts and pairs as the preparation),
 * h[q, :] = bf16((silu(gate[q, :]) * up[q, :]) * weight[q]); other rows of h
 * are not written. gate, up: float32 [pairs, inter]; h: bfloat16.
 *
 * iqk_pairs_combine: out[r, :] = sum over j < top_k, in order, of
 * y[r * top_k + j, :] for the slots whose sel lies in [0, num_experts); rows
 * without one are zeros. y: float32 [rows * top_k, hidden]; out: float32 or
 * bfloat16 [rows, hidden]; hidden a multiple of 4.
 */
int iqk_grouped_prepare_shard(const void *x, int x_dtype, int64_t x_rows, int64_t in_features,
                              int64_t num_experts, const int32_t *sel, const int32_t *tok,
                              int64_t pairs, void *workspace, size_t workspace_bytes,
                              iqk_stream_t stream);

int iqk_pairs_swiglu(const float *gate, const float *up, const float *weight, int64_t inter,
                     int64_t in_features, int64_t num_experts, int64_t pairs,
                     const void *workspace, size_t workspace_bytes, void *h,
                     iqk_stream_t stream);

int iqk_pairs_combine(const float *y, const int32_t *sel, int64_t rows, int top_k,
                      int64_t num_experts, int64_t hidden, void *out, int out_dtype,
                      iqk_stream_t stream);

/*
 * iqk_gemv without a workspace argument, for callers that cannot allocate
 * device memory where they launch (a runtime with a fixed memory plan, code
 * inside an allocator's own hooks, a binding without a device allocator).
 * No counterpart in the reference: its kernels get their buffers from MLX.
 *
 * Scratch is one static device array of iqk_gemv_static_max_bytes() (1 MiB)
 * per device; a call whose iqk_gemv_workspace_bytes exceeds it returns
 * IQK_ERR_WORKSPACE (1 MiB holds 64 activation rows with 512 pairs at
 * in_features 4096). Nothing is allocated and no byte of the scratch has to
 * start at zero. The first call on each device looks up the array's address
 * (cudaGetSymbolAddress, which may load the library's device code); make that
 * first call outside any stream capture. Each CUDA context that loads the
 * library holds its own copy of the array (so separate processes never share
 * one); the address is cached per device together with the context it was
 * resolved in and looked up again when another context is current. All calls
 * in one context on one device share the one array, so calls that overlap in
 * time there -- different streams or threads without an ordering between
 * them -- race on it; order them on one stream. Results equal iqk_gemv's.
 *
 * iqk_gemv_static_read_error: the device error bits (IQK_DEVERR_*) of the
 * last iqk_gemv_static call of this geometry in the current context, as
 * iqk_read_error gives them for a workspace; synchronises the stream.
 */
size_t iqk_gemv_static_max_bytes(void);

int iqk_gemv_static(int member, const void *x, int x_dtype, int64_t x_rows,
                    const void *const *streams, int64_t num_experts, int64_t out_features,
                    int64_t in_features, const int32_t *sel, const int32_t *tok,
                    int64_t pairs, void *y, int y_dtype, iqk_stream_t stream);

int iqk_gemv_static_read_error(int64_t in_features, int64_t x_rows, int64_t pairs,
                               int32_t *flags, iqk_stream_t stream);

/*
 * Dense members: one [out_features, in_features] matrix of IQ4_KS, IQ4_K,
 * IQ5_K or IQ6_K rows, streams in the reference's dense component order
 * (src/mlx_iqk/format.py:898-915):
 *
 *   IQK_IQ4_KS {qs u32[o,n/8], scl u8[o,n/32], dv f32[o]}
 *   IQK_IQ4_K  {qs u32[o,n/8], scl u8[o,n/32], sch u8[o,n/64], sex u8[o,n/128],
 *               dv f16[o,n/256]}
 *   IQK_IQ5_K  {qs u32[o,n/8], qh u32[o,n/32], scl u8[o,n/32], sch u8[o,n/64],
 *               sex u8[o,n/128], dv f16[o,n/256]}
 *   IQK_IQ6_K  {qs u32[o,n/8], qh u32[o,n/16], scl u8[o,n/16], sex u8[o,n/128],
 *               dv f16[o,n/256]}
 *
 * in_features is 1024, 2048, 4096 or 8192 (src/mlx_iqk/dense_kernels.py:56).
 * Every stream and the GEMV's x must be 16-byte aligned (IQK_ERR_ALIGNMENT).
 *
 * iqk_dense_dequant: rows [row_start, row_start + rows) into dst[rows, n] in
 * f32, f16 or bf16, bit for bit the reference decode rounded once
 * (src/mlx_iqk/dense.py:145-189, dense_dequantized / _range; the reference
 * stores fp16).
 *
 * iqk_dense_gemv: y[tokens, out] = x[tokens, n] W^T for f16 x (the
 * reference's call seam casts to fp16, src/mlx_iqk/dense.py:107-112), y in
 * f16 (the reference's output) or f32; out_features a multiple of 16
 * (src/mlx_iqk/dense_kernels.py:70-81). Replaces dense_gemv
 * (src/mlx_iqk/dense.py:116-142): each sub-block's scale is applied to its
 * own float32 partial sum.
 */
int iqk_dense_dequant(int member, const void *const *streams, int64_t out_features,
                      int64_t in_features, int64_t row_start, int64_t rows, int out_dtype,
                      void *dst, iqk_stream_t stream);
int iqk_dense_gemv(int member, const void *x, int64_t tokens, const void *const *streams,
                   int64_t out_features, int64_t in_features, void *y, int y_dtype,
                   iqk_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* IQK_B200_H */
