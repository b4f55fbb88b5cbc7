// Grouped per-expert GEMM (prefill route): host-side layout and launchers.
#pragma once

#include "iqk_common.cuh"

namespace iqk {

// Workspace of one grouped call, all written by the preparation:
//   hdr     [16] int32: [0] device error bits, [1] work tiles, [2] routable pairs,
//           [3] 1 for a shard preparation (pairs of other ranks' experts skipped)
//   order   [pairs] int32: sorted position -> pair (unroutable pairs at the tail)
//   pscale  [pairs] int32: power-of-two exponent S of each position's activation row
//   tiles   [max_tiles] int4: {expert, first position, tokens (<= tok_cap), 0}
//   xs      [pairs, n] f16: activation rows in sorted order, scaled by 2^S and
//           permuted inside every 16-element block to the weight operand's order
struct GroupedLayout {
    size_t hdr, order, pscale, tiles, xs;
    int64_t max_tiles;
    int tok_cap;  // tokens per work tile (64: the MMA N and the accumulator width)
    size_t total;
};

constexpr int kGroupTokMax = 128;  // largest work tile (the MMA's N, padded to 16)
constexpr int kGroupRows = 128;    // output rows per work item (the MMA's M)

GroupedLayout grouped_layout(int64_t n, int64_t num_experts, int64_t pairs);

cudaError_t launch_grouped_prepare(const void *x, int x_dtype, int64_t x_rows, int n,
                                   int64_t num_experts, const int32_t *sel, const int32_t *tok,
                                   int64_t pairs, void *ws, cudaStream_t stream,
                                   bool shard = false);

// Pair-list helpers of the expert-parallel layer, over a prepared workspace
// (iqk_ep.cu): h[q] = bf16(silu(g[q]) * u[q] * w[q]) for the routed pairs q,
// and out[r] = sum_j y[r*k + j] over the slots of row r whose expert lies in
// [0, num_experts).
cudaError_t launch_pairs_swiglu(const float *g, const float *u, const float *w, int inter,
                                int n, int64_t num_experts, int64_t pairs, const void *ws,
                                void *h, cudaStream_t stream);
cudaError_t launch_rows_swiglu(const float *g, const float *u, const float *w, int64_t rows,
                               int cols, float *h, cudaStream_t stream);
cudaError_t launch_pairs_combine(const float *y, const int32_t *sel, int64_t rows, int top_k,
                                 int64_t num_experts, int hidden, void *out, int out_dtype,
                                 cudaStream_t stream);

cudaError_t launch_grouped_run(int member, const void *const *streams, int64_t num_experts,
                               int64_t out_features, int n, int64_t pairs, void *y, int y_dtype,
                               const void *ws, cudaStream_t stream, int num_sms,
                               int64_t row_start = 0, int64_t rows_out = -1);

}  // namespace iqk
