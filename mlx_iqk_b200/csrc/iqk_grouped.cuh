// Grouped per-expert GEMM (prefill route): host-side layout and launchers.
#pragma once

#include "iqk_common.cuh"

namespace iqk {

// Workspace of one grouped call, all written by the preparation:
//   hdr     [16] int32: [0] device error bits, [1] work tiles, [2] routable pairs
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
                                   int64_t pairs, void *ws, cudaStream_t stream);

cudaError_t launch_grouped_run(int member, const void *const *streams, int64_t num_experts,
                               int64_t out_features, int n, int64_t pairs, void *y, int y_dtype,
                               const void *ws, cudaStream_t stream, int num_sms);

}  // namespace iqk
