// Host/device layout of the decode GEMV's workspace.
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

namespace iqk {

// Exponent sentinel for an activation row that held a NaN or infinity.
constexpr int kScaleNonFinite = -0x40000000;

// One work tile of the run kernel: an expert and one of its pairs (the
// pair1/tok1/sh1 slots are spare). sh0 is filled in by the run kernel from
// the row exponent.
struct TileRef {
    int32_t e, pair0, pair1, tok0, tok1, sh0, sh1, npair;
};
static_assert(sizeof(TileRef) == 32, "TileRef is 32 bytes");

// Byte offsets inside the caller's workspace (all 256-byte aligned).
struct GemvLayout {
    size_t hdr;     // int32[16]: [0] error bits, [3] routable pairs (work tiles),
                    //   [8] items claimed, [9] CTAs done (the run kernels' counters)
    size_t order;   // int32[P]      pair ids bucketed by expert, unroutable ones last
    size_t ptok;    // int32[P]      activation row of each pair
    size_t tiles1;  // TileRef[P]    one work tile per routable pair, grouped by expert
    size_t xscale;  // int32[x_rows] power-of-two exponent S of each row
    size_t xbuf;    // per row: int8 planes [n/32][3][4][8], int32 block sums [n/32][4]
    int64_t xrow_bytes;
    size_t total;
};

GemvLayout gemv_layout(int member, int64_t n, int64_t x_rows, int64_t pairs);
int gemv_smem_for(int member, int n, bool narrow);
cudaError_t launch_gemv_prepare(const void *x, int x_dtype, int64_t x_rows, int n,
                                int64_t num_experts, const int32_t *sel, const int32_t *tok,
                                int64_t pairs, void *ws, cudaStream_t stream);
cudaError_t launch_gemv_run(int member, const void *const *streams, int64_t num_experts,
                            int64_t out_features, int n, int64_t x_rows, int64_t pairs, void *y,
                            int y_dtype, const void *ws, cudaStream_t stream, int num_sms,
                            bool floor = false, const void *const *up_streams = nullptr,
                            const float *router_weight = nullptr);
cudaError_t launch_bounded_wait_check(int64_t limit_ns, int32_t *flags, cudaStream_t stream);
cudaError_t launch_pack(int member, const void *wire, int64_t rows, int n,
                        void *const *streams, cudaStream_t stream, int num_sms);
cudaError_t launch_dequant(int member, const void *const *streams, int64_t num_experts,
                           int64_t out_features, int n, int64_t row_start,
                           int64_t rows, int out_dtype, void *dst, cudaStream_t stream,
                           int num_sms, bool floor = false);

}  // namespace iqk
