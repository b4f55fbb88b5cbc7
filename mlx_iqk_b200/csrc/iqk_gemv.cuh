// Host/device layout of the decode GEMV's workspace.
#pragma once
#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

namespace iqk {

// Exponent sentinel for an activation row that held a NaN or infinity.
constexpr int kScaleNonFinite = -0x40000000;

// Byte offsets inside the caller's workspace (all 256-byte aligned).
struct GemvLayout {
    size_t hdr;     // int32[16]: [0] device error bits, [1] distinct experts U, [2] items
    size_t uniq;    // int32[U]    distinct expert ids, ascending
    size_t seg;     // int32[U+1]  pair-list offsets per distinct expert
    size_t ubase;   // int32[U+1]  first warp item of each distinct expert
    size_t order;   // int32[P]    pair ids bucketed by expert
    size_t ptok;    // int32[P]    activation row of each pair
    size_t xscale;  // int32[x_rows] power-of-two exponent S of each row
    size_t xbuf;    // int8 [x_rows][n/32][4][4][8] digit planes (+ block sums)
    int64_t xrow_bytes;
    size_t total;
};

GemvLayout gemv_layout(int member, int64_t n, int64_t x_rows, int64_t pairs);
int gemv_smem_for(int member, int n);
cudaError_t launch_gemv(int member, const void *x, int x_dtype, int64_t x_rows,
                        const void *const *streams, int64_t num_experts,
                        int64_t out_features, int n, const int32_t *sel,
                        const int32_t *tok, int64_t pairs, void *y, int y_dtype,
                        void *ws, cudaStream_t stream, int num_sms);
cudaError_t launch_dequant(int member, const void *const *streams, int64_t num_experts,
                           int64_t out_features, int n, int64_t row_start,
                           int64_t rows, int out_dtype, void *dst, cudaStream_t stream,
                           int num_sms);

}  // namespace iqk
