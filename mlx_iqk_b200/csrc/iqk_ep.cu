// Pair-list helpers of the expert-parallel layer (sm_100a).
//
// The reference serves a whole MoE layer on one device; its SwitchGLU seam
// (src/mlx_iqk/nn.py:1-22: gate and up on the token, SiLU(gate) * up, down,
// router-weighted sum over top-k) is what the expert-parallel layer shards.
// Each rank runs the grouped GEMMs over the full pair list of all ranks'
// tokens with a shard preparation (pairs of other ranks' experts skipped), so
// these two kernels touch only this rank's pairs:
//
//   pairs_swiglu_kernel   h[q] = bf16((silu(g[q]) * u[q]) * w[q]) for every
//                         routed pair q of a prepared workspace (the router
//                         weight goes in before the down projection, which is
//                         linear); one block per sorted position, positions
//                         past the routable count exit at once.
//   pairs_combine_kernel  out[r] = sum over j < k, in order, of y[r*k + j]
//                         for the slots whose expert lies in [0, E); rows
//                         without one are written as zeros.
//
// Both are HBM-bound streams: 16-byte loads, no shared memory.

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "iqk_grouped.cuh"

namespace iqk {
namespace {

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

__device__ __forceinline__ uint32_t bf16x2_bits(float lo, float hi) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&b);
}

__global__ void __launch_bounds__(256)
pairs_swiglu_kernel(const float *__restrict__ g, const float *__restrict__ u,
                    const float *__restrict__ w, int inter, const int32_t *__restrict__ hdr,
                    const int32_t *__restrict__ order, __nv_bfloat16 *__restrict__ h) {
    const int pos = blockIdx.x;
    if (pos >= hdr[2]) return;
    const int64_t q = order[pos];
    const float wq = w[q];
    const float4 *g4 = reinterpret_cast<const float4 *>(g + q * inter);
    const float4 *u4 = reinterpret_cast<const float4 *>(u + q * inter);
    uint2 *h4 = reinterpret_cast<uint2 *>(h + q * inter);
    for (int i = threadIdx.x; i < inter / 4; i += blockDim.x) {
        const float4 a = __ldcs(g4 + i), b = __ldcs(u4 + i);
        h4[i] = make_uint2(bf16x2_bits(silu(a.x) * b.x * wq, silu(a.y) * b.y * wq),
                           bf16x2_bits(silu(a.z) * b.z * wq, silu(a.w) * b.w * wq));
    }
}

template <typename OUT>
__global__ void __launch_bounds__(256)
pairs_combine_kernel(const float *__restrict__ y, const int32_t *__restrict__ sel, int top_k,
                     int num_experts, int hidden, OUT *__restrict__ out) {
    const int64_t r = blockIdx.x;
    const int32_t *s = sel + r * top_k;
    const float4 *y4 = reinterpret_cast<const float4 *>(y);
    const int h4 = hidden / 4;
    for (int i = threadIdx.x; i < h4; i += blockDim.x) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < top_k; ++j) {
            const int e = s[j];
            if (e < 0 || e >= num_experts) continue;
            const float4 v = __ldcs(y4 + (r * top_k + j) * h4 + i);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        if constexpr (sizeof(OUT) == 4) {
            reinterpret_cast<float4 *>(out)[r * h4 + i] = acc;
        } else {
            reinterpret_cast<uint2 *>(out)[r * h4 + i] =
                make_uint2(bf16x2_bits(acc.x, acc.y), bf16x2_bits(acc.z, acc.w));
        }
    }
}

// h[r, c] = silu(g[r, c]) * u[r, c] * (w ? w[r] : 1), float32 rows: the
// SwitchGLU step of a layer whose gate and up projections have different
// members (one decode launch serves a same-member pair).
__global__ void __launch_bounds__(256)
rows_swiglu_kernel(const float *__restrict__ g, const float *__restrict__ u,
                   const float *__restrict__ w, int cols, float *__restrict__ h) {
    const int64_t r = blockIdx.x;
    const float wr = w ? w[r] : 1.f;
    const float4 *g4 = reinterpret_cast<const float4 *>(g + r * cols);
    const float4 *u4 = reinterpret_cast<const float4 *>(u + r * cols);
    float4 *h4 = reinterpret_cast<float4 *>(h + r * cols);
    for (int i = threadIdx.x; i < cols / 4; i += blockDim.x) {
        const float4 a = g4[i], b = u4[i];
        h4[i] = make_float4(silu(a.x) * b.x * wr, silu(a.y) * b.y * wr, silu(a.z) * b.z * wr,
                            silu(a.w) * b.w * wr);
    }
}

}  // namespace

cudaError_t launch_rows_swiglu(const float *g, const float *u, const float *w, int64_t rows,
                               int cols, float *h, cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    rows_swiglu_kernel<<<(unsigned)rows, 256, 0, stream>>>(g, u, w, cols, h);
    return cudaGetLastError();
}

cudaError_t launch_pairs_swiglu(const float *g, const float *u, const float *w, int inter,
                                int n, int64_t num_experts, int64_t pairs, const void *ws,
                                void *h, cudaStream_t stream) {
    if (pairs == 0) return cudaSuccess;
    const GroupedLayout L = grouped_layout(n, num_experts, pairs);
    const char *b = static_cast<const char *>(ws);
    pairs_swiglu_kernel<<<(unsigned)pairs, 256, 0, stream>>>(
        g, u, w, inter, reinterpret_cast<const int32_t *>(b + L.hdr),
        reinterpret_cast<const int32_t *>(b + L.order), static_cast<__nv_bfloat16 *>(h));
    return cudaGetLastError();
}

cudaError_t launch_pairs_combine(const float *y, const int32_t *sel, int64_t rows, int top_k,
                                 int64_t num_experts, int hidden, void *out, int out_dtype,
                                 cudaStream_t stream) {
    if (rows == 0) return cudaSuccess;
    if (out_dtype == IQK_F32)
        pairs_combine_kernel<float><<<(unsigned)rows, 256, 0, stream>>>(
            y, sel, top_k, (int)num_experts, hidden, static_cast<float *>(out));
    else
        pairs_combine_kernel<__nv_bfloat16><<<(unsigned)rows, 256, 0, stream>>>(
            y, sel, top_k, (int)num_experts, hidden, static_cast<__nv_bfloat16 *>(out));
    return cudaGetLastError();
}

}  // namespace iqk
