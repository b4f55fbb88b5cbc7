// Dense IQ_K members (IQ4_KS, IQ4_K, IQ5_K, IQ6_K): dequantization and the
// few-token decode GEMV over one [out_features, in_features] matrix.
//
// Reference: src/mlx_iqk/dense.py:116-220 (the serving functions) over the
// Metal kernels of src/mlx_iqk/dense_kernels.py:212-300; the relayout is
// src/mlx_iqk/format.py:898-1100 and the decode it must reproduce
// src/mlx_iqk/format.py:1166-1240.
//
// Streams per row (k-contiguous, little-endian):
//   qs  u32[n/8]   4-bit codes, weight k in nibble k % 8 of word k / 8
//   qh  u32        IQ5_K: 1 high bit per weight (n/32 words);
//                  IQ6_K: 2 high bits per weight (n/16 words)
//   scl u8         IQ4_KS: [n/32] bit 0 alphabet, bits 1-7 scale (index = (b & 254) - 127)
//                  IQ4_K / IQ5_K: [n/32] two 4-bit low scale parts per byte
//                  IQ6_K: [n/16] the signed scale itself
//   sch u8[n/64]   IQ4_K / IQ5_K: four 2-bit high scale parts per byte (index = lo | hi << 4, - 32)
//   sex u8[n/128]  block members: alphabet bit of 16-weight sub-block s at bit s % 8
//   dv             IQ4_KS: f32 per row; the others: f16 per 256 weights
// A weight is dl * value[(alphabet << W) | code] with dl = d * float(index),
// two separate float32 multiplies (the CPU dequantizer's chain), W = 4, 4, 5,
// 6; IQ6_K's values are the float32 outputs of ik's cubic, the others small
// integers.
//
// Dequantization (bit-exact): one thread per 16 weights; values from a
// shared-memory float table replicated once per lane (entry e of lane l at
// word 32 e + l: no bank conflicts whatever the codes), 16-byte chunks staged
// per warp so each store instruction writes 512 contiguous bytes.
//
// GEMV: a CTA owns 16 rows, its four warps a quarter of k each. Per 16-weight
// k tile a lane needs rows g and g + 8 at k = 2t, 2t + 1, 8 + 2t, 9 + 2t (the
// f16 m16n8k16 A fragment): byte t of two consecutive code words, so each
// weight is one table lookup of its f16 value (IQ6_K: an f16 pair hi + lo
// whose sum is the float32 value to 2^-22, through two MMAs). The tokens (up
// to 16 per pass, f16 as at the reference's call seam) are the N dimension;
// each sub-block's float32 partial sum is scaled by its dl into the float32
// accumulators, the four warps' sums meet in shared memory in a fixed order.
#include "iqk_common.cuh"
#include "iqk_dense_tables.h"

namespace iqk {
namespace {

__constant__ int8_t c_iq4k[32] = {IQK_IQ4K_VALUES};
__constant__ int8_t c_iq5nl[64] = {IQK_IQ5NL_VALUES};
__constant__ uint32_t c_iq6k[128] = {IQK_IQ6K_BITS};

template <int M> struct DenseGeo {
    static constexpr int kW = M == IQK_IQ5_K ? 5 : M == IQK_IQ6_K ? 6 : 4;  // code bits
    static constexpr int kEntries = 2 << kW;                                // both alphabets
    static constexpr int kSub = M == IQK_IQ4_KS ? 32 : 16;                  // weights per scale
};

struct DenseStreams {
    const uint32_t *qs;
    const uint32_t *qh;
    const uint8_t *scl, *sch, *sex;
    const void *dv;
};

__device__ __forceinline__ float table_value(int member, int e) {
    if (member == IQK_IQ6_K) return __uint_as_float(c_iq6k[e]);
    return (float)(member == IQK_IQ5_K ? c_iq5nl[e] : c_iq4k[e]);
}

// Scale of sub-block s of `row` (IQ4_KS: 32 weights, the others 16): dl and
// the alphabet bit.
template <int M>
__device__ __forceinline__ float sub_scale(const DenseStreams &st, int n, int64_t row, int s,
                                           int &alpha) {
    int index;
    float d;
    if (M == IQK_IQ4_KS) {
        const int b = st.scl[row * (n / 32) + s];
        index = (b & 254) - 127;
        alpha = b & 1;
        d = static_cast<const float *>(st.dv)[row];
    } else {
        if (M == IQK_IQ6_K) {
            index = (int)(int8_t)st.scl[row * (n / 16) + s];
        } else {
            const int lo = (st.scl[row * (n / 32) + (s >> 1)] >> (4 * (s & 1))) & 15;
            const int hi = (st.sch[row * (n / 64) + (s >> 2)] >> (2 * (s & 3))) & 3;
            index = (lo | (hi << 4)) - 32;
        }
        alpha = (st.sex[row * (n / 128) + (s >> 3)] >> (s & 7)) & 1;
        d = __half2float(__ushort_as_half(
            static_cast<const uint16_t *>(st.dv)[row * (n / 256) + (s >> 4)]));
    }
    return __fmul_rn(d, (float)index);
}

// High code bits of the 16 weights of unit u (weights 16u .. 16u + 15), at
// bit 4 of each weight's code: returned as a word holding W - 4 bits per weight.
template <int M>
__device__ __forceinline__ uint32_t unit_high(const DenseStreams &st, int n, int64_t row, int u) {
    if (M == IQK_IQ5_K) return (st.qh[row * (n / 32) + (u >> 1)] >> (16 * (u & 1))) & 0xffffu;
    if (M == IQK_IQ6_K) return st.qh[row * (n / 16) + u];
    return 0u;
}

template <typename OUT> __device__ __forceinline__ uint16_t bits16(float v) {
    const OUT h = from_float<OUT>(v);
    return *reinterpret_cast<const uint16_t *>(&h);
}

// ------------------------------------------------------------- dequant

template <int M, typename OUT>
__global__ void __launch_bounds__(256)
dense_dequant_kernel(DenseStreams st, int n, int64_t row_start, int64_t rows,
                     OUT *__restrict__ dst) {
    using DG = DenseGeo<M>;
    constexpr int CH = sizeof(OUT) == 4 ? 4 : 2;  // 16-byte chunks per unit
    __shared__ float tab[DG::kEntries * 32];
    __shared__ uint4 stage[256 / 32][32 * CH];
    const int lane = threadIdx.x & 31;
    for (int i = threadIdx.x; i < DG::kEntries * 32; i += blockDim.x)
        tab[i] = table_value(M, i >> 5);
    __syncthreads();
    const float *mytab = tab + lane;
    uint4 *my_stage = stage[threadIdx.x >> 5];
    const int upr = n / 16;  // units per row (a power of two, >= 64)
    const int64_t total = rows * upr;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    // total and stride are multiples of 32: every warp is all in or all out
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int64_t lr = i / upr;
        const int u = (int)(i - lr * upr);
        const int64_t row = row_start + lr;
        int alpha;
        const float dl = sub_scale<M>(st, n, row, M == IQK_IQ4_KS ? u >> 1 : u, alpha);
        const uint2 w = *reinterpret_cast<const uint2 *>(st.qs + row * (n / 8) + 2 * u);
        const uint32_t hi = unit_high<M>(st, n, row, u);
        const int base = alpha << DG::kW;
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            int c = (int)(((j < 8 ? w.x : w.y) >> (4 * (j & 7))) & 15u);
            if (M == IQK_IQ5_K) c |= (int)((hi >> j) & 1u) << 4;
            if (M == IQK_IQ6_K) c |= (int)((hi >> (2 * j)) & 3u) << 4;
            v[j] = __fmul_rn(dl, mytab[(base | c) * 32]);
        }
        uint4 out[CH];
        if constexpr (sizeof(OUT) == 4) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
                out[q] = make_uint4(__float_as_uint(v[4 * q]), __float_as_uint(v[4 * q + 1]),
                                    __float_as_uint(v[4 * q + 2]), __float_as_uint(v[4 * q + 3]));
        } else {
            uint32_t p[8];
#pragma unroll
            for (int q = 0; q < 8; ++q)
                p[q] = (uint32_t)bits16<OUT>(v[2 * q]) | ((uint32_t)bits16<OUT>(v[2 * q + 1]) << 16);
            out[0] = make_uint4(p[0], p[1], p[2], p[3]);
            out[1] = make_uint4(p[4], p[5], p[6], p[7]);
        }
        // a warp's 32 units are consecutive in one output row
#pragma unroll
        for (int c = 0; c < CH; ++c) my_stage[lane * CH + c] = out[c];
        __syncwarp();
        uint4 *wout = reinterpret_cast<uint4 *>(dst + lr * n + (int64_t)(u - lane) * 16);
#pragma unroll
        for (int c = 0; c < CH; ++c) __stcs(wout + 32 * c + lane, my_stage[32 * c + lane]);
        __syncwarp();
    }
}

// ---------------------------------------------------------------- GEMV

__device__ __forceinline__ void mma_f16(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(0.f));
}
__device__ __forceinline__ void mma_f16_acc(float d[4], const uint32_t a[4], uint32_t b0,
                                            uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

constexpr int kDenseWarps = 4;
constexpr int kDenseRows = 16;

// Table entry e of lane l at word 32 e + l: the value as f16 in the low half
// and, for IQ6_K, the f16 residual (float32 value - hi) in the high half.
template <int M> __device__ __forceinline__ uint32_t gemv_entry(int e) {
    const float v = table_value(M, e);
    const __half hi = __float2half_rn(v);
    const __half lo = M == IQK_IQ6_K ? __float2half_rn(v - __half2float(hi)) : __float2half_rn(0.f);
    return (uint32_t)__half_as_ushort(hi) | ((uint32_t)__half_as_ushort(lo) << 16);
}

// NT token tiles of 8 per pass (tokens t0 .. t0 + 8 NT - 1).
template <int M, int NT>
__global__ void __launch_bounds__(kDenseWarps * 32)
dense_gemv_kernel(DenseStreams st, int n, int out, const __half *__restrict__ x, int tokens,
                  void *__restrict__ y, int y_dtype) {
    using DG = DenseGeo<M>;
    __shared__ uint32_t tab[DG::kEntries * 32];
    __shared__ float red[kDenseWarps - 1][32][NT * 4];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    for (int i = threadIdx.x; i < DG::kEntries * 32; i += blockDim.x) tab[i] = gemv_entry<M>(i >> 5);
    __syncthreads();
    const uint32_t *mytab = tab + lane;
    const int r0 = blockIdx.x * kDenseRows;
    const int64_t ra = r0 + g, rb = r0 + g + 8;
    const int kq = n / kDenseWarps;       // this warp's k range: [wid * kq, (wid + 1) * kq)
    const int kbeg = wid * kq;
    for (int t0 = 0; t0 < tokens; t0 += 8 * NT) {
        float acc[NT][4];
#pragma unroll
        for (int q = 0; q < NT; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
        // B rows: token t0 + 8 q + g (zero past the last token)
        const __half *xb[NT];
        bool xok[NT];
#pragma unroll
        for (int q = 0; q < NT; ++q) {
            const int tk = t0 + 8 * q + g;
            xok[q] = tk < tokens;
            xb[q] = x + (int64_t)(xok[q] ? tk : 0) * n + 2 * t;
        }
#pragma unroll 1
        for (int k0 = kbeg; k0 < kbeg + kq; k0 += 32) {
            // two 16-weight tiles: code words k0/8 .. k0/8 + 3 of rows ra, rb
            const uint4 wa = *reinterpret_cast<const uint4 *>(st.qs + ra * (n / 8) + (k0 >> 3));
            const uint4 wb = *reinterpret_cast<const uint4 *>(st.qs + rb * (n / 8) + (k0 >> 3));
            uint32_t ha = 0, hb = 0;  // high bits of this lane's weights, both tiles
            if (M == IQK_IQ5_K) {
                ha = st.qh[ra * (n / 32) + (k0 >> 5)];
                hb = st.qh[rb * (n / 32) + (k0 >> 5)];
            }
            uint2 qa = make_uint2(0, 0), qb = make_uint2(0, 0);
            if (M == IQK_IQ6_K) {
                qa = *reinterpret_cast<const uint2 *>(st.qh + ra * (n / 16) + (k0 >> 4));
                qb = *reinterpret_cast<const uint2 *>(st.qh + rb * (n / 16) + (k0 >> 4));
            }
            int al_a, al_b;
            float dla[2], dlb[2];
            if (M == IQK_IQ4_KS) {
                dla[0] = dla[1] = sub_scale<M>(st, n, ra, k0 >> 5, al_a);
                dlb[0] = dlb[1] = sub_scale<M>(st, n, rb, k0 >> 5, al_b);
            }
#pragma unroll
            for (int h = 0; h < 2; ++h) {  // tile h: k0 + 16 h
                const uint32_t w0a = h ? wa.z : wa.x, w1a = h ? wa.w : wa.y;
                const uint32_t w0b = h ? wb.z : wb.x, w1b = h ? wb.w : wb.y;
                int aa = al_a, ab = al_b;
                if (M != IQK_IQ4_KS) {
                    dla[h] = sub_scale<M>(st, n, ra, (k0 >> 4) + h, aa);
                    dlb[h] = sub_scale<M>(st, n, rb, (k0 >> 4) + h, ab);
                }
                // codes of k = 16h + {2t, 2t+1} (word w0) and {8+2t, 9+2t} (word w1)
                int ca[4], cb[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int sh = 4 * (2 * t + (i & 1));
                    ca[i] = (int)(((i < 2 ? w0a : w1a) >> sh) & 15u);
                    cb[i] = (int)(((i < 2 ? w0b : w1b) >> sh) & 15u);
                    const int kk = 16 * h + 2 * t + (i & 1) + 8 * (i >> 1);  // weight within k0 .. k0+31
                    if (M == IQK_IQ5_K) {
                        ca[i] |= (int)((ha >> kk) & 1u) << 4;
                        cb[i] |= (int)((hb >> kk) & 1u) << 4;
                    }
                    if (M == IQK_IQ6_K) {
                        const uint32_t wa2 = kk < 16 ? qa.x : qa.y, wb2 = kk < 16 ? qb.x : qb.y;
                        ca[i] |= (int)((wa2 >> (2 * (kk & 15))) & 3u) << 4;
                        cb[i] |= (int)((wb2 >> (2 * (kk & 15))) & 3u) << 4;
                    }
                }
                uint32_t ea[4], eb[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    ea[i] = mytab[((aa << DG::kW) | ca[i]) * 32];
                    eb[i] = mytab[((ab << DG::kW) | cb[i]) * 32];
                }
                // A: a0 = row g (k 2t, 2t+1), a1 = row g+8, a2 = row g (k 8+2t, 9+2t), a3 = row g+8
                uint32_t A[4] = {__byte_perm(ea[0], ea[1], 0x5410), __byte_perm(eb[0], eb[1], 0x5410),
                                 __byte_perm(ea[2], ea[3], 0x5410), __byte_perm(eb[2], eb[3], 0x5410)};
                uint32_t L[4];
                if (M == IQK_IQ6_K) {
                    L[0] = __byte_perm(ea[0], ea[1], 0x7632);
                    L[1] = __byte_perm(eb[0], eb[1], 0x7632);
                    L[2] = __byte_perm(ea[2], ea[3], 0x7632);
                    L[3] = __byte_perm(eb[2], eb[3], 0x7632);
                }
#pragma unroll
                for (int q = 0; q < NT; ++q) {
                    const int kx = k0 + 16 * h;
                    const uint32_t b0 = xok[q] ? __ldg(reinterpret_cast<const unsigned int *>(xb[q] + kx)) : 0u;
                    const uint32_t b1 = xok[q] ? __ldg(reinterpret_cast<const unsigned int *>(xb[q] + kx + 8)) : 0u;
                    float d[4];
                    mma_f16(d, A, b0, b1);
                    if (M == IQK_IQ6_K) mma_f16_acc(d, L, b0, b1);
                    // this tile's partial sums, scaled by its sub-block's dl (rows g, g+8)
                    acc[q][0] = fmaf(dla[h], d[0], acc[q][0]);
                    acc[q][1] = fmaf(dla[h], d[1], acc[q][1]);
                    acc[q][2] = fmaf(dlb[h], d[2], acc[q][2]);
                    acc[q][3] = fmaf(dlb[h], d[3], acc[q][3]);
                }
            }
        }
        // the four k quarters meet in warp 0, added in warp order
        if (wid > 0) {
#pragma unroll
            for (int q = 0; q < NT; ++q)
#pragma unroll
                for (int i = 0; i < 4; ++i) red[wid - 1][lane][q * 4 + i] = acc[q][i];
        }
        __syncthreads();
        if (wid == 0) {
#pragma unroll
            for (int w = 0; w < kDenseWarps - 1; ++w)
#pragma unroll
                for (int q = 0; q < NT; ++q)
#pragma unroll
                    for (int i = 0; i < 4; ++i) acc[q][i] += red[w][lane][q * 4 + i];
            // D fragment: d0 = (row g, token 2t), d1 = (row g, 2t+1), d2/d3 rows g+8
#pragma unroll
            for (int q = 0; q < NT; ++q) {
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int tk = t0 + 8 * q + 2 * t + (i & 1);
                    const int64_t row = (i < 2) ? ra : rb;
                    if (tk < tokens) {
                        const int64_t o = (int64_t)tk * out + row;
                        if (y_dtype == IQK_F32) static_cast<float *>(y)[o] = acc[q][i];
                        else static_cast<__half *>(y)[o] = __float2half_rn(acc[q][i]);
                    }
                }
            }
        }
        __syncthreads();
    }
}

template <int M> DenseStreams dense_streams(const void *const *s) {
    DenseStreams st{};
    st.qs = static_cast<const uint32_t *>(s[0]);
    int i = 1;
    if (M == IQK_IQ5_K || M == IQK_IQ6_K) st.qh = static_cast<const uint32_t *>(s[i++]);
    st.scl = static_cast<const uint8_t *>(s[i++]);
    if (M == IQK_IQ4_K || M == IQK_IQ5_K) st.sch = static_cast<const uint8_t *>(s[i++]);
    if (M != IQK_IQ4_KS) st.sex = static_cast<const uint8_t *>(s[i++]);
    st.dv = s[i];
    return st;
}

template <int M>
cudaError_t dequant_m(const void *const *s, int n, int64_t row_start, int64_t rows, void *dst,
                      int out_dtype, cudaStream_t stream, int num_sms) {
    const DenseStreams st = dense_streams<M>(s);
    const int64_t units = rows * (n / 16);
    int64_t blocks = (units + 255) / 256;
    const int64_t cap = (int64_t)num_sms * 8;
    if (blocks > cap) blocks = cap;
    if (out_dtype == IQK_F32)
        dense_dequant_kernel<M, float><<<(unsigned)blocks, 256, 0, stream>>>(
            st, n, row_start, rows, static_cast<float *>(dst));
    else if (out_dtype == IQK_F16)
        dense_dequant_kernel<M, __half><<<(unsigned)blocks, 256, 0, stream>>>(
            st, n, row_start, rows, static_cast<__half *>(dst));
    else
        dense_dequant_kernel<M, __nv_bfloat16><<<(unsigned)blocks, 256, 0, stream>>>(
            st, n, row_start, rows, static_cast<__nv_bfloat16 *>(dst));
    return cudaGetLastError();
}

template <int M>
cudaError_t gemv_m(const void *const *s, int n, int out, const void *x, int tokens, void *y,
                   int y_dtype, cudaStream_t stream) {
    const DenseStreams st = dense_streams<M>(s);
    const unsigned blocks = (unsigned)(out / kDenseRows);
    const __half *xh = static_cast<const __half *>(x);
    if (tokens <= 8)
        dense_gemv_kernel<M, 1><<<blocks, kDenseWarps * 32, 0, stream>>>(st, n, out, xh, tokens, y, y_dtype);
    else
        dense_gemv_kernel<M, 2><<<blocks, kDenseWarps * 32, 0, stream>>>(st, n, out, xh, tokens, y, y_dtype);
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_dense_dequant(int member, const void *const *streams, int n, int64_t row_start,
                                 int64_t rows, void *dst, int out_dtype, cudaStream_t stream,
                                 int num_sms) {
    if (rows <= 0) return cudaSuccess;
    switch (member) {
        case IQK_IQ4_KS: return dequant_m<IQK_IQ4_KS>(streams, n, row_start, rows, dst, out_dtype, stream, num_sms);
        case IQK_IQ4_K: return dequant_m<IQK_IQ4_K>(streams, n, row_start, rows, dst, out_dtype, stream, num_sms);
        case IQK_IQ5_K: return dequant_m<IQK_IQ5_K>(streams, n, row_start, rows, dst, out_dtype, stream, num_sms);
        default: return dequant_m<IQK_IQ6_K>(streams, n, row_start, rows, dst, out_dtype, stream, num_sms);
    }
}

cudaError_t launch_dense_gemv(int member, const void *const *streams, int n, int out,
                              const void *x, int tokens, void *y, int y_dtype,
                              cudaStream_t stream) {
    if (tokens <= 0) return cudaSuccess;
    switch (member) {
        case IQK_IQ4_KS: return gemv_m<IQK_IQ4_KS>(streams, n, out, x, tokens, y, y_dtype, stream);
        case IQK_IQ4_K: return gemv_m<IQK_IQ4_K>(streams, n, out, x, tokens, y, y_dtype, stream);
        case IQK_IQ5_K: return gemv_m<IQK_IQ5_K>(streams, n, out, x, tokens, y, y_dtype, stream);
        default: return gemv_m<IQK_IQ6_K>(streams, n, out, x, tokens, y, y_dtype, stream);
    }
}

}  // namespace iqk
