// Bit-exact stacked dequantization of the IQ_K relayout streams.
//
// One thread reconstructs one 16-weight code word (2-bit members) or one
// 32-weight block (IQ1_S_R4) of one output row and writes it with 16-byte
// streaming stores. Every weight of a group (block) is one of the group's
// four (three) float32 products, computed once per thread; 16-bit outputs
// place them with byte permutes. The arithmetic is the
// CPU dequantizer's float32 chain in its order
// (vendor/ik_llama/iqk_iq2.cpp:502-562, vendor/ik_llama/iqk_iq1sr4.cpp:581-604;
// the reference's Metal restatement is src/mlx_iqk/kernels.py:631-742):
//
//   2-bit members  dl = d * float(idx);             w = dl * float(value)
//   IQ1_S_R4       dl = d * float(2 * ls + 1);      w = dl * (float(g) + shift)
//
// Two separate multiplies cannot be contracted into an FMA, so the float32
// result equals the CPU's bit for bit; a 16-bit output is then one
// round-to-nearest-even conversion, the same as numpy's astype.
#include "iqk_common.cuh"
#include "iqk_tables.cuh"

namespace iqk {

struct StreamPtrs {
    const void *p[5];
};

#ifndef IQK_DQ_ST
#define IQK_DQ_ST(p, v) __stcs(p, v)  // streaming stores: the output is not re-read here
#endif

__device__ __forceinline__ uint32_t prmt_dq(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// A warp's 32 units are consecutive in one output row, CH 16-byte chunks each.
// HBM writes run at full rate when every warp store instruction covers 512
// contiguous bytes (measured on B200: 6.2 TB/s, against 3.5 TB/s for 32
// bytes per thread in two stores), so a unit's chunks go through a per-warp
// shared-memory stage and come out lane-contiguous.
template <int CH>
__device__ __forceinline__ void warp_store(uint4 *warp_out, const uint4 (&v)[CH], uint4 *stage,
                                           int lane) {
#pragma unroll
    for (int c = 0; c < CH; ++c) stage[lane * CH + c] = v[c];
    __syncwarp();
#pragma unroll
    for (int c = 0; c < CH; ++c) IQK_DQ_ST(warp_out + 32 * c + lane, stage[32 * c + lane]);
    __syncwarp();
}

template <typename OUT> __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    const OUT a = from_float<OUT>(lo), b = from_float<OUT>(hi);
    return (uint32_t)*reinterpret_cast<const uint16_t *>(&a) |
           ((uint32_t)*reinterpret_cast<const uint16_t *>(&b) << 16);
}

// 2-bit members, one 16-weight code word per thread. A group's four
// float32 products dl * value are computed once with the CPU's
// chain; every weight is then one of them, so the result is the same bit for
// bit. 16-bit outputs place them with byte permutes (selector bytes 2c, 2c+1
// pick entry c of the {T0,T1,T2,T3} table; pairs come out as (k, k+4) and
// one more permute restores k order).
template <typename OUT>
__device__ __forceinline__ void expand_word(uint32_t word, const float t[4],
                                            uint4 (&v)[sizeof(OUT) == 4 ? 4 : 2]) {
    if constexpr (sizeof(OUT) == 4) {
        float w[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const uint32_t c = (word >> (2 * k)) & 3u;
            const float lo2 = (c & 1u) ? t[1] : t[0], hi2 = (c & 1u) ? t[3] : t[2];
            w[k] = (c & 2u) ? hi2 : lo2;
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
            v[q] = make_uint4(__float_as_uint(w[4 * q]), __float_as_uint(w[4 * q + 1]),
                              __float_as_uint(w[4 * q + 2]), __float_as_uint(w[4 * q + 3]));
    } else {
        const uint32_t t01 = pack2<OUT>(t[0], t[1]), t23 = pack2<OUT>(t[2], t[3]);
        uint32_t r[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t m = (word >> (2 * j)) & 0x03030303u;  // codes j, 4+j, 8+j, 12+j
            const uint32_t sel = m * 0x22u + 0x10101010u;
            r[j] = prmt_dq(t01, t23, sel);
            r[4 + j] = prmt_dq(t01, t23, sel >> 16);
        }
        v[0] = make_uint4(prmt_dq(r[0], r[1], 0x5410u), prmt_dq(r[2], r[3], 0x5410u),
                          prmt_dq(r[0], r[1], 0x7632u), prmt_dq(r[2], r[3], 0x7632u));
        v[1] = make_uint4(prmt_dq(r[4], r[5], 0x5410u), prmt_dq(r[6], r[7], 0x5410u),
                          prmt_dq(r[4], r[5], 0x7632u), prmt_dq(r[6], r[7], 0x7632u));
    }
}

// IQ1_S_R4 octet: its 2-bit grid values (g + 1 in bits 2j, 2j+1 of the
// 16-bit grid entry) pick one of the block's three float32 products
// t[g + 1] = dl * (g + shift), computed once with the CPU's chain -- so the
// result is the same bit for bit -- placed like the low half of a code word.
template <typename OUT>
__device__ __forceinline__ void expand_octet(uint32_t code, const float t[4], uint4 *v) {
    if constexpr (sizeof(OUT) == 4) {
        float w[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t c = (code >> (2 * k)) & 3u;
            w[k] = c == 0u ? t[0] : (c == 1u ? t[1] : t[2]);
        }
        v[0] = make_uint4(__float_as_uint(w[0]), __float_as_uint(w[1]), __float_as_uint(w[2]),
                          __float_as_uint(w[3]));
        v[1] = make_uint4(__float_as_uint(w[4]), __float_as_uint(w[5]), __float_as_uint(w[6]),
                          __float_as_uint(w[7]));
    } else {
        const uint32_t t01 = pack2<OUT>(t[0], t[1]), t23 = pack2<OUT>(t[2], t[3]);
        uint32_t r[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t m = (code >> (2 * j)) & 0x00000303u;  // codes j, 4+j
            r[j] = prmt_dq(t01, t23, m * 0x22u + 0x10101010u);
        }
        v[0] = make_uint4(prmt_dq(r[0], r[1], 0x5410u), prmt_dq(r[2], r[3], 0x5410u),
                          prmt_dq(r[0], r[1], 0x7632u), prmt_dq(r[2], r[3], 0x7632u));
    }
}

__device__ __forceinline__ void group_table(float dl, int alpha, float t[4]) {
    const uint32_t tab = alpha ? kIq2Tab1 : kIq2Tab0;
#pragma unroll
    for (int c = 0; c < 4; ++c) t[c] = dl * (float)(int)(int8_t)(tab >> (8 * c));
}

// FLOOR (both kernels): the address floor the reference prices its
// dequantization against (bench/floors.py:1-17, dequant_floor_source): the
// same loads and the same warp-staged stores, with the decode deleted -- the
// loaded words are folded into an integer that is what gets stored. Only the
// benchmark's floor entry point uses it.
template <bool FLOOR, int CH>
__device__ __forceinline__ void fold_store(uint32_t f, uint4 (&v)[CH]) {
#pragma unroll
    for (int c = 0; c < CH; ++c) v[c] = make_uint4(f, f + 1u, f + 2u, f + 3u);
}

template <int MEMBER, typename OUT, bool FLOOR = false>
__global__ void __launch_bounds__(256)
dequant_words_kernel(StreamPtrs sp, uint32_t total_words, int log2_words, int n,
                     int64_t out_features, int64_t row_start, uint32_t rows,
                     OUT *__restrict__ dst) {
    constexpr int CH = sizeof(OUT) == 4 ? 4 : 2;  // 16-byte chunks per word
    __shared__ uint4 stage[256 / 32][32 * CH];
    const int lane = threadIdx.x & 31;
    uint4 *my_stage = stage[threadIdx.x >> 5];
    const uint32_t stride = gridDim.x * blockDim.x;
    const uint32_t *qs = static_cast<const uint32_t *>(sp.p[0]);
    // total_words and stride are multiples of 32: every warp is all in or all out
    for (uint32_t u = blockIdx.x * blockDim.x + threadIdx.x; u < total_words; u += stride) {
        const uint32_t lin = u >> log2_words;  // [expert, local row]
        const int wi = (int)(u & ((1u << log2_words) - 1u));
        const uint32_t e = lin / rows;
        const int64_t srow = (int64_t)e * out_features + row_start + (lin - e * rows);
        const uint32_t word = __ldg(qs + srow * (n / 16) + wi);
        float t[4];
        if (MEMBER == IQK_IQ2_KS) {
            const uint8_t *scl = static_cast<const uint8_t *>(sp.p[1]);
            const uint8_t *sch = static_cast<const uint8_t *>(sp.p[2]);
            const uint8_t *sex = static_cast<const uint8_t *>(sp.p[3]);
            const uint16_t *dv = static_cast<const uint16_t *>(sp.p[4]);
            const int g = wi >> 1;
            const int lo = (__ldg(scl + srow * (n / 64) + (g >> 1)) >> (4 * (g & 1))) & 15;
            const int hi = (__ldg(sch + srow * (n / 256) + (g >> 3)) >> (g & 7)) & 1;
            const int alpha = (__ldg(sex + srow * (n / 256) + (g >> 3)) >> (g & 7)) & 1;
            if (FLOOR) {
                t[0] = __uint_as_float(word + 3u * lo + 5u * hi + 7u * alpha +
                                       11u * __ldg(dv + srow));
            } else {
                group_table(half_bits_to_float(__ldg(dv + srow)) *
                                (float)((lo | (hi << 4)) - 16), alpha, t);
            }
        } else {
            const uint8_t *scl = static_cast<const uint8_t *>(sp.p[1]);
            const uint8_t *sex = static_cast<const uint8_t *>(sp.p[2]);
            const uint16_t *dv = static_cast<const uint16_t *>(sp.p[3]);
            const int sb = wi;
            const int lo = (__ldg(scl + srow * (n / 32) + (sb >> 1)) >> (4 * (sb & 1))) & 15;
            const int alpha = (__ldg(sex + srow * (n / 128) + (sb >> 3)) >> (sb & 7)) & 1;
            if (FLOOR) {
                t[0] = __uint_as_float(word + 3u * lo + 7u * alpha +
                                       11u * __ldg(dv + srow * (n / 256) + (sb >> 4)));
            } else {
                group_table(half_bits_to_float(__ldg(dv + srow * (n / 256) + (sb >> 4))) *
                                (float)(lo - 8), alpha, t);
            }
        }
        uint4 v[CH];
        if (FLOOR) fold_store<FLOOR, CH>(__float_as_uint(t[0]), v);
        else expand_word<OUT>(word, t, v);
        warp_store<CH>(reinterpret_cast<uint4 *>(dst + (int64_t)lin * n + (wi - lane) * 16), v,
                       my_stage, lane);
    }
}

// IQ1_S_R4: one half block (16 weights, two octets: two grid bytes of the qs
// word and their qh bits) per thread, so a thread writes 32 contiguous bytes
// at 16-bit outputs -- the store pattern of the 2-bit word kernel.
template <typename OUT, bool FLOOR = false>
__global__ void __launch_bounds__(256)
dequant_iq1_kernel(StreamPtrs sp, uint32_t total_halves, int log2_halves, int n,
                   int64_t out_features, int64_t row_start, uint32_t rows,
                   OUT *__restrict__ dst) {
    __shared__ uint16_t grid[2048];
    for (int i = threadIdx.x; i < 2048; i += blockDim.x) grid[i] = g_iq1s_grid[i];
    __syncthreads();
    const uint32_t *qs = static_cast<const uint32_t *>(sp.p[0]);
    const uint16_t *qh = static_cast<const uint16_t *>(sp.p[1]);
    const uint16_t *dv = static_cast<const uint16_t *>(sp.p[2]);
    constexpr int CH = sizeof(OUT) == 4 ? 4 : 2;  // 16-byte chunks per half block
    __shared__ uint4 stage[256 / 32][32 * CH];
    const int lane = threadIdx.x & 31;
    uint4 *my_stage = stage[threadIdx.x >> 5];
    const uint32_t stride = gridDim.x * blockDim.x;
    const bool whole = rows == out_features;
    // total_halves and stride are multiples of 32: every warp is all in or all out  // whole experts: source row == output row
    for (uint32_t u = blockIdx.x * blockDim.x + threadIdx.x; u < total_halves; u += stride) {
        const uint32_t lin = u >> log2_halves;  // [expert, local row]
        const int hb = (int)(u & ((1u << log2_halves) - 1u));
        const int b = hb >> 1;
        int64_t srow = lin;
        if (!whole) {
            const uint32_t e = lin / rows;
            srow = (int64_t)e * out_features + row_start + (lin - e * rows);
        }
        const uint32_t qw = __ldg(qs + srow * (n / 32) + b);
        const uint32_t h = __ldg(qh + srow * (n / 32) + b);
        const float dl = half_bits_to_float(__ldg(dv + srow)) *
                         (float)(int)(2u * ((h >> 12) & 7u) + 1u);
        const float shift = (h & 0x8000u) ? -0.125f : 0.125f;
        const float t[4] = {dl * (-1.0f + shift), dl * (0.0f + shift), dl * (1.0f + shift), 0.0f};
        uint4 v[CH];
        if (FLOOR) {
            // the grid gathers are addressing, not decode: kept
            uint32_t f = qw + 3u * h + 5u * __ldg(dv + srow);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int i = 2 * (hb & 1) + q;
                f += (7u + 4u * q) * grid[((qw >> (8 * i)) & 0xffu) | (((h >> (3 * i)) & 7u) << 8)];
            }
            fold_store<FLOOR, CH>(f, v);
        } else {
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int i = 2 * (hb & 1) + q;  // octet of the block
                const uint32_t code = grid[((qw >> (8 * i)) & 0xffu) | (((h >> (3 * i)) & 7u) << 8)];
                expand_octet<OUT>(code, t, v + q * (CH / 2));
            }
        }
        warp_store<CH>(reinterpret_cast<uint4 *>(dst + (int64_t)lin * n + (hb - lane) * 16), v,
                       my_stage, lane);
    }
}

cudaError_t launch_dequant(int member, const void *const *streams, int64_t num_experts,
                           int64_t out_features, int n, int64_t row_start,
                           int64_t rows, int out_dtype, void *dst, cudaStream_t stream,
                           int num_sms, bool floor) {
    StreamPtrs sp{};
    const RowBytes rb = row_bytes(member, n);
    for (int i = 0; i < rb.count; ++i) sp.p[i] = streams[i];
    const int log2_octs = n == 4096 ? 9 : 8;  // n / 8 octets per row
    const int elem = out_dtype == IQK_F32 ? 4 : 2;
    // 32-bit unit indices: split the expert range so each launch stays below 2^31.
    const int64_t per_expert = rows * (n / 16);  // 16-weight units of both kernels
    if (per_expert == 0 || num_experts == 0) return cudaSuccess;
    const int64_t chunk = ((int64_t)1 << 31) / per_expert;
    for (int64_t e0 = 0; e0 < num_experts; e0 += chunk) {
        const int64_t ne = num_experts - e0 < chunk ? num_experts - e0 : chunk;
        const uint32_t total = (uint32_t)(ne * per_expert);
        StreamPtrs spc = sp;
        for (int i = 0; i < rb.count; ++i)
            spc.p[i] = static_cast<const char *>(sp.p[i]) + e0 * out_features * rb.b[i];
        void *dstc = static_cast<char *>(dst) + e0 * rows * n * elem;
        const int threads = 256;
        int64_t blocks = ((int64_t)total + threads - 1) / threads;
        const int64_t cap = (int64_t)num_sms * 8;  // resident blocks; grid-stride beyond
        if (blocks > cap) blocks = cap;
#define IQK_DQF(M, T, F)                                                              \
        if (M != IQK_IQ1_S_R4)                                                        \
            dequant_words_kernel<M, T, F><<<(unsigned)blocks, threads, 0, stream>>>(   \
                spc, total, log2_octs - 1, n, out_features, row_start, (uint32_t)rows, \
                static_cast<T *>(dstc));                                              \
        else                                                                          \
            dequant_iq1_kernel<T, F><<<(unsigned)blocks, threads, 0, stream>>>(        \
                spc, total, log2_octs - 1, n, out_features, row_start, (uint32_t)rows, \
                static_cast<T *>(dstc))
#define IQK_DQ(M, T)                                                   \
        do {                                                           \
            if (floor) { IQK_DQF(M, T, true); }                        \
            else { IQK_DQF(M, T, false); }                             \
        } while (0)
#define IQK_DQ_MEMBER(M)                                             \
    do {                                                             \
        if (out_dtype == IQK_F32) IQK_DQ(M, float);                  \
        else if (out_dtype == IQK_F16) IQK_DQ(M, __half);            \
        else IQK_DQ(M, __nv_bfloat16);                               \
    } while (0)
        if (member == IQK_IQ2_KS) IQK_DQ_MEMBER(IQK_IQ2_KS);
        else if (member == IQK_IQ2_K) IQK_DQ_MEMBER(IQK_IQ2_K);
        else IQK_DQ_MEMBER(IQK_IQ1_S_R4);
#undef IQK_DQ_MEMBER
#undef IQK_DQ
#undef IQK_DQF
        cudaError_t err = cudaGetLastError();
        if (err != cudaSuccess) return err;
    }
    return cudaSuccess;
}

}  // namespace iqk
