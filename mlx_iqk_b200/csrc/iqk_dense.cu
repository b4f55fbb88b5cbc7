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
// GEMV: f16 m16n8k16 MMAs whose A fragments (rows g and g + 8, two weights
// per register) come from lane-replicated value tables in shared memory; the
// tokens (up to 16 per pass, f16 as at the reference's call seam) are the N
// dimension; each sub-block's float32 partial sum is scaled by its dl into
// float32 accumulators, and the warps sharing a row tile's k range add their
// sums in a fixed order.
//   IQ4_KS / IQ4_K (dense_gemv_p4_kernel): one f16 pair per code byte from a
//     table at a fixed shared address, so one byte permute forms each lookup
//     address; one 16-warp CTA per SM.
//   IQ5_K / IQ6_K (dense_gemv_kernel): one f16 value per code (IQ6_K: an f16
//     pair hi + lo whose sum is the float32 value to 2^-22, through two MMAs);
//     persistent CTAs of 8 warps, two per SM.
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
    // one unit's inputs: its two code words, high bits and scale
    struct Unit {
        uint2 w;
        uint32_t hi;
        float dl;
        int base;
        int64_t lr;
        int u;
    };
    auto load = [&](int64_t i) {
        Unit U;
        U.lr = i / upr;
        U.u = (int)(i - U.lr * upr);
        const int64_t row = row_start + U.lr;
        int alpha;
        U.dl = sub_scale<M>(st, n, row, M == IQK_IQ4_KS ? U.u >> 1 : U.u, alpha);
        U.w = *reinterpret_cast<const uint2 *>(st.qs + row * (n / 8) + 2 * U.u);
        U.hi = unit_high<M>(st, n, row, U.u);
        U.base = alpha << DG::kW;
        return U;
    };
    auto emit = [&](const Unit &U) {
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            int c = (int)(((j < 8 ? U.w.x : U.w.y) >> (4 * (j & 7))) & 15u);
            if (M == IQK_IQ5_K) c |= (int)((U.hi >> j) & 1u) << 4;
            if (M == IQK_IQ6_K) c |= (int)((U.hi >> (2 * j)) & 3u) << 4;
            v[j] = __fmul_rn(U.dl, mytab[(U.base | c) * 32]);
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
        uint4 *wout = reinterpret_cast<uint4 *>(dst + U.lr * n + (int64_t)(U.u - lane) * 16);
#pragma unroll
        for (int c = 0; c < CH; ++c) __stcs(wout + 32 * c + lane, my_stage[32 * c + lane]);
        __syncwarp();
    };
    // total and stride are multiples of 32: every warp is all in or all out of
    // each unit; two units per pass, both units' loads issued before either
    // is decoded (twice the reads in flight)
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += 2 * stride) {
        const bool two = i + stride < total;
        const Unit a = load(i);
        Unit b{};
        if (two) b = load(i + stride);
        emit(a);
        if (two) emit(b);
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

constexpr int kDenseRows = 16;

// GEMV value table in shared memory, one copy per lane (entry e of lane l at
// word 32 e + l, so every lookup is conflict-free whatever the codes).
//   IQ4_KS / IQ4_K: pair entries, index alphabet << 8 | code byte: the f16
//     values of the byte's two weights (low nibble first), which is exactly
//     one A-fragment register.
//   IQ5_K / IQ6_K: single entries, index alphabet << W | code: the f16 value
//     in the low half (IQ6_K: the f16 residual of the float32 value in the
//     high half, for the second MMA).
template <int M> struct GemvTab {
    static constexpr bool kPair = M == IQK_IQ4_KS || M == IQK_IQ4_K;
    static constexpr int kEntries = kPair ? 512 : DenseGeo<M>::kEntries;
    static constexpr int kBytes = kEntries * 32 * 4;
};

template <int M> __device__ __forceinline__ uint32_t gemv_entry(int e) {
    if (GemvTab<M>::kPair) {
        const int a = e >> 8;
        const __half v0 = __float2half_rn(table_value(M, (a << 4) | (e & 15)));
        const __half v1 = __float2half_rn(table_value(M, (a << 4) | ((e >> 4) & 15)));
        return (uint32_t)__half_as_ushort(v0) | ((uint32_t)__half_as_ushort(v1) << 16);
    }
    const float v = table_value(M, e);
    const __half hi = __float2half_rn(v);
    const __half lo = M == IQK_IQ6_K ? __float2half_rn(v - __half2float(hi)) : __float2half_rn(0.f);
    return (uint32_t)__half_as_ushort(hi) | ((uint32_t)__half_as_ushort(lo) << 16);
}

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];\n" : "=r"(v) : "r"(a));
    return v;
}

__device__ __forceinline__ void cp_async(uint32_t dst, const void *src, int bytes) {
    if (bytes == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src));
    else if (bytes == 8)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(dst), "l"(src));
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(src));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds8(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u8 %0, [%1];\n" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u16 %0, [%1];\n" : "=r"(v) : "r"(a));
    return v;
}

// Geometry of the GEMV's staging. A CTA has 8 warps; KW of them (4, or 2 at
// in_features 1024) split one 16-row tile's k range, so a CTA iteration
// covers 8 / KW row tiles. Each warp streams its rows x k range in 64-weight
// steps through its own ring of D shared-memory slots (cp.async: code words,
// high bits), D - 1 steps ahead, and the scale bytes of its rows x k range
// per row tile through two buffers, issued with the tile's first step.
template <int M> struct DenseStage {
    static constexpr int kQs = 16 * 32;                                  // qs bytes per step
    static constexpr int kQh = M == IQK_IQ6_K ? 16 * 16 : M == IQK_IQ5_K ? 16 * 8 : 0;
    static constexpr int kSlot = kQs + kQh;
};
// scale bytes per row of each stream over a k range of kq weights
struct ScaleRows {
    int scl, sch, sex, dv;  // bytes per row
    int off_sch, off_sex, off_dv, total;  // region offsets in a buffer (16 rows each)
};
__host__ __device__ inline ScaleRows scale_rows(int member, int kq) {
    ScaleRows r{};
    if (member == IQK_IQ4_KS) {
        r.scl = kq / 32;
        r.dv = 0;  // the f32 row scale is read once per row tile
    } else {
        r.scl = member == IQK_IQ6_K ? kq / 16 : kq / 32;
        r.sch = (member == IQK_IQ4_K || member == IQK_IQ5_K) ? kq / 64 : 0;
        r.sex = kq / 128;
        r.dv = 2 * (kq / 256);
    }
    r.off_sch = 16 * r.scl;
    r.off_sex = r.off_sch + 16 * r.sch;
    r.off_dv = r.off_sex + 16 * r.sex;
    r.total = (r.off_dv + 16 * r.dv + 15) / 16 * 16;
    return r;
}

template <int M>
__host__ __device__ inline int dense_gemv_smem(int n, int D) {
    const int KW = n >= 2048 ? 4 : 2;
    const ScaleRows sr = scale_rows(M, n / KW);
    return GemvTab<M>::kBytes + 8 * (D * DenseStage<M>::kSlot + 2 * sr.total);
}

// NT token tiles of 8 per pass (tokens t0 .. t0 + 8 NT - 1); D ring slots.
template <int M, int NT, int D>
__global__ void __launch_bounds__(256, 2)
dense_gemv_kernel(DenseStreams st, int n, int out, const __half *__restrict__ x, int tokens,
                  void *__restrict__ y, int y_dtype) {
    using DG = DenseGeo<M>;
    using TB = GemvTab<M>;
    using SG = DenseStage<M>;
    extern __shared__ __align__(16) uint32_t dsm[];
    __shared__ float red[8][32][NT * 4];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int KW = n >= 2048 ? 4 : 2, RT = 8 / KW;
    const int rt = wid / KW, kw = wid % KW;  // this warp's row tile in the iteration, k part
    const int kq = n / KW, kbeg = kw * kq, steps = kq / 64;
    const ScaleRows sr = scale_rows(M, kq);
    for (int i = threadIdx.x; i < TB::kEntries * 32; i += blockDim.x) dsm[i] = gemv_entry<M>(i >> 5);
    const uint32_t smem0 = (uint32_t)__cvta_generic_to_shared(dsm);
    const uint32_t tab_u = smem0 + 4u * lane;
    const uint32_t ring = smem0 + TB::kBytes + (uint32_t)wid * (D * SG::kSlot + 2 * sr.total);
    const uint32_t scb = ring + D * SG::kSlot;  // two scale buffers
    __syncthreads();

    const int tiles = out / kDenseRows;
    const int groups = (tiles + RT - 1) / RT;  // row-tile groups: one per CTA iteration
    const int iters = (int)blockIdx.x < groups ? (groups - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int total = iters * steps;  // this warp's steps
    auto tile_of = [&](int it) { return ((int)blockIdx.x + it * (int)gridDim.x) * RT + rt; };
    // issue the copies of step f: its code words and high bits into slot f % D,
    // and at a row tile's first step that tile's scale bytes into buffer it & 1
    // (step f = it * steps + sidx; both walks below advance (it, sidx) by
    // one step at a time instead of dividing)
    auto issue = [&](int f, int it, int sidx) {
        const int tile = tile_of(it);
        if (tile >= tiles) return;
        const int64_t r0 = (int64_t)tile * kDenseRows;
        const int k0 = kbeg + 64 * sidx;
        const uint32_t slot = ring + (uint32_t)(f % D) * SG::kSlot;
        {
            const int row = lane >> 1, half = lane & 1;
            cp_async(slot + (uint32_t)(row * 32 + half * 16),
                     st.qs + (r0 + row) * (n / 8) + (k0 >> 3) + 4 * half, 16);
        }
        if (M == IQK_IQ5_K && lane < 16)
            cp_async(slot + SG::kQs + lane * 8, st.qh + (r0 + lane) * (n / 32) + (k0 >> 5), 8);
        if (M == IQK_IQ6_K && lane < 16)
            cp_async(slot + SG::kQs + lane * 16, st.qh + (r0 + lane) * (n / 16) + (k0 >> 4), 16);
        if (sidx == 0 && lane < 16) {
            const uint32_t b = scb + (uint32_t)(it & 1) * sr.total;
            const int64_t row = r0 + lane;
            auto piece = [&](uint32_t dst, const uint8_t *src, int bytes) {
                for (int o = 0; o < bytes; o += 16)
                    cp_async(dst + o, src + o, bytes - o >= 16 ? 16 : bytes - o);
            };
            if (M == IQK_IQ6_K)
                piece(b + lane * sr.scl, st.scl + row * (n / 16) + kbeg / 16, sr.scl);
            else
                piece(b + lane * sr.scl, st.scl + row * (n / 32) + kbeg / 32, sr.scl);
            if (sr.sch) piece(b + sr.off_sch + lane * sr.sch, st.sch + row * (n / 64) + kbeg / 64, sr.sch);
            if (sr.sex) piece(b + sr.off_sex + lane * sr.sex, st.sex + row * (n / 128) + kbeg / 128, sr.sex);
            if (sr.dv)
                piece(b + sr.off_dv + lane * sr.dv,
                      reinterpret_cast<const uint8_t *>(static_cast<const uint16_t *>(st.dv) + row * (n / 256) + kbeg / 256),
                      sr.dv);
        }
    };
    // dl of local sub-block `ls` of row `lr` (0..15) of the scale buffer `b`,
    // the alphabet bit in the lowest mantissa bit (at most one float32 ulp)
    auto scale_of = [&](uint32_t b, int lr, int ls, float drow) -> float {
        int index, alpha;
        float d;
        if (M == IQK_IQ4_KS) {
            const uint32_t v = lds8(b + lr * sr.scl + ls);
            index = (int)(v & 254u) - 127;
            alpha = (int)(v & 1u);
            d = drow;
        } else {
            if (M == IQK_IQ6_K) {
                index = (int)(int8_t)lds8(b + lr * sr.scl + ls);
            } else {
                const int lo = (int)((lds8(b + lr * sr.scl + (ls >> 1)) >> (4 * (ls & 1))) & 15u);
                const int hi = (int)((lds8(b + sr.off_sch + lr * sr.sch + (ls >> 2)) >> (2 * (ls & 3))) & 3u);
                index = (lo | (hi << 4)) - 32;
            }
            alpha = (int)((lds8(b + sr.off_sex + lr * sr.sex + (ls >> 3)) >> (ls & 7)) & 1u);
            d = __half2float(__ushort_as_half((unsigned short)lds16(b + sr.off_dv + lr * sr.dv + 2 * (ls >> 4))));
        }
        const float dl = __fmul_rn(d, (float)index);
        return __int_as_float((__float_as_int(dl) & ~1) | alpha);
    };
    // pairs: byte t of a word to bits 7..14 (entry index * 128 bytes) by one rotate
    const uint32_t prot = (uint32_t)(8 * t - 7) & 31u;
    constexpr uint32_t kAlphaShift = TB::kPair ? 15 : DG::kW + 7;

    for (int t0 = 0; t0 < tokens; t0 += 8 * NT) {
        const __half *xb[NT];
        bool xok[NT];
#pragma unroll
        for (int q = 0; q < NT; ++q) {
            const int tk = t0 + 8 * q + g;
            xok[q] = tk < tokens;
            xb[q] = x + (int64_t)(xok[q] ? tk : 0) * n + 2 * t;
        }
        float acc[NT][4];
#pragma unroll
        for (int q = 0; q < NT; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
        // prologue: D - 1 steps in flight
        int iit = 0, isidx = 0;  // the issue walk: the next step to copy
#pragma unroll 1
        for (int f = 0; f < D - 1; ++f) {
            if (f < total) issue(f, iit, isidx);
            cp_async_commit();
            if (++isidx == steps) {
                isidx = 0;
                ++iit;
            }
        }
        float dra = 0.f, drb = 0.f;
        int it = 0, sidx = -1;  // the compute walk
#pragma unroll 1
        for (int f = 0; f < total; ++f) {
            if (++sidx == steps) {
                sidx = 0;
                ++it;
            }
            const int tile = tile_of(it);
            const bool live = tile < tiles;
            const int64_t ra = (int64_t)tile * kDenseRows + g, rb = ra + 8;
            // the slot of step f - 1 is free again: refill it with step f + D - 1
            __syncwarp();
            if (f + D - 1 < total) issue(f + D - 1, iit, isidx);
            cp_async_commit();
            if (++isidx == steps) {
                isidx = 0;
                ++iit;
            }
            cp_async_wait<D - 1>();
            __syncwarp();
            if (live) {
                if (M == IQK_IQ4_KS && sidx == 0) {
                    dra = __ldg(static_cast<const float *>(st.dv) + ra);
                    drb = __ldg(static_cast<const float *>(st.dv) + rb);
                }
                const uint32_t slot = ring + (uint32_t)(f % D) * SG::kSlot;
                const uint32_t b = scb + (uint32_t)(it & 1) * sr.total;
                const int ls = M == IQK_IQ4_KS ? 2 * sidx + (t >> 1) : 4 * sidx + t;
                const float dla_m = scale_of(b, g, ls, dra);
                const float dlb_m = scale_of(b, g + 8, ls, drb);
                const uint4 qa0 = lds128(slot + g * 32), qa1 = lds128(slot + g * 32 + 16);
                const uint4 qb0 = lds128(slot + (g + 8) * 32), qb1 = lds128(slot + (g + 8) * 32 + 16);
                uint4 ha = make_uint4(0, 0, 0, 0), hb = make_uint4(0, 0, 0, 0);
                if (M == IQK_IQ5_K) {
                    const uint32_t h = slot + SG::kQs;
                    ha.x = lds32(h + g * 8);
                    ha.y = lds32(h + g * 8 + 4);
                    hb.x = lds32(h + (g + 8) * 8);
                    hb.y = lds32(h + (g + 8) * 8 + 4);
                }
                if (M == IQK_IQ6_K) {
                    ha = lds128(slot + SG::kQs + g * 16);
                    hb = lds128(slot + SG::kQs + (g + 8) * 16);
                }
                const int k0 = kbeg + 64 * sidx;
#pragma unroll
                for (int tt = 0; tt < 4; ++tt) {
                    const float dla = __shfl_sync(0xffffffffu, dla_m, (lane & ~3) | tt);
                    const float dlb = __shfl_sync(0xffffffffu, dlb_m, (lane & ~3) | tt);
                    const uint32_t offa = tab_u + (((uint32_t)__float_as_int(dla) & 1u) << kAlphaShift);
                    const uint32_t offb = tab_u + (((uint32_t)__float_as_int(dlb) & 1u) << kAlphaShift);
                    const uint4 &qa4 = tt < 2 ? qa0 : qa1;
                    const uint4 &qb4 = tt < 2 ? qb0 : qb1;
                    const uint32_t w0a = (tt & 1) ? qa4.z : qa4.x, w1a = (tt & 1) ? qa4.w : qa4.y;
                    const uint32_t w0b = (tt & 1) ? qb4.z : qb4.x, w1b = (tt & 1) ? qb4.w : qb4.y;
                    uint32_t A[4], L[4];
                    if (TB::kPair) {
                        A[0] = lds32(offa + (__funnelshift_r(w0a, w0a, prot) & 0x7f80u));
                        A[1] = lds32(offb + (__funnelshift_r(w0b, w0b, prot) & 0x7f80u));
                        A[2] = lds32(offa + (__funnelshift_r(w1a, w1a, prot) & 0x7f80u));
                        A[3] = lds32(offb + (__funnelshift_r(w1b, w1b, prot) & 0x7f80u));
                    } else {
                        // single entries: weights 16 tt + {2t, 2t+1, 8+2t, 9+2t} of the step
                        uint32_t e[2][4];
#pragma unroll
                        for (int r = 0; r < 2; ++r) {
                            const uint32_t w0 = r ? w0b : w0a, w1 = r ? w1b : w1a;
                            const uint4 &h4 = r ? hb : ha;
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const uint32_t w = i < 2 ? w0 : w1;
                                const int kk = 16 * tt + 2 * t + (i & 1) + 8 * (i >> 1);
                                uint32_t c = (w >> (4 * (2 * t + (i & 1)))) & 15u;
                                if (M == IQK_IQ5_K) {
                                    const uint32_t hw = kk < 32 ? h4.x : h4.y;
                                    c |= ((hw >> (kk & 31)) & 1u) << 4;
                                } else {
                                    const uint32_t hw = (kk >> 4) == 0 ? h4.x : (kk >> 4) == 1 ? h4.y
                                                        : (kk >> 4) == 2 ? h4.z : h4.w;
                                    c |= ((hw >> (2 * (kk & 15))) & 3u) << 4;
                                }
                                e[r][i] = lds32((r ? offb : offa) + (c << 7));
                            }
                        }
                        A[0] = __byte_perm(e[0][0], e[0][1], 0x5410);
                        A[1] = __byte_perm(e[1][0], e[1][1], 0x5410);
                        A[2] = __byte_perm(e[0][2], e[0][3], 0x5410);
                        A[3] = __byte_perm(e[1][2], e[1][3], 0x5410);
                        if (M == IQK_IQ6_K) {
                            L[0] = __byte_perm(e[0][0], e[0][1], 0x7632);
                            L[1] = __byte_perm(e[1][0], e[1][1], 0x7632);
                            L[2] = __byte_perm(e[0][2], e[0][3], 0x7632);
                            L[3] = __byte_perm(e[1][2], e[1][3], 0x7632);
                        }
                    }
                    const int kx = k0 + 16 * tt;
#pragma unroll
                    for (int q = 0; q < NT; ++q) {
                        const uint32_t b0 = xok[q] ? __ldg(reinterpret_cast<const unsigned int *>(xb[q] + kx)) : 0u;
                        const uint32_t b1 = xok[q] ? __ldg(reinterpret_cast<const unsigned int *>(xb[q] + kx + 8)) : 0u;
                        float d[4];
                        mma_f16(d, A, b0, b1);
                        if (M == IQK_IQ6_K) mma_f16_acc(d, L, b0, b1);
                        acc[q][0] = fmaf(dla, d[0], acc[q][0]);
                        acc[q][1] = fmaf(dla, d[1], acc[q][1]);
                        acc[q][2] = fmaf(dlb, d[2], acc[q][2]);
                        acc[q][3] = fmaf(dlb, d[3], acc[q][3]);
                    }
                }
            }
            if (sidx + 1 < steps) continue;
            // end of the iteration's row tiles: each tile's KW k parts meet in
            // its first warp, added in k order
            if (kw > 0) {
#pragma unroll
                for (int q = 0; q < NT; ++q)
#pragma unroll
                    for (int i = 0; i < 4; ++i) red[wid][lane][q * 4 + i] = acc[q][i];
            }
            __syncthreads();
            if (kw == 0 && live) {
                for (int w = 1; w < KW; ++w)
#pragma unroll
                    for (int q = 0; q < NT; ++q)
#pragma unroll
                        for (int i = 0; i < 4; ++i) acc[q][i] += red[wid + w][lane][q * 4 + i];
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
#pragma unroll
            for (int q = 0; q < NT; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
        }
        cp_async_wait<0>();
        __syncthreads();
    }
}

// ---- IQ4 members: the pair table at a fixed shared-window address.
//
// IQ4_KS and IQ4_K look up one f16 pair per code byte. With the table's
// 64 KB at shared address 64 KB, entry (code byte c, alphabet a) of lane l
// sits at 64 KB | c << 8 | a << 7 | l << 2, so one byte permute of the code
// word with a per-lane base word forms each lookup address. That fixes the
// CTA: one per SM, 16 warps, the code rings below 64 KB, the table at
// [64 KB, 128 KB), the scale buffers and the k-part reduction area above.
//
// Each warp walks 16-row tiles over 1024 weights of k (KW = n / 1024 warps
// share a tile, RT = 16 / KW tiles per CTA iteration) in 64-weight steps. In
// one MMA a lane takes two code bytes of a row, so the MMA's logical k pairs
// (2t, 2t+1) and (2t+8, 2t+9) map to four consecutive weights of the step:
//   IQ4_KS  MMA (s, m) of 32-weight sub-block s: bytes 2m, 2m+1 of word
//           4s + t, weights 32s + 8t + 4m .. + 3 (two MMAs per scale);
//   IQ4_K   MMA s of 16-weight sub-block s: bytes 2(t&1), 2(t&1)+1 of word
//           2s + (t>>1), weights 16s + 4t .. + 3 (one MMA per scale);
// so a lane's activation fragment is one 8-byte load.
constexpr uint32_t kPairTab = 65536;  // shared-window address of the pair table
constexpr int kP4Warps = 16;
constexpr int kP4Steps = 16;  // 64-weight steps of a warp's 1024-weight k part

template <int M, int NT> __host__ __device__ inline int p4_tail_bytes(int n) {
    const ScaleRows sr = scale_rows(M, 1024);
    return kP4Warps * 2 * sr.total + (n > 1024 ? 2 * kP4Warps * 32 * NT * 16 : 0);
}

__device__ __forceinline__ void sts32(uint32_t a, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;\n" ::"r"(a), "r"(v));
}
__device__ __forceinline__ void sts128(uint32_t a, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};\n" ::"r"(a), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w));
}
__device__ __forceinline__ float4 lds128f(uint32_t a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];\n"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ void bar_tile(int id, int threads) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(threads) : "memory");
}
// the lookup address of code byte j of word w: 64 KB | byte << 8 | base byte 0
__device__ __forceinline__ uint32_t pair_addr(uint32_t w, uint32_t base, uint32_t sel) {
    return __byte_perm(w, base, sel);
}

// XS: the pass's activation rows are staged in shared memory after the tail
// (when they fit), so the fragment loads are shared-memory broadcasts.
template <int M, int NT, int D, bool XS>
__global__ void __launch_bounds__(kP4Warps * 32, 1)
dense_gemv_p4_kernel(DenseStreams st, int n, int out, const __half *__restrict__ x, int tokens,
                     void *__restrict__ y, int y_dtype) {
    static_assert(M == IQK_IQ4_KS || M == IQK_IQ4_K, "pair-table members only");
    extern __shared__ __align__(128) uint8_t p4sm[];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int KW = n >> 10, RT = kP4Warps / KW;
    const int rt = wid / KW, kw = wid % KW;
    const int kbeg = kw * 1024;
    const ScaleRows sr = scale_rows(M, 1024);
    const uint32_t s0 = (uint32_t)__cvta_generic_to_shared(p4sm);
    uint32_t dyn;
    asm("mov.u32 %0, %%dynamic_smem_size;\n" : "=r"(dyn));
    const uint32_t ring0 = (s0 + 127u) & ~127u;
    const uint32_t tail = kPairTab + 65536u;
    // the rings must end below the table and the tail lie inside the
    // allocation (the host sizes it so); otherwise the outputs are NaN
    if (ring0 + (uint32_t)(kP4Warps * D * 512) > kPairTab ||
        s0 + dyn < tail + (uint32_t)p4_tail_bytes<M, NT>(n) +
                       (XS ? (uint32_t)(min(tokens, 8 * NT) * n * 2) : 0u)) {
        const int64_t total = (int64_t)tokens * out;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
             i += (int64_t)gridDim.x * blockDim.x) {
            if (y_dtype == IQK_F32) static_cast<float *>(y)[i] = __int_as_float(0x7fc00000);
            else static_cast<__half *>(y)[i] = __ushort_as_half((unsigned short)0x7e00u);
        }
        return;
    }
    // the table: word i is entry (code byte i >> 6, alphabet (i >> 5) & 1), lane i & 31
    for (int i = threadIdx.x; i < 16384; i += kP4Warps * 32) {
        const int c = i >> 6, a = (i >> 5) & 1;
        const __half v0 = __float2half_rn((float)c_iq4k[(a << 4) | (c & 15)]);
        const __half v1 = __float2half_rn((float)c_iq4k[(a << 4) | (c >> 4)]);
        sts32(kPairTab + 4u * (uint32_t)i,
              (uint32_t)__half_as_ushort(v0) | ((uint32_t)__half_as_ushort(v1) << 16));
    }
    const uint32_t ring = ring0 + (uint32_t)wid * (D * 512);
    const uint32_t scb = tail + (uint32_t)wid * 2 * sr.total;  // two scale buffers
    const uint32_t red0 = tail + (uint32_t)(kP4Warps * 2 * sr.total);
    const uint32_t lbase = kPairTab | ((uint32_t)lane << 2);
    // code words of rows g, g+8 in a slot: row r's 16-byte halves swapped when
    // (r >> 2) is odd, so the eight rows a load touches fall in distinct banks
    const uint32_t sw = (uint32_t)((g >> 2) & 1);
    __syncthreads();

    const int tiles = out / kDenseRows;
    const int groups = (tiles + RT - 1) / RT;
    const int iters = (int)blockIdx.x < groups ? (groups - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int total = iters * kP4Steps;
    auto tile_of = [&](int it) { return ((int)blockIdx.x + it * (int)gridDim.x) * RT + rt; };
    // Copy walk: the next step to issue, this lane's 16-byte source and the
    // ring slot, advanced one step at a time (a tile's first step recomputes
    // the row pointer and sends the tile's scale bytes to buffer it & 1).
    const uint32_t dsto = (uint32_t)((lane >> 1) * 32 + (((lane & 1) ^ ((lane >> 3) & 1)) * 16));
    int iit = 0, isidx = 0, ileft = 0, islot = 0;
    const uint32_t *iq = st.qs;
    auto issue_next = [&]() {
        if (ileft > 0) {
            --ileft;
            const int tile = tile_of(iit);
            if (tile < tiles) {
                if (isidx == 0) {
                    const int64_t r0 = (int64_t)tile * kDenseRows;
                    iq = st.qs + (r0 + (lane >> 1)) * (n / 8) + (kbeg >> 3) + 4 * (lane & 1);
                    if (lane < 16) {
                        const uint32_t b = scb + (uint32_t)(iit & 1) * sr.total;
                        const int64_t row = r0 + lane;
                        auto piece = [&](uint32_t dst, const uint8_t *src, int bytes) {
                            for (int o = 0; o < bytes; o += 16)
                                cp_async(dst + o, src + o, bytes - o >= 16 ? 16 : bytes - o);
                        };
                        piece(b + lane * sr.scl, st.scl + row * (n / 32) + kbeg / 32, sr.scl);
                        if (M == IQK_IQ4_K) {
                            piece(b + sr.off_sch + lane * sr.sch, st.sch + row * (n / 64) + kbeg / 64, sr.sch);
                            piece(b + sr.off_sex + lane * sr.sex, st.sex + row * (n / 128) + kbeg / 128, sr.sex);
                            piece(b + sr.off_dv + lane * sr.dv,
                                  reinterpret_cast<const uint8_t *>(static_cast<const uint16_t *>(st.dv) +
                                                                    row * (n / 256) + kbeg / 256),
                                  sr.dv);
                        }
                    }
                }
                cp_async(ring + (uint32_t)islot * 512u + dsto, iq, 16);
                iq += 8;  // the row's next 64 codes
            }
            if (++isidx == kP4Steps) {
                isidx = 0;
                ++iit;
            }
        }
        cp_async_commit();
        islot = islot + 1 == D ? 0 : islot + 1;
    };

    const uint32_t xsm = tail + (uint32_t)p4_tail_bytes<M, NT>(n);  // XS: staged rows
    for (int t0 = 0; t0 < tokens; t0 += 8 * NT) {
        if (XS) {
            // this pass's rows t0 .. t0 + rows - 1, contiguous as in x
            const int rows = min(8 * NT, tokens - t0);
            const uint4 *src = reinterpret_cast<const uint4 *>(x + (int64_t)t0 * n);
            for (int i = threadIdx.x; i < rows * n / 8; i += kP4Warps * 32) {
                const uint4 v = __ldg(src + i);
                asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(xsm + 16u * (uint32_t)i),
                             "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w));
            }
            __syncthreads();
        }
        // B column g of token tile q: token t0 + 8q + g (clamped: columns
        // past the last token are computed and never stored)
        const __half *xq[NT];
        uint32_t xs[NT];
#pragma unroll
        for (int q = 0; q < NT; ++q) {
            const int tk = min(t0 + 8 * q + g, tokens - 1);
            const int kk = kbeg + (M == IQK_IQ4_KS ? 8 * t : 4 * t);
            xq[q] = x + (int64_t)tk * n + kk;
            xs[q] = xsm + 2u * (uint32_t)((tk - t0) * n + kk);
        }
        float acc[NT][4];
#pragma unroll
        for (int q = 0; q < NT; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
        iit = 0;
        isidx = 0;
        ileft = total;
        islot = 0;
        // D - 2 steps in flight ahead of the pair of steps being computed
#pragma unroll 1
        for (int f = 0; f < D - 2; ++f) issue_next();
        float drow = 0.f;  // IQ4_KS: the row scale of row lane & 15
        int it = 0, sidx = 0, cslot = 0;
        const int lr = lane & 15, hs = lane >> 4;  // scale lane: row, sub-block parity
#pragma unroll 1
        for (int f = 0; f < total; f += 2) {
            const int tile = tile_of(it);
            const bool live = tile < tiles;
            const int64_t r0 = (int64_t)tile * kDenseRows;
            // the slots of steps f - 2, f - 1 are free again
            __syncwarp();
            issue_next();
            issue_next();
            cp_async_wait<D - 2>();
            __syncwarp();
            if (live) {
                const uint32_t b = scb + (uint32_t)(it & 1) * sr.total;
                if (M == IQK_IQ4_KS) {
                    if (sidx == 0) drow = __ldg(static_cast<const float *>(st.dv) + r0 + lr);
                    // scale bytes of sub-blocks 2 sidx .. 2 sidx + 3 (this pair of steps)
                    const uint32_t v4 = lds32(b + lr * sr.scl + 2 * sidx);
                    // both steps' code words first: rows g, g + 8, words t and 4 + t
                    uint32_t wa[2][2], wb[2][2];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t ra = ring + (uint32_t)cslot * 512u + (uint32_t)g * 32u + 4u * (uint32_t)t;
                        cslot = cslot + 1 == D ? 0 : cslot + 1;
                        wa[h][0] = lds32(ra + 16u * sw);
                        wa[h][1] = lds32(ra + 16u * (sw ^ 1u));
                        wb[h][0] = lds32(ra + 256u + 16u * sw);
                        wb[h][1] = lds32(ra + 256u + 16u * (sw ^ 1u));
                    }
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int kx = 64 * (sidx + h);
                        // dl of (row lr, sub-block hs), alphabet bit in the lowest mantissa bit
                        const uint32_t v = (v4 >> (8 * (2 * h + hs))) & 255u;
                        const float dl = __fmul_rn(drow, (float)((int)(v & 254u) - 127));
                        const float dm = __int_as_float((__float_as_int(dl) & ~1) | (int)(v & 1u));
#pragma unroll
                        for (int s = 0; s < 2; ++s) {
                            const float dla = __shfl_sync(0xffffffffu, dm, 16 * s + g);
                            const float dlb = __shfl_sync(0xffffffffu, dm, 16 * s + 8 + g);
                            const uint32_t la = lbase | (((uint32_t)__float_as_int(dla) & 1u) << 7);
                            const uint32_t lb = lbase | (((uint32_t)__float_as_int(dlb) & 1u) << 7);
                            uint4 bx[NT];
#pragma unroll
                            for (int q = 0; q < NT; ++q)
                                bx[q] = XS ? lds128(xs[q] + 2u * (uint32_t)(kx + 32 * s))
                                           : __ldg(reinterpret_cast<const uint4 *>(xq[q] + kx + 32 * s));
                            float d[NT][4];
#pragma unroll
                            for (int m = 0; m < 2; ++m) {
                                uint32_t A[4];
                                A[0] = lds32(pair_addr(wa[h][s], la, 0x7604u | (2u * m) << 4));
                                A[1] = lds32(pair_addr(wb[h][s], lb, 0x7604u | (2u * m) << 4));
                                A[2] = lds32(pair_addr(wa[h][s], la, 0x7604u | (2u * m + 1u) << 4));
                                A[3] = lds32(pair_addr(wb[h][s], lb, 0x7604u | (2u * m + 1u) << 4));
#pragma unroll
                                for (int q = 0; q < NT; ++q) {
                                    if (m == 0) {
                                        d[q][0] = d[q][1] = d[q][2] = d[q][3] = 0.f;
                                        mma_f16(d[q], A, bx[q].x, bx[q].y);
                                    } else {
                                        mma_f16_acc(d[q], A, bx[q].z, bx[q].w);
                                    }
                                }
                            }
#pragma unroll
                            for (int q = 0; q < NT; ++q) {
                                acc[q][0] = fmaf(dla, d[q][0], acc[q][0]);
                                acc[q][1] = fmaf(dla, d[q][1], acc[q][1]);
                                acc[q][2] = fmaf(dlb, d[q][2], acc[q][2]);
                                acc[q][3] = fmaf(dlb, d[q][3], acc[q][3]);
                            }
                        }
                    }
                } else {
                    // scale parts of sub-blocks 4 sidx .. 4 sidx + 7 (this pair of steps)
                    const uint32_t lo4 = lds32(b + lr * sr.scl + 2 * sidx);
                    const uint32_t hi2 = lds16(b + sr.off_sch + lr * sr.sch + sidx);
                    const uint32_t ex = lds8(b + sr.off_sex + lr * sr.sex + (sidx >> 1));
                    const float d0 = __half2float(__ushort_as_half(
                        (unsigned short)lds16(b + sr.off_dv + lr * sr.dv + 2 * (sidx >> 2))));
                    // both steps' code words first: word 2s + (t >> 1) of rows g, g + 8
                    uint32_t wa[2][4], wb[2][4];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t ra = ring + (uint32_t)cslot * 512u + (uint32_t)g * 32u + 4u * (uint32_t)(t >> 1);
                        cslot = cslot + 1 == D ? 0 : cslot + 1;
#pragma unroll
                        for (int s = 0; s < 4; ++s) {
                            const uint32_t wo = 16u * ((uint32_t)(s >> 1) ^ sw) + 8u * (uint32_t)(s & 1);
                            wa[h][s] = lds32(ra + wo);
                            wb[h][s] = lds32(ra + 256u + wo);
                        }
                    }
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const int kx = 64 * (sidx + h);
                        // dl of (row lr, sub-blocks hs and 2 + hs of step h)
                        float dm[2];
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            const int ls = 4 * h + 2 * u + hs;  // sub-block of the pair of steps
                            const int idx = (int)(((lo4 >> (4 * ls)) & 15u) | (((hi2 >> (2 * ls)) & 3u) << 4)) - 32;
                            const float dl = __fmul_rn(d0, (float)idx);
                            dm[u] = __int_as_float((__float_as_int(dl) & ~1) | (int)((ex >> ls) & 1u));
                        }
                        const uint32_t sel0 = 0x7604u | ((uint32_t)(2 * (t & 1)) << 4);
                        const uint32_t sel1 = sel0 + 0x10u;
#pragma unroll
                        for (int s = 0; s < 4; ++s) {
                            const float dla = __shfl_sync(0xffffffffu, dm[s >> 1], 16 * (s & 1) + g);
                            const float dlb = __shfl_sync(0xffffffffu, dm[s >> 1], 16 * (s & 1) + 8 + g);
                            const uint32_t la = lbase | (((uint32_t)__float_as_int(dla) & 1u) << 7);
                            const uint32_t lb = lbase | (((uint32_t)__float_as_int(dlb) & 1u) << 7);
                            uint32_t A[4];
                            A[0] = lds32(pair_addr(wa[h][s], la, sel0));
                            A[1] = lds32(pair_addr(wb[h][s], lb, sel0));
                            A[2] = lds32(pair_addr(wa[h][s], la, sel1));
                            A[3] = lds32(pair_addr(wb[h][s], lb, sel1));
#pragma unroll
                            for (int q = 0; q < NT; ++q) {
                                const uint2 bx = XS ? lds64(xs[q] + 2u * (uint32_t)(kx + 16 * s))
                                                    : __ldg(reinterpret_cast<const uint2 *>(xq[q] + kx + 16 * s));
                                float d[4] = {0.f, 0.f, 0.f, 0.f};
                                mma_f16(d, A, bx.x, bx.y);
                                acc[q][0] = fmaf(dla, d[0], acc[q][0]);
                                acc[q][1] = fmaf(dla, d[1], acc[q][1]);
                                acc[q][2] = fmaf(dlb, d[2], acc[q][2]);
                                acc[q][3] = fmaf(dlb, d[3], acc[q][3]);
                            }
                        }
                    }
                }
            } else {
                cslot = cslot + 2 >= D ? cslot + 2 - D : cslot + 2;
            }
            sidx += 2;
            if (sidx < kP4Steps) continue;
            sidx = 0;
            // end of the iteration's row tiles: each tile's KW k parts meet in
            // its first warp, added in k order (reduction area by iteration
            // parity, so one barrier per iteration suffices)
            if (KW > 1) {
                const uint32_t rp = red0 + (uint32_t)((it & 1) * kP4Warps) * (32u * NT * 16u);
                if (kw > 0) {
#pragma unroll
                    for (int q = 0; q < NT; ++q)
                        sts128(rp + ((uint32_t)wid * 32u + lane) * (NT * 16u) + 16u * q,
                               make_float4(acc[q][0], acc[q][1], acc[q][2], acc[q][3]));
                }
                bar_tile(1 + rt, KW * 32);
                if (kw == 0 && live) {
                    for (int w = 1; w < KW; ++w) {
#pragma unroll
                        for (int q = 0; q < NT; ++q) {
                            const float4 v = lds128f(rp + ((uint32_t)(wid + w) * 32u + lane) * (NT * 16u) + 16u * q);
                            acc[q][0] += v.x;
                            acc[q][1] += v.y;
                            acc[q][2] += v.z;
                            acc[q][3] += v.w;
                        }
                    }
                }
            }
            if (kw == 0 && live) {
                // D fragment: d0 = (row g, token 2t), d1 = (row g, 2t+1), d2/d3 rows g+8
#pragma unroll
                for (int q = 0; q < NT; ++q) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int tk = t0 + 8 * q + 2 * t + (i & 1);
                        const int64_t row = r0 + g + (i < 2 ? 0 : 8);
                        if (tk < tokens) {
                            const int64_t o = (int64_t)tk * out + row;
                            if (y_dtype == IQK_F32) static_cast<float *>(y)[o] = acc[q][i];
                            else static_cast<__half *>(y)[o] = __float2half_rn(acc[q][i]);
                        }
                    }
                }
            }
#pragma unroll
            for (int q = 0; q < NT; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.f;
            ++it;
        }
        cp_async_wait<0>();
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

template <int M, int NT, int D>
cudaError_t gemv_launch(const DenseStreams &st, int n, int out, const __half *xh, int tokens,
                        void *y, int y_dtype, cudaStream_t stream, int dev) {
    const int smem = dense_gemv_smem<M>(n, D);
    // per (device, n) shared-memory opt-in and resident CTAs, queried once
    static int per_sm[64][4] = {};
    const int wi = n == 1024 ? 0 : n == 2048 ? 1 : n == 4096 ? 2 : 3;
    int &ps = per_sm[dev & 63][wi];
    if (ps == 0) {
        cudaError_t e = cudaFuncSetAttribute(dense_gemv_kernel<M, NT, D>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        int nb = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, dense_gemv_kernel<M, NT, D>, 256, smem);
        if (e != cudaSuccess) return e;
        ps = nb > 0 ? nb : 1;
    }
    int sms = 148;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
    const int RT = n >= 2048 ? 2 : 4;
    const int groups = (out / kDenseRows + RT - 1) / RT;
    const int grid = groups < sms * ps ? groups : sms * ps;
    dense_gemv_kernel<M, NT, D><<<grid, 256, smem, stream>>>(st, n, out, xh, tokens, y, y_dtype);
    return cudaGetLastError();
}

template <int M, int NT>
cudaError_t p4_launch(const DenseStreams &st, int n, int out, const __half *xh, int tokens,
                      void *y, int y_dtype, cudaStream_t stream, int dev) {
    constexpr int D = 7;  // ring slots a warp: 16 x 7 x 512 B end below the table
    // per device: the shared memory reserved below a CTA's own (+1; 0 = not
    // yet queried), which places the dynamic allocation in the window
    static int reserved[64] = {}, optin[64] = {};
    int &rs = reserved[dev & 63];
    if (rs == 0) {
        int v = 0, o = 0;
        cudaError_t e = cudaDeviceGetAttribute(&v, cudaDevAttrReservedSharedMemoryPerBlock, dev);
        if (e != cudaSuccess) return e;
        e = cudaDeviceGetAttribute(&o, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(dense_gemv_p4_kernel<M, NT, D, false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(kPairTab + 65536u) + p4_tail_bytes<M, NT>(8192) - v);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(dense_gemv_p4_kernel<M, NT, D, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, o);
        if (e != cudaSuccess) return e;
        optin[dev & 63] = o;
        rs = v + 1;
    }
    const int smem = (int)(kPairTab + 65536u) + p4_tail_bytes<M, NT>(n) - (rs - 1);
    // stage the activation rows when they fit in the opt-in shared memory
    const int xs_bytes = (tokens < 8 * NT ? tokens : 8 * NT) * n * 2;
    const bool xs = smem + xs_bytes <= optin[dev & 63];
    int sms = 148;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
    const int RT = kP4Warps / (n >> 10);
    const int groups = (out / kDenseRows + RT - 1) / RT;
    const int grid = groups < sms ? groups : sms;
    if (xs)
        dense_gemv_p4_kernel<M, NT, D, true><<<grid, kP4Warps * 32, smem + xs_bytes, stream>>>(
            st, n, out, xh, tokens, y, y_dtype);
    else
        dense_gemv_p4_kernel<M, NT, D, false><<<grid, kP4Warps * 32, smem, stream>>>(
            st, n, out, xh, tokens, y, y_dtype);
    return cudaGetLastError();
}

template <int M>
cudaError_t gemv_m(const void *const *s, int n, int out, const void *x, int tokens, void *y,
                   int y_dtype, cudaStream_t stream) {
    const DenseStreams st = dense_streams<M>(s);
    const __half *xh = static_cast<const __half *>(x);
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = 0;
    if constexpr (M == IQK_IQ4_KS || M == IQK_IQ4_K) {
        return tokens <= 8 ? p4_launch<M, 1>(st, n, out, xh, tokens, y, y_dtype, stream, dev)
                           : p4_launch<M, 2>(st, n, out, xh, tokens, y, y_dtype, stream, dev);
    } else {
        // the deepest ring (8, 6 or 4 slots a warp) at which two CTAs still fit
        // on an SM (228 KB: the dynamic part, the 8 KB reduction buffer, 1 KB
        // reserved per CTA)
        constexpr int kBudget = 104 * 1024;
        const int D = dense_gemv_smem<M>(n, 8) <= kBudget ? 8 : dense_gemv_smem<M>(n, 6) <= kBudget ? 6 : 4;
#define IQK_DG(NT_, D_) gemv_launch<M, NT_, D_>(st, n, out, xh, tokens, y, y_dtype, stream, dev)
        if (tokens <= 8) return D == 8 ? IQK_DG(1, 8) : D == 6 ? IQK_DG(1, 6) : IQK_DG(1, 4);
        return D == 8 ? IQK_DG(2, 8) : D == 6 ? IQK_DG(2, 6) : IQK_DG(2, 4);
#undef IQK_DG
    }
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
