// Shared device helpers for the IQ_K routed-expert kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/iqk_b200.h"

namespace iqk {

// iq2nl_values (base alphabet 0..3, shifted alphabet 4..7) as int8 bytes:
// T0 = {-31, -13, 1, 17}, T1 = {-26, -8, 6, 22}, little-endian in one word so
// a byte permute indexes them directly.
constexpr uint32_t kIq2Tab0 = 0x1101F3E1u;
constexpr uint32_t kIq2Tab1 = 0x1606F8E6u;
// IQ1_S grid positions decode to {-1, 0, +1}: bytes {0xFF, 0x00, 0x01, 0x00}.
constexpr uint32_t kTernTab = 0x000100FFu;

__host__ __device__ constexpr int sub_weights(int member) {
    return member == IQK_IQ2_K ? 16 : 32;
}

// Bytes of each relayout stream per row, in component order
// (src/mlx_iqk/format.py:352-377). Unused slots are 0.
struct RowBytes {
    int64_t b[5];
    int count;
};

__host__ __device__ inline RowBytes row_bytes(int member, int64_t n) {
    RowBytes r{};
    if (member == IQK_IQ2_KS) {
        r.b[0] = n / 4;   // qs  u32[n/16]
        r.b[1] = n / 64;  // scl u8[n/64]
        r.b[2] = n / 256; // sch u8[n/256]
        r.b[3] = n / 256; // sex u8[n/256]
        r.b[4] = 2;       // dv  f16[1]
        r.count = 5;
    } else if (member == IQK_IQ2_K) {
        r.b[0] = n / 4;        // qs  u32[n/16]
        r.b[1] = n / 32;       // scl u8[n/32]
        r.b[2] = n / 128;      // sex u8[n/128]
        r.b[3] = 2 * (n / 256);// dv  f16[n/256]
        r.count = 4;
    } else {
        r.b[0] = n / 8;        // qs u32[n/32]
        r.b[1] = n / 16;       // qh u16[n/32]
        r.b[2] = 2;            // dv f16[1]
        r.count = 3;
    }
    return r;
}

__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

template <typename T> __device__ __forceinline__ float to_float(T v);
template <> __device__ __forceinline__ float to_float<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_float<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_float<__nv_bfloat16>(__nv_bfloat16 v) {
    return __bfloat162float(v);
}

template <typename T> __device__ __forceinline__ T from_float(float v);
template <> __device__ __forceinline__ float from_float<float>(float v) { return v; }
template <> __device__ __forceinline__ __half from_float<__half>(float v) { return __float2half_rn(v); }
template <> __device__ __forceinline__ __nv_bfloat16 from_float<__nv_bfloat16>(float v) {
    return __float2bfloat16_rn(v);
}

}  // namespace iqk
