// On-device relayout: ik wire rows -> the k-contiguous streams the kernels read.
//
// Reference: format.pack (src/mlx_iqk/format.py:449-588, 612-678), a numpy
// pass on the host at load time. Here one launch does the same re-placement of
// bits on the GPU, so a layer's wire can be uploaded as it is stored and
// converted where it will be served. Pure byte work, HBM-bound: every wire
// byte is read once and every stream byte written once.
//
// Wire layouts (ggml rows; vendor/ik_llama block structs):
//   IQ2_KS   row = dv f16 | per 256 weights: extra_lo u8 (alphabet bits),
//            extra_hi u8 (scale high bits), scales u8[4] (nibbles), qs u8[64]
//   IQ2_K    per 256 weights: d f16 | extra u16 (alphabet bits) |
//            scales u8[8] (nibbles) | qs u8[64]
//   IQ1_S_R4 groups of 4 rows: d f16[4] | per 32 weights: qs u8[16] (byte
//            4i + k: sub-group i of row k), qh u16[4] (row k's block word)
// Code order inside qs (iqk_iq2.cpp:512-558): weight w of a super-block sits
// in byte 32*(w/128) + 16*((w%32)/16) + w%16 at shift 2*((w/32)%4) (IQ2_K),
// or byte 32*(w/128) + w%32 at shift 4*((w/64)%2) + 2*((w%64)/32) (IQ2_KS).
// Either way the 16 weights of one output code word come from 16 consecutive
// wire bytes at one shift, so a thread loads 16 bytes and compacts them.
#include "iqk_common.cuh"

namespace iqk {
namespace {

// Four bytes whose low two bits are codes -> one byte of four 2-bit codes.
__device__ __forceinline__ uint32_t pack4(uint32_t v) {
    v &= 0x03030303u;
    v |= v >> 6;            // bits 0-3: codes 0, 1; bits 16-19: codes 2, 3
    return (v & 0xFu) | ((v >> 12) & 0xF0u);
}

// 16 bytes at one shift -> 16 codes, k order, little-endian 2-bit fields.
__device__ __forceinline__ uint32_t compact16(uint4 b, int shift) {
    return pack4(b.x >> shift) | (pack4(b.y >> shift) << 8) | (pack4(b.z >> shift) << 16) |
           (pack4(b.w >> shift) << 24);
}

__device__ __forceinline__ uint4 load16(const uint8_t *p) {
    // wire offsets of a code run are not 16-byte aligned in general (2-byte
    // row header, 70-byte blocks): four 32-bit loads at 2-byte alignment
    const uint16_t *h = reinterpret_cast<const uint16_t *>(p);
    return make_uint4(h[0] | ((uint32_t)h[1] << 16), h[2] | ((uint32_t)h[3] << 16),
                      h[4] | ((uint32_t)h[5] << 16), h[6] | ((uint32_t)h[7] << 16));
}

// One thread per output code word (16 weights); the thread that owns a
// super-block's first word also moves its scale bytes.
template <int MEMBER>
__global__ void __launch_bounds__(256)
pack_iq2_kernel(const uint8_t *__restrict__ wire, int64_t rows, int n, uint32_t *__restrict__ qs,
                uint8_t *__restrict__ s1, uint8_t *__restrict__ s2, uint8_t *__restrict__ s3,
                uint16_t *__restrict__ dv) {
    const int nb = n / 256, wpr = n / 16;  // super-blocks, code words per row
    const int rb = MEMBER == IQK_IQ2_KS ? 2 + 70 * nb : 76 * nb;
    const int64_t total = rows * wpr;
    for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total;
         u += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = u / wpr;
        const int wi = (int)(u - row * wpr), b = wi >> 4, q = wi & 15;
        const uint8_t *r = wire + row * rb;
        if (MEMBER == IQK_IQ2_KS) {
            const uint8_t *blk = r + 2 + 70 * b;
            const int ib64 = q >> 2;  // the word's 16 weights: w = 16q .. 16q+15
            const uint32_t word = compact16(load16(blk + 6 + 32 * (ib64 >> 1) + 16 * (q & 1)),
                                            4 * (ib64 & 1) + 2 * ((q >> 1) & 1));
            qs[u] = word;
            if (q == 0) {
                // s1 = scl u8[n/64], s2 = sch u8[n/256], s3 = sex u8[n/256]
                for (int i = 0; i < 4; ++i) s1[row * (n / 64) + 4 * b + i] = blk[2 + i];
                s2[row * nb + b] = blk[1];
                s3[row * nb + b] = blk[0];
                if (b == 0) dv[row] = (uint16_t)(r[0] | (r[1] << 8));
            }
        } else {
            const uint8_t *blk = r + 76 * b;
            const int ib32 = q >> 1;
            const uint32_t word = compact16(load16(blk + 12 + 32 * (ib32 >> 2) + 16 * (q & 1)),
                                            2 * (ib32 & 3));
            qs[u] = word;
            if (q == 0) {
                // s1 = scl u8[n/32], s2 = sex u8[n/128], s3 unused, dv f16[n/256]
                for (int i = 0; i < 8; ++i) s1[row * (n / 32) + 8 * b + i] = blk[4 + i];
                s2[row * (n / 128) + 2 * b] = blk[2];
                s2[row * (n / 128) + 2 * b + 1] = blk[3];
                dv[row * nb + b] = (uint16_t)(blk[0] | (blk[1] << 8));
            }
        }
    }
}

// IQ1_S_R4: one thread per (4-row group, 32-weight block): its 16 qs bytes
// are transposed into the four rows' words, its four qh words scattered.
__global__ void __launch_bounds__(256)
pack_iq1_kernel(const uint8_t *__restrict__ wire, int64_t groups, int n,
                uint32_t *__restrict__ qs, uint16_t *__restrict__ qh, uint16_t *__restrict__ dv) {
    const int nblock = n / 32;
    const int gb = 4 * (2 + 6 * nblock);  // bytes of one 4-row group
    const int64_t total = groups * nblock;
    for (int64_t u = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; u < total;
         u += (int64_t)gridDim.x * blockDim.x) {
        const int64_t g = u / nblock;
        const int b = (int)(u - g * nblock);
        const uint8_t *grp = wire + g * gb;
        const uint8_t *blk = grp + 8 + 24 * b;  // 8-byte aligned: 16 qs bytes, 4 qh words
        const uint2 lo = *reinterpret_cast<const uint2 *>(blk);
        const uint2 hi = *reinterpret_cast<const uint2 *>(blk + 8);
        const uint2 hw = *reinterpret_cast<const uint2 *>(blk + 16);
        // byte 4i + k -> row k, byte i: a 4x4 byte transpose
        const uint32_t w0 = lo.x, w1 = lo.y, w2 = hi.x, w3 = hi.y;  // sub-groups i = 0..3
        const uint32_t t01a = __byte_perm(w0, w1, 0x5140), t01b = __byte_perm(w0, w1, 0x7362);
        const uint32_t t23a = __byte_perm(w2, w3, 0x5140), t23b = __byte_perm(w2, w3, 0x7362);
        const uint32_t r[4] = {__byte_perm(t01a, t23a, 0x5410), __byte_perm(t01a, t23a, 0x7632),
                               __byte_perm(t01b, t23b, 0x5410), __byte_perm(t01b, t23b, 0x7632)};
        const uint16_t h[4] = {(uint16_t)hw.x, (uint16_t)(hw.x >> 16), (uint16_t)hw.y,
                               (uint16_t)(hw.y >> 16)};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int64_t row = 4 * g + k;
            qs[row * nblock + b] = r[k];
            qh[row * nblock + b] = h[k];
            if (b == 0) dv[row] = (uint16_t)(grp[2 * k] | (grp[2 * k + 1] << 8));
        }
    }
}

}  // namespace

cudaError_t launch_pack(int member, const void *wire, int64_t rows, int n,
                        void *const *streams, cudaStream_t stream, int num_sms) {
    const int threads = 256;
    const int64_t units = member == IQK_IQ1_S_R4 ? (rows / 4) * (n / 32) : rows * (n / 16);
    if (units == 0) return cudaSuccess;
    int64_t blocks = (units + threads - 1) / threads;
    const int64_t cap = (int64_t)num_sms * 8;
    if (blocks > cap) blocks = cap;
    const uint8_t *w = static_cast<const uint8_t *>(wire);
    if (member == IQK_IQ2_KS)
        pack_iq2_kernel<IQK_IQ2_KS><<<(unsigned)blocks, threads, 0, stream>>>(
            w, rows, n, static_cast<uint32_t *>(streams[0]), static_cast<uint8_t *>(streams[1]),
            static_cast<uint8_t *>(streams[2]), static_cast<uint8_t *>(streams[3]),
            static_cast<uint16_t *>(streams[4]));
    else if (member == IQK_IQ2_K)
        pack_iq2_kernel<IQK_IQ2_K><<<(unsigned)blocks, threads, 0, stream>>>(
            w, rows, n, static_cast<uint32_t *>(streams[0]), static_cast<uint8_t *>(streams[1]),
            static_cast<uint8_t *>(streams[2]), nullptr, static_cast<uint16_t *>(streams[3]));
    else
        pack_iq1_kernel<<<(unsigned)blocks, threads, 0, stream>>>(
            w, rows / 4, n, static_cast<uint32_t *>(streams[0]),
            static_cast<uint16_t *>(streams[1]), static_cast<uint16_t *>(streams[2]));
    return cudaGetLastError();
}

}  // namespace iqk
