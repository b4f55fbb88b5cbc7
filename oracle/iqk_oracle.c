/*
 * CPU oracle for the IQ_K routed-expert hot path: TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement of the reference's bit-exact decode, used by tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline leg as the checker.
 * The product library (mlx_iqk_b200/libiqk_b200.so) never links or calls it.
 *
 * Pinned by tests/test_oracle.py against golden vectors that the reference
 * itself produced (tests/golden/make_golden.py runs the reference's
 * format.pack + codec.dequantize on the same wire bytes).
 *
 * Two families of functions:
 *
 *   orc_decode_<member>   decode the k-contiguous relayout streams, the
 *                         reference's format.decode
 *                         (src/mlx_iqk/format.py:819-877);
 *   orc_dequant_<member>  decode ik wire bytes, the reference's vendored CPU
 *                         dequantizers (vendor/ik_llama/iqk_iq2.cpp:502-562,
 *                         vendor/ik_llama/iqk_iq1sr4.cpp:581-604).
 *
 * Both perform the CPU dequantizer's float32 product chain in its order:
 *   2-bit members: dl = d * (float)idx;  w = dl * (float)value
 *   IQ1_S_R4:      dl = d * (float)(2*ls + 1);  w = dl * ((float)g + shift)
 * Compile with -ffp-contract=off so no multiply is fused.
 *
 * orc_gemv_f64 is the float64 reference GEMV the decode tolerance is
 * stated against (tests/test_kernels.py:172-177 in the reference).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "iq1s_grid.h"

/* iq2nl_values: base alphabet in 0..3, shifted alphabet in 4..7
 * (src/mlx_iqk/format.py:110). */
static const int8_t kIq2nl[8] = {-31, -13, 1, 17, -26, -8, 6, 22};

/* IEEE binary16 bits -> float, exact for every pattern (subnormals, inf, nan). */
static float orc_half(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            /* subnormal: value = man * 2^-24; normalise into float32 */
            int e = -1;
            do {
                man <<= 1;
                e++;
            } while ((man & 0x400) == 0);
            man &= 0x3ff;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, sizeof f);
    return f;
}

float orc_half_to_float(uint16_t h) { return orc_half(h); }

/* ---------------------------------------------------------------- relayout */

/* IQ2_KS streams: qs u32[rows, n/16], scl u8[rows, n/64], sch u8[rows, n/256],
 * sex u8[rows, n/256], dv f16[rows]  (src/mlx_iqk/format.py:360-366). */
void orc_decode_iq2_ks(const uint32_t *qs, const uint8_t *scl, const uint8_t *sch,
                       const uint8_t *sex, const uint16_t *dv, int64_t rows,
                       int64_t n, float *out) {
    for (int64_t r = 0; r < rows; ++r) {
        const float d = orc_half(dv[r]);
        for (int64_t g = 0; g < n / 32; ++g) {
            int lo = (scl[r * (n / 64) + g / 2] >> (4 * (g & 1))) & 0xf;
            int hi = (sch[r * (n / 256) + g / 8] >> (g & 7)) & 1;
            int alpha = (sex[r * (n / 256) + g / 8] >> (g & 7)) & 1;
            const float dl = d * (float)((lo | (hi << 4)) - 16);
            for (int j = 0; j < 32; ++j) {
                int64_t k = g * 32 + j;
                int code = (qs[r * (n / 16) + k / 16] >> (2 * (k % 16))) & 3;
                out[r * n + k] = dl * (float)kIq2nl[4 * alpha + code];
            }
        }
    }
}

/* IQ2_K streams: qs u32[rows, n/16], scl u8[rows, n/32], sex u8[rows, n/128],
 * dv f16[rows, n/256]  (src/mlx_iqk/format.py:373-377). */
void orc_decode_iq2_k(const uint32_t *qs, const uint8_t *scl, const uint8_t *sex,
                      const uint16_t *dv, int64_t rows, int64_t n, float *out) {
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t s = 0; s < n / 16; ++s) {
            const float d = orc_half(dv[r * (n / 256) + s / 16]);
            int lo = (scl[r * (n / 32) + s / 2] >> (4 * (s & 1))) & 0xf;
            int alpha = (sex[r * (n / 128) + s / 8] >> (s & 7)) & 1;
            const float dl = d * (float)(lo - 8);
            for (int j = 0; j < 16; ++j) {
                int64_t k = s * 16 + j;
                int code = (qs[r * (n / 16) + k / 16] >> (2 * (k % 16))) & 3;
                out[r * n + k] = dl * (float)kIq2nl[4 * alpha + code];
            }
        }
    }
}

/* IQ1_S_R4 streams: qs u32[rows, n/32], qh u16[rows, n/32], dv f16[rows]
 * (src/mlx_iqk/format.py:367-372, decode at format.py:780-816). */
void orc_decode_iq1_s_r4(const uint32_t *qs, const uint16_t *qh, const uint16_t *dv,
                         int64_t rows, int64_t n, float *out) {
    for (int64_t r = 0; r < rows; ++r) {
        const float d = orc_half(dv[r]);
        for (int64_t b = 0; b < n / 32; ++b) {
            uint32_t qw = qs[r * (n / 32) + b];
            uint32_t h = qh[r * (n / 32) + b];
            const float dl = d * (float)(2 * ((h >> 12) & 7) + 1);
            const float shift = (h & 0x8000) ? -0.125f : 0.125f;
            for (int i = 0; i < 4; ++i) {
                uint32_t idx = ((qw >> (8 * i)) & 0xff) | (((h >> (3 * i)) & 7) << 8);
                uint32_t code = orc_iq1s_grid[idx];
                for (int j = 0; j < 8; ++j) {
                    int g = (int)((code >> (2 * j)) & 3) - 1;
                    out[r * n + b * 32 + 8 * i + j] = dl * ((float)g + shift);
                }
            }
        }
    }
}

/* -------------------------------------------------------------- ik wire */

/* block_iq2_k: d f16, extra u16, scales[8], qs[64]; 76 bytes per 256 weights
 * (vendor/ik_llama/iqk_iq2.cpp:70-76, dequantize_row_iq2_k at 502-529). */
void orc_dequant_iq2_k(const uint8_t *wire, int64_t rows, int64_t n, float *out) {
    const int64_t nb = n / 256, row_bytes = 76 * nb;
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t *blk = wire + r * row_bytes + 76 * b;
            const float d = orc_half((uint16_t)(blk[0] | (blk[1] << 8)));
            uint32_t extra = blk[2] | (blk[3] << 8);
            const uint8_t *sc = blk + 4, *q = blk + 12;
            float *y = out + r * n + 256 * b;
            for (int ib32 = 0; ib32 < 8; ++ib32) {
                const int shift = 2 * (ib32 % 4);
                const uint8_t *qq = q + 32 * (ib32 / 4);
                const float dl1 = d * (float)((sc[ib32] & 0xf) - 8);
                const float dl2 = d * (float)((sc[ib32] >> 4) - 8);
                const int8_t *v1 = kIq2nl + ((extra >> (2 * ib32)) & 1) * 4;
                const int8_t *v2 = kIq2nl + ((extra >> (2 * ib32 + 1)) & 1) * 4;
                for (int j = 0; j < 16; ++j) {
                    y[32 * ib32 + j] = dl1 * (float)v1[(qq[j] >> shift) & 3];
                    y[32 * ib32 + 16 + j] = dl2 * (float)v2[(qq[16 + j] >> shift) & 3];
                }
            }
        }
    }
}

/* IQ2_KS row: f16 row scale, then blocks {extra u16, scales[4], qs[64]} of 70
 * bytes (vendor/ik_llama/iqk_iq2.cpp:78-83, dequantize_row_iq2_ks 532-562). */
void orc_dequant_iq2_ks(const uint8_t *wire, int64_t rows, int64_t n, float *out) {
    const int64_t nb = n / 256, row_bytes = 2 + 70 * nb;
    for (int64_t r = 0; r < rows; ++r) {
        const uint8_t *row = wire + r * row_bytes;
        const float d = orc_half((uint16_t)(row[0] | (row[1] << 8)));
        for (int64_t b = 0; b < nb; ++b) {
            const uint8_t *blk = row + 2 + 70 * b;
            uint32_t extra = blk[0] | (blk[1] << 8);
            const uint8_t *sc = blk + 2, *q = blk + 6;
            float *y = out + r * n + 256 * b;
            for (int ib64 = 0; ib64 < 4; ++ib64) {
                const int shift = 4 * (ib64 % 2);
                const uint8_t *qq = q + 32 * (ib64 / 2);
                int i1 = (sc[ib64] & 0xf) | (((extra >> (8 + 2 * ib64)) & 1) << 4);
                int i2 = (sc[ib64] >> 4) | (((extra >> (9 + 2 * ib64)) & 1) << 4);
                const float dl1 = d * (float)(i1 - 16);
                const float dl2 = d * (float)(i2 - 16);
                const int8_t *v1 = kIq2nl + ((extra >> (2 * ib64)) & 1) * 4;
                const int8_t *v2 = kIq2nl + ((extra >> (2 * ib64 + 1)) & 1) * 4;
                for (int j = 0; j < 32; ++j) {
                    y[64 * ib64 + j] = dl1 * (float)v1[(qq[j] >> shift) & 3];
                    y[64 * ib64 + 32 + j] = dl2 * (float)v2[(qq[j] >> (shift + 2)) & 3];
                }
            }
        }
    }
}

/* IQ1_S_R4 wire: groups of 4 rows; 4 x f16 row scales, then per 32 weights a
 * 24-byte block {qs[16] (byte 4i+k: sub-group i of row k), qh u16[4]}
 * (vendor/ik_llama/iqk_iq1sr4.cpp:581-604). rows must be a multiple of 4. */
void orc_dequant_iq1_s_r4(const uint8_t *wire, int64_t rows, int64_t n, float *out) {
    const int64_t nblock = n / 32, row_bytes = 2 + 6 * nblock;
    for (int64_t g0 = 0; g0 < rows; g0 += 4) {
        const uint8_t *grp = wire + g0 * row_bytes;
        float d[4];
        for (int k = 0; k < 4; ++k) d[k] = orc_half((uint16_t)(grp[2 * k] | (grp[2 * k + 1] << 8)));
        for (int64_t ib = 0; ib < nblock; ++ib) {
            const uint8_t *blk = grp + 8 + 24 * ib;
            for (int k = 0; k < 4; ++k) {
                uint32_t h = blk[16 + 2 * k] | (blk[17 + 2 * k] << 8);
                const float shift = (h & 0x8000) ? -0.125f : 0.125f;
                const float dl = d[k] * (float)(2 * ((h >> 12) & 7) + 1);
                for (int i = 0; i < 4; ++i) {
                    uint32_t idx = blk[4 * i + k] | (((h >> (3 * i)) & 7) << 8);
                    uint32_t code = orc_iq1s_grid[idx];
                    for (int j = 0; j < 8; ++j) {
                        int g = (int)((code >> (2 * j)) & 3) - 1;
                        out[(g0 + k) * n + 32 * ib + 8 * i + j] = dl * ((float)g + shift);
                    }
                }
            }
        }
    }
}

/* ------------------------------------------------------------------ gemv */

/* y[p, r] = sum_k w[sel[p], r, k] * x[tok[p], k], all in float64.
 * w: float32 [E, out, n]; x: float64 [x_rows, n]; y: float64 [pairs, out]. */
void orc_gemv_f64(const float *w, const double *x, const int32_t *sel,
                  const int32_t *tok, int64_t pairs, int64_t out, int64_t n, double *y) {
    for (int64_t p = 0; p < pairs; ++p) {
        const float *we = w + (int64_t)sel[p] * out * n;
        const double *xt = x + (int64_t)tok[p] * n;
        for (int64_t r = 0; r < out; ++r) {
            double acc = 0.0;
            const float *wr = we + r * n;
            for (int64_t k = 0; k < n; ++k) acc += (double)wr[k] * xt[k];
            y[p * out + r] = acc;
        }
    }
}
