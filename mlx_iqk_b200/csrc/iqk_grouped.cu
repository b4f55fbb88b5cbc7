// Grouped per-expert GEMM for the prefill route (sm_100a, tcgen05 + TMEM).
//
//   y[p, r] = sum_k W[sel[p], r, k] * x[tok[p], k]   for every routed pair p
//
// Reference: the prefill route of IqkSwitchLinear.__call__
// (src/mlx_iqk/nn.py:221-238): a full fp16 dequantization of the stacked
// experts followed by mx.gather_mm over (optionally sorted) indices. Here the
// weights are never materialised in HBM: each expert's relayout streams are
// read once per token tile (at most 64 tokens) and dequantized stage by stage
// straight into tensor memory, where they are the A operand of tcgen05.mma.
//
// Numerics. Activations are scaled per row by a power of two 2^S (so the row
// maximum lies in [2^14, 2^15)) and converted to f16 -- exact for bf16 input.
// IQ2_KS weights enter the MMA as the exact small integers idx * value
// (|.| <= 496, exact in f16); the row's f16 scale is applied in the epilogue.
// IQ2_K weights enter as (idx * value) * f16(d_sb * 2^-E): the integer
// product is exact and one f16 multiply applies the super-block scale (E, the
// row's largest super-block exponent, goes back in the epilogue), so one f16
// rounding separates them from the CPU's float weights. Products are exact and accumulate in f32.
//
// Preparation (two launches): a single-block routing kernel counting-sorts
// the pairs by expert and cuts each expert's run into tiles of at most 64
// tokens; a conversion kernel writes each routed pair's scaled, permuted f16
// activation row in sorted order.
//
// GEMM kernel: persistent, one CTA per SM, 26 warps (72 registers each).
//   warp 0      TMA producer of the activation stages (128 weights x the
//               tile's tokens, two 64-wide k atoms, 128-byte swizzle)
//   warp 1      TMEM owner (allocates 512 columns, frees them at exit)
//   warps 2-3   scale loaders: per work item, every row's scale streams
//               packed per 128-weight stage (one table index byte per
//               group), the row factors and the tile's column table
//   warps 4-19  dequantization: every stage, warp (q, j, kh) expands k
//               slice kh of its 32 rows (lane quarter q of row half j) into
//               f16x2 words with byte permutes on the group's table of the
//               four alphabet products, and stores them into the stage's
//               TMEM A buffer (tcgen05.st)
//   warp 20     TMA producer of the 2-bit code chunks (512 weights of every
//               row of the item, 128-byte swizzle)
//   warp 21     MMA issuer (one elected lane): per stage RB x 8
//               M128 N<=64 K16 MMAs, A from TMEM, B from shared memory,
//               into the item's accumulator set (item parity)
//   warps 22-25 epilogue, one per TMEM lane quarter: tcgen05.ld of the
//               finished accumulators, row scale, 2^-S, store y -- while the
//               other roles already run the next item
// Work items are (tile, 256- or 128-row block), expert-major, so CTAs running
// at the same time share one expert's activation tile in L2.
//
// Operand order inside each 16-weight block: the TMEM word pair (c, c + 4)
// of a code word (k = j and 4 + j, then 8 + j and 12 + j) is what one byte
// permute produces from a selector built with one shift, mask and multiply;
// the conversion kernel writes the activations in that same k order.
//
// Every wait is bounded (2 s): a wait that expires sets IQK_DEVERR_TIMEOUT and
// an abort flag that ends the other roles' waits, copies in flight are
// drained, and tensor memory is freed before the CTA exits.
#include <cuda.h>

#include <atomic>

#include "iqk_common.cuh"
#include "iqk_grouped.cuh"
#include "iqk_sync.cuh"
#include "iqk_tables.cuh"

namespace iqk {
namespace {

using namespace dev;

constexpr int kThreadsG = 832;                       // 26 warps
constexpr int kProducer = 0, kTmemWarp = 1, kLoader0 = 2, kDq0 = 4, kCodeWarp = 20,
              kIssuer = 21, kEpi0 = 22;
constexpr int kStageK = 128;                         // weights per k-stage (8 MMAs of K=16)
constexpr int kMaxKS = 4096 / kStageK;               // k-stages of the widest row
constexpr int kCodeK = 512;                          // weights per code load (4 stages)
constexpr int kCodeBox = kGroupRows * kCodeK / 4;    // 16 KB: 128 rows x 128 B, 128-byte swizzle
// IQ1_S_R4 codes: 4 qs bytes (grid index low bytes) per 32 weights, so one
// 512-weight chunk is 128 rows x 64 B (64-byte swizzle)
__host__ __device__ constexpr int code_box(int member) {
    return member == IQK_IQ1_S_R4 ? kGroupRows * kCodeK / 8 : kCodeBox;
}
constexpr int kMaxCodeSlots = 4;
constexpr int kMaxXSlots = 8;
constexpr int kMinXSlots = 4;
constexpr int kNumA = 2;  // A buffers in TMEM: the dequant runs up to one stage ahead
// Work item = one token tile x RB*128 output rows (RB "halves" of 128 rows,
// RB = 1 or 2). Every k-stage (128 weights) goes through the same steps: the
// 16 dequant warps write its A tile (f16, RB halves x 128 rows) into TMEM
// buffer b = stage mod kNumA -- warp (q, j, kh) its lane quarter q of half j
// and k slice kh -- and the issuer runs the stage's RB x 8 MMAs into the
// item's RB accumulators, in stage order, then commits afree[b]. (One issuer
// measured faster overall than one per half on B200: the dequantization
// bounds the kernel, and a second issuer warp takes issue slots from it.)
// Accumulators are double-buffered by item parity, so the four epilogue
// warps drain item i while the dequant warps and the issuer run item i + 1.
// TMEM columns, 64 each: accumulator set s half j at 64*(s*RB + j), A buffer
// b half j at 64*(2*RB + b*RB + j): 4*RB*64 <= 512 columns.
// No wait is ever lapped: a warp writes A buffer b again for stage g + kNumA
// only after afree[b] completes for stage g, which needs the issuer, which
// in turn waits for every warp's aready[b] of stage g + kNumA before
// committing the next phase; the issuer starts item i + 2 in accumulator set
// s only after dempty[s] of item i, which needs item i's dfull[s].
constexpr int kTmemCols = 512;
constexpr int kTok = 64;                             // tokens per work tile
// Barriers, the TMEM slot word and the abort flag; then the group tables.
constexpr int kTabOff = 8 * (2 * kMaxXSlots + 2 * kMaxCodeSlots + 2 * kNumA + 5 + 4) + 16;
constexpr int kTabEntries = 64;  // IQ2_KS: (scale index + 16) | alphabet << 5; IQ2_K: idx + 8 | alpha << 4
// Per epilogue warp: the current item's column table {y offset of the
// pair's row (int64), 2^-S (float), pad}, copied out of the scale buffer so
// that the buffer is released before the accumulators are final.
constexpr int kEcolOff = (kTabOff + 8 * kTabEntries + 15) & ~15;  // 16-byte entries
constexpr int kBarBytes = kEcolOff + 4 * kTok * 16;
// IQ1_S_R4: the 2048-entry grid (16-bit codes) after the barrier region
__host__ __device__ constexpr int bar_bytes(int member) {
    return kBarBytes + (member == IQK_IQ1_S_R4 ? 4096 : 0);
}
static_assert(kEcolOff % 16 == 0 && kTabOff % 8 == 0, "barrier-region alignment");
constexpr int kSmemCap = 227 * 1024;

// Per-item scale buffer: per (stage, row) scale words, transposed so that a
// warp's 32 rows read 32 consecutive words; then row factors and the tile's
// column table (pair index, 2^-S).
// Scale words per (stage, row): IQ2_KS one (four packed group bytes), IQ2_K
// two (sub-block nibbles; alphabet bits and the f16 super-block scale),
// IQ1_S_R4 two (the 16-bit qh of the stage's four blocks).
__host__ __device__ constexpr int scale_words(int member) { return member == IQK_IQ2_KS ? 1 : 2; }
__host__ __device__ constexpr int scale_buf_bytes(int member, int n, int rows) {
    return scale_words(member) * (n / kStageK) * rows * 4 + rows * 4 + 2 * kTok * 4;
}
__host__ __device__ constexpr int x_slot_bytes(int tok_cap) { return tok_cap * 2 * 128; }

// f16x2 alphabet pairs {V[4a], V[4a+1]} and {V[4a+2], V[4a+3]}, IQ2NL values
// (-31, -13, 1, 17) and (-26, -8, 6, 22).
constexpr uint32_t kV01a0 = 0xca80cfc0u, kV01a1 = 0xc800ce80u;
constexpr uint32_t kV23a0 = 0x4c403c00u, kV23a1 = 0x4d804600u;

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(s));
    return d;
}
__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
    __half2 x = *reinterpret_cast<__half2 *>(&a), y = *reinterpret_cast<__half2 *>(&b);
    __half2 r = __hmul2(x, y);
    return *reinterpret_cast<uint32_t *>(&r);
}
__device__ __forceinline__ uint32_t h2_bcast(float f) {
    __half2 r = __float2half2_rn(f);
    return *reinterpret_cast<uint32_t *>(&r);
}

// One code word (16 codes, k = 16w .. 16w+15) -> 8 f16x2 words for TMEM
// columns 8w .. 8w+7, given the group's products t01 = {T0, T1}, t23 = {T2, T3}.
__device__ __forceinline__ void expand_word(uint32_t w, uint32_t t01, uint32_t t23,
                                            uint32_t *out) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t m = (w >> (2 * j)) & 0x03030303u;   // codes j, 4+j, 8+j, 12+j
        const uint32_t s = m * 0x22u + 0x10101010u;        // byte-pair selectors
        out[j] = prmt(t01, t23, s);
        out[4 + j] = prmt(t01, t23, s >> 16);
    }
}

__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];\n" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}

// ------------------------------------------------------------ preparation

__device__ __forceinline__ int block_scan(int v, int *warp_tot, int *total) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
    }
    if (lane == 31) warp_tot[wid] = inc;
    __syncthreads();
    if (wid == 0) {
        const int w = lane < nw ? warp_tot[lane] : 0;
        int winc = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, winc, o);
            if (lane >= o) winc += t;
        }
        if (lane < nw) warp_tot[lane] = winc - w;
        if (lane == nw - 1) warp_tot[32] = winc;
    }
    __syncthreads();
    const int excl = warp_tot[wid] + inc - v;
    *total = warp_tot[32];
    __syncthreads();
    return excl;
}

// One block: bucket the pairs by expert, cut each bucket into tiles of at
// most L.tok_cap tokens. Shared memory: counts, then scatter cursors.
__global__ void __launch_bounds__(1024)
grouped_route_kernel(const int32_t *__restrict__ sel, const int32_t *__restrict__ tok, int pairs,
                     int x_rows, int num_experts, int shard, GroupedLayout L, char *ws) {
    const int cap = L.tok_cap;
    extern __shared__ int32_t cnt[];
    __shared__ int32_t warp_tot[33];
    __shared__ int32_t s_bad, s_tail;
    const int tid = threadIdx.x, nt = blockDim.x;
    int32_t *hdr = reinterpret_cast<int32_t *>(ws + L.hdr);
    int32_t *order = reinterpret_cast<int32_t *>(ws + L.order);
    int4 *tiles = reinterpret_cast<int4 *>(ws + L.tiles);
    for (int e = tid; e < num_experts; e += nt) cnt[e] = 0;
    if (tid == 0) s_bad = 0;
    __syncthreads();
    const int dims = tok ? 1 : pairs / x_rows;
    int err = 0;
    for (int p = tid; p < pairs; p += nt) {
        const int e = sel[p];
        const int t = tok ? tok[p] : p / dims;
        if (e < 0 || e >= num_experts) {
            if (!shard) err |= IQK_DEVERR_EXPERT;  // shard: another rank's expert
        } else if (t < 0 || t >= x_rows) {
            err |= IQK_DEVERR_TOKEN;
        } else {
            atomicAdd(&cnt[e], 1);
        }
    }
    if (err) atomicOr(&s_bad, err);
    __syncthreads();
    const int per = (num_experts + nt - 1) / nt;
    const int b0 = min(tid * per, num_experts), b1 = min(b0 + per, num_experts);
    int c_cnt = 0, c_tiles = 0;
    for (int e = b0; e < b1; ++e) {
        c_cnt += cnt[e];
        c_tiles += (cnt[e] + cap - 1) / cap;
    }
    int n_valid, n_tiles;
    int run = block_scan(c_cnt, warp_tot, &n_valid);
    int trun = block_scan(c_tiles, warp_tot, &n_tiles);
    for (int e = b0; e < b1; ++e) {
        const int c = cnt[e];
        for (int i = 0; i * cap < c; ++i)
            tiles[trun++] = make_int4(e, run + i * cap, min(cap, c - i * cap), 0);
        cnt[e] = run;  // becomes the scatter cursor
        run += c;
    }
    if (tid == 0) {
        hdr[0] = s_bad;
        hdr[1] = n_tiles;
        hdr[2] = n_valid;
        hdr[3] = shard;
        s_tail = n_valid;
    }
    __syncthreads();
    for (int p = tid; p < pairs; p += nt) {
        const int e = sel[p];
        const int t = tok ? tok[p] : p / dims;
        const bool ok = e >= 0 && e < num_experts && t >= 0 && t < x_rows;
        const int pos = ok ? atomicAdd(&cnt[e], 1) : atomicAdd(&s_tail, 1);
        order[pos] = p;
    }
}

// Position of natural index k (0..15) inside a 16-element block of the
// operand order: k = j, 4+j -> 2j, 2j+1; k = 8+j, 12+j -> 8+2j, 9+2j.
__device__ __forceinline__ int perm16(int k) {
    const int h = k & 8, kk = k & 7;
    return h + 2 * (kk & 3) + (kk >> 2);
}

// One block per sorted position: the pair's activation row, scaled by 2^S
// and permuted, as f16 -- plus S. Positions past the routable count exit.
template <typename XT>
__global__ void __launch_bounds__(256)
grouped_convert_kernel(const XT *__restrict__ x, const int32_t *__restrict__ tok, int pairs,
                       int x_rows, int n, GroupedLayout L, char *ws) {
    __shared__ float red[8];
    __shared__ int redb[8];
    __shared__ uint4 stage[8][64];  // per warp: its 32 threads' 32-byte blocks, in order
    const int32_t *hdr = reinterpret_cast<const int32_t *>(ws + L.hdr);
    const int pos = blockIdx.x;
    if (pos >= hdr[2]) return;
    const int p = reinterpret_cast<const int32_t *>(ws + L.order)[pos];
    const int dims = tok ? 1 : pairs / x_rows;
    const int t = tok ? tok[p] : p / dims;
    const XT *xr = x + (int64_t)t * n;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int nblk = n / 16;  // 16-element blocks, at most one per thread (n <= 4096)
    float v[16];
    float amax = 0.f;
    int bad = 0;
    if (tid < nblk) {
        if (sizeof(XT) == 2) {
            const uint4 *src = reinterpret_cast<const uint4 *>(xr + tid * 16);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint4 u = src[h];
                const XT *e = reinterpret_cast<const XT *>(&u);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[8 * h + j] = to_float<XT>(e[j]);
            }
        } else {
            const float4 *src = reinterpret_cast<const float4 *>(xr + tid * 16);
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const float4 f = src[h];
                v[4 * h] = f.x; v[4 * h + 1] = f.y; v[4 * h + 2] = f.z; v[4 * h + 3] = f.w;
            }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            if (!isfinite(v[j])) bad = 1;
            else amax = fmaxf(amax, fabsf(v[j]));
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    if (lane == 0) {
        red[wid] = amax;
        redb[wid] = bad;
    }
    __syncthreads();
    amax = 0.f;
    bad = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        amax = fmaxf(amax, red[w]);
        bad |= redb[w];
    }
    // S <= 126 keeps 2^-S a normal float for the epilogue; only rows whose
    // maximum is below 2^-112 are then not fully normalised.
    const int S = (bad || amax == 0.f) ? 0 : min(14 - ilogbf(amax), 126);
    if (tid == 0) {
        reinterpret_cast<int32_t *>(ws + L.pscale)[pos] = S;
        if (bad) atomicOr(reinterpret_cast<int32_t *>(ws + L.hdr), IQK_DEVERR_NONFINITE);
    }
    // n / 16 is a multiple of 32 (n = 2048 or 4096): a warp is all in or all out
    if (tid < nblk) {
        float f[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) f[perm16(k)] = ldexpf(v[k], S);
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const __half2 h2 = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
            w[i] = *reinterpret_cast<const uint32_t *>(&h2);
        }
        // staged through shared memory so that each store instruction of the
        // warp writes 512 contiguous bytes
        stage[wid][2 * lane] = make_uint4(w[0], w[1], w[2], w[3]);
        stage[wid][2 * lane + 1] = make_uint4(w[4], w[5], w[6], w[7]);
        __syncwarp();
        uint4 *dst = reinterpret_cast<uint4 *>(
            reinterpret_cast<__half *>(ws + L.xs) + (int64_t)pos * n + (tid - lane) * 16);
        dst[lane] = stage[wid][lane];
        dst[32 + lane] = stage[wid][32 + lane];
    }
}

// ------------------------------------------------------------- GEMM kernel

// Activation tensor maps, one per box height 16, 32, ..., 128 rows: a tile's
// k-atom then arrives in one copy of exactly its padded token count.
struct XMaps {
    CUtensorMap m[kGroupTokMax / 16];
};

struct GroupedArgs {
    const void *s[5];
    int64_t out_features;
    // output-row window: rows [row0, row0 + rows_out) of every expert; y is
    // [pairs, rows_out] (the whole projection: row0 = 0, rows_out = out)
    int row0, rows_out;  // experts x out_features <= 2^30 (checked by the C ABI)
    int n, pairs, rblocks;
    int xslots, cslots, tok_cap;  // ring depths (activation, code), token cap
    const char *ws;
    GroupedLayout L;
    int32_t *err;
    void *y;
    int y_dtype;
};

template <typename T>
__device__ __forceinline__ void store_out(void *y, int64_t i, float v) {
    static_cast<T *>(y)[i] = from_float<T>(v);
}

__device__ __forceinline__ uint4 ldg128(const void *p) {
    return __ldg(reinterpret_cast<const uint4 *>(p));
}

// Scale loader (2 warps): one item's scale streams for its 128 rows, repacked
// per (stage, row) into the transposed buffer, plus row factors and the
// tile's column table. Each thread owns rows t and t + 64.
template <int MEMBER>
__device__ __forceinline__ void load_item_scales(const GroupedArgs &a, int4 tl, int rb, int rows,
                                                 int t, uint32_t *sc, float *rsc, int32_t *colp,
                                                 float *colf) {
    const int n = a.n, KS = n / kStageK;
    const bool wide = n == 4096;
    const int64_t out = a.out_features;
    // column table first: independent loads
    const int32_t *order = reinterpret_cast<const int32_t *>(a.ws + a.L.order);
    const int32_t *pscale = reinterpret_cast<const int32_t *>(a.ws + a.L.pscale);
    for (int j = t; j < tl.z; j += 64) {
        colp[j] = order[tl.y + j];
        colf[j] = __int_as_float((127 - pscale[tl.y + j]) << 23);  // 2^-S, S <= 126
    }
#pragma unroll 1
    for (int r = t; r < rows; r += 64) {
        const int64_t rl = (int64_t)rb * rows + r;  // window-local row
        const int64_t row = (int64_t)tl.x * out + a.row0 + (rl < a.rows_out ? rl : 0);
        if (MEMBER == IQK_IQ2_KS) {
            // every load of the row is issued before any is used
            const uint8_t *scl = static_cast<const uint8_t *>(a.s[1]) + row * (n / 64);
            const uint8_t *sch = static_cast<const uint8_t *>(a.s[2]) + row * (n / 256);
            const uint8_t *sex = static_cast<const uint8_t *>(a.s[3]) + row * (n / 256);
            uint4 v[4];
            uint2 hb[2], xb[2];
            v[0] = ldg128(scl);
            v[1] = ldg128(scl + 16);
            if (wide) {
                v[2] = ldg128(scl + 32);
                v[3] = ldg128(scl + 48);
            }
            hb[0] = __ldg(reinterpret_cast<const uint2 *>(sch));
            xb[0] = __ldg(reinterpret_cast<const uint2 *>(sex));
            if (wide) {
                hb[1] = __ldg(reinterpret_cast<const uint2 *>(sch + 8));
                xb[1] = __ldg(reinterpret_cast<const uint2 *>(sex + 8));
            }
            const uint16_t dvb = static_cast<const uint16_t *>(a.s[4])[row];
#pragma unroll
            for (int c = 0; c < 4; ++c) {  // 8 stages per 16 scl bytes
                if (c >= n / 1024) break;
                const uint32_t sv[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
                const uint32_t h32 = (c & 1) ? hb[c >> 1].y : hb[c >> 1].x;
                const uint32_t x32 = (c & 1) ? xb[c >> 1].y : xb[c >> 1].x;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    // stage 8c+j: groups 4(8c+j) .. +3, one byte each:
                    // 5-bit scale (low nibble | high bit << 4) | alphabet << 5
                    const uint32_t lo = (sv[j >> 1] >> (16 * (j & 1))) & 0xffffu;
                    const uint32_t hi = (h32 >> (4 * j)) & 15u, al = (x32 >> (4 * j)) & 15u;
                    uint32_t packed = 0;
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        packed |= (((lo >> (4 * q)) & 15u) | (((hi >> q) & 1u) << 4) |
                                   (((al >> q) & 1u) << 5)) << (8 * q);
                    sc[(8 * c + j) * rows + r] = packed;
                }
            }
            rsc[r] = half_bits_to_float(dvb);
        } else if (MEMBER == IQK_IQ1_S_R4) {
            // qh u16[n/32] (n/16 bytes): stage ks = blocks 4ks .. 4ks+3 = words 2ks, 2ks+1
            const uint8_t *qh = reinterpret_cast<const uint8_t *>(a.s[1]) + row * (n / 16);
            const uint16_t dvb = static_cast<const uint16_t *>(a.s[2])[row];
            // four 16-byte loads in flight at a time (eight stages)
#pragma unroll 1
            for (int i0 = 0; i0 < n / 256; i0 += 4) {
                uint4 v[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) v[i] = ldg128(qh + 16 * (i0 + i));
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int ks = 2 * (i0 + i);
                    sc[ks * rows + r] = v[i].x;
                    sc[(KS + ks) * rows + r] = v[i].y;
                    sc[(ks + 1) * rows + r] = v[i].z;
                    sc[(KS + ks + 1) * rows + r] = v[i].w;
                }
            }
            // the operand carries (2ls + 1) * 8 * (g + shift); d / 8 goes here
            rsc[r] = half_bits_to_float(dvb) * 0.125f;
        } else {
            const uint8_t *scl = static_cast<const uint8_t *>(a.s[1]) + row * (n / 32);
            const uint8_t *sex = static_cast<const uint8_t *>(a.s[2]) + row * (n / 128);
            const uint16_t *dv = static_cast<const uint16_t *>(a.s[3]) + row * (n / 256);
            uint4 v[8], xv[2], dq[2];
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (i < n / 512) v[i] = ldg128(scl + 16 * i);
            xv[0] = ldg128(sex);
            dq[0] = ldg128(dv);
            if (wide) {
                xv[1] = ldg128(sex + 16);
                dq[1] = ldg128(dv + 8);
            }
            const int nd = n / 256;
            float m = 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                if (i >= nd) break;
                const uint32_t w = reinterpret_cast<const uint32_t *>(&dq[i >> 3])[(i & 7) >> 1];
                m = fmaxf(m, fabsf(half_bits_to_float((uint16_t)(w >> (16 * (i & 1))))));
            }
            const int E = m > 0.f ? ilogbf(m) + 1 : 0;
            rsc[r] = ldexpf(1.f, E);
            const float dn = ldexpf(1.f, -E);
#pragma unroll
            for (int ks = 0; ks < 32; ++ks) {
                if (ks >= KS) break;
                const uint32_t s32 = reinterpret_cast<const uint32_t *>(&v[ks >> 2])[ks & 3];
                const uint32_t x32 = reinterpret_cast<const uint32_t *>(&xv[ks >> 4])[(ks & 15) >> 2];
                const int di = ks >> 1;
                const uint32_t dw = reinterpret_cast<const uint32_t *>(&dq[di >> 3])[(di & 7) >> 1];
                const float d = half_bits_to_float((uint16_t)(dw >> (16 * (di & 1)))) * dn;
                const __half dh = __float2half_rn(d);
                const uint32_t db = (uint32_t)*reinterpret_cast<const uint16_t *>(&dh);
                sc[ks * rows + r] = s32;
                sc[(KS + ks) * rows + r] = ((x32 >> (8 * (ks & 3))) & 0xffu) | (db << 16);
            }
        }
    }
}

// Shared-memory carve-up of the GEMM kernel (base 1024-aligned).
struct GemmSmem {
    uint32_t x, code, sbuf, bars;  // offsets
    int sb;                        // bytes of one scale buffer
};
__host__ __device__ inline GemmSmem gemm_smem(int member, int n, int rb_rows, int xslots,
                                              int cslots) {
    GemmSmem g;
    g.x = 0;
    g.code = (uint32_t)(xslots * x_slot_bytes(kTok));
    g.sbuf = g.code + cslots * (rb_rows / kGroupRows) * code_box(member);
    g.sb = (scale_buf_bytes(member, n, rb_rows) + 15) & ~15;
    g.bars = g.sbuf + 2 * g.sb;
    return g;
}

template <int MEMBER, int RB>
__global__ void __launch_bounds__(kThreadsG, 1)
grouped_gemm_kernel(const GroupedArgs a, const __grid_constant__ CUtensorMap qs_map,
                    const __grid_constant__ XMaps x_maps) {
    constexpr int kRows = RB * kGroupRows;    // output rows per work item
    constexpr uint32_t kACol = 2 * RB * 64u;  // first A-buffer column (after both accumulator sets)
    constexpr int kCodeSlot = RB * code_box(MEMBER);  // codes of one 512-weight chunk, all rows
    constexpr uint32_t kCodeRow = MEMBER == IQK_IQ1_S_R4 ? 64u : 128u;  // code bytes per row
    extern __shared__ char smem_raw[];
    char *smem = smem_raw + ((1024u - (saddr(smem_raw) & 1023u)) & 1023u);
    const uint32_t smem_u = saddr(smem);
    const int n = a.n, KS = n / kStageK, XS = a.xslots, CS = a.cslots;
    const int cap = a.tok_cap;
    const GemmSmem G = gemm_smem(MEMBER, n, kRows, XS, CS);
    const uint32_t xatom = (uint32_t)cap * 128u;  // bytes of one 64-wide k atom
    char *sbuf = smem + G.sbuf;
    // xfull: a stage's activations landed; sdone: the stage's MMAs finished
    // (frees its activation slot).
    uint64_t *xfull = reinterpret_cast<uint64_t *>(smem + G.bars);
    uint64_t *sdone = xfull + kMaxXSlots;
    uint64_t *cfull = sdone + kMaxXSlots;
    uint64_t *cempty = cfull + kMaxCodeSlots;
    uint64_t *aready = cempty + kMaxCodeSlots;  // [kNumA] A buffer written (16 warps)
    uint64_t *afree = aready + kNumA;           // [kNumA] A buffer read by its MMAs
    uint64_t *dfull = afree + kNumA;  // [2] an item's accumulators final (by parity)
    uint64_t *dempty = dfull + 2;     // [2] the epilogue warps read them
    uint64_t *drain = dempty + 2;
    uint64_t *sfull = drain + 1;   // [2]
    uint64_t *sempty = sfull + 2;  // [2]
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(sempty + 2);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
    // f16x2 pair tables of every (scale index, alphabet): {V0, V1} and {V2, V3}
    // times the index (IQ2_KS), or times the index before the super-block
    // scale (IQ2_K). Products of small integers: exact in f16.
    uint2 *gtab = reinterpret_cast<uint2 *>(smem + G.bars + kTabOff);
    uint16_t *grid = reinterpret_cast<uint16_t *>(smem + G.bars + kBarBytes);  // IQ1_S_R4

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int32_t *hdr = reinterpret_cast<const int32_t *>(a.ws + a.L.hdr);
    const int4 *tiles = reinterpret_cast<const int4 *>(a.ws + a.L.tiles);
    const int32_t *order = reinterpret_cast<const int32_t *>(a.ws + a.L.order);
    const int64_t out = a.out_features;
    const int ntiles = hdr[1], n_valid = hdr[2];
    const int64_t items = (int64_t)ntiles * a.rblocks;

    if (threadIdx.x == 0) {
        for (int i = 0; i < XS; ++i) {
            bar_init(&xfull[i], 1);
            bar_init(&sdone[i], 1);
        }
        for (int i = 0; i < CS; ++i) {
            bar_init(&cfull[i], 1);
            bar_init(&cempty[i], 16);
        }
        for (int i = 0; i < kNumA; ++i) {
            bar_init(&aready[i], 16);
            bar_init(&afree[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            bar_init(&dfull[i], 1);
            bar_init(&dempty[i], 4);
        }
        bar_init(drain, 1);
        for (int i = 0; i < 2; ++i) {
            bar_init(&sfull[i], 64);
            bar_init(&sempty[i], 16 + 4);  // dequant warps, then the epilogue warps
        }
        *abort_flag = 0;
        bar_fence_init();
    }
    if (MEMBER == IQK_IQ1_S_R4) {
        for (int i = threadIdx.x; i < 2048; i += blockDim.x) grid[i] = g_iq1s_grid[i];
    }
    if (MEMBER == IQK_IQ1_S_R4 && threadIdx.x < 16) {
        // block table (ls | sign << 3): {T0, T1}, {T2, 0} with
        // T[c] = (2ls + 1) * (8 * (c - 1) + s), s = -1 for a set sign bit:
        // small integers, exact in f16
        const int i = threadIdx.x;
        const float m = (float)(2 * (i & 7) + 1), sg = (i & 8) ? -1.f : 1.f;
        const __half2 a01 = __floats2half2_rn(m * (sg - 8.f), m * sg);
        const __half2 a23 = __floats2half2_rn(m * (sg + 8.f), 0.f);
        gtab[i] = make_uint2(*reinterpret_cast<const uint32_t *>(&a01),
                             *reinterpret_cast<const uint32_t *>(&a23));
    } else if (MEMBER != IQK_IQ1_S_R4 && threadIdx.x < kTabEntries) {
        const int i = threadIdx.x;
        const int idx = MEMBER == IQK_IQ2_KS ? (i & 31) - 16 : (i & 15) - 8;
        const bool alpha = MEMBER == IQK_IQ2_KS ? (i >> 5) & 1 : (i >> 4) & 1;
        const uint32_t hv = h2_bcast((float)idx);
        gtab[i] = make_uint2(hmul2_bits(hv, alpha ? kV01a1 : kV01a0),
                             hmul2_bits(hv, alpha ? kV23a1 : kV23a0));
    }
    if (warp == kTmemWarp) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
        tc_fence_before();
    }
    // Zero the outputs of unroutable pairs (bad expert or row index); a
    // shard preparation leaves the rows of other ranks' pairs untouched.
    {
        const int tail = hdr[3] ? 0 : a.pairs - n_valid;
        const int ro = a.rows_out;
        const int64_t total = (int64_t)tail * ro;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
             i += (int64_t)gridDim.x * blockDim.x) {
            const int64_t p = order[n_valid + i / ro];
            const int64_t r = i % ro;
            if (a.y_dtype == IQK_F32) store_out<float>(a.y, p * ro + r, 0.f);
            else if (a.y_dtype == IQK_F16) store_out<__half>(a.y, p * ro + r, 0.f);
            else store_out<__nv_bfloat16>(a.y, p * ro + r, 0.f);
        }
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    auto give_up = [&]() {
        if (!*abort_flag) {
            *abort_flag = 1;
            atomicOr(a.err, IQK_DEVERR_TIMEOUT);
        }
    };

    if (warp == kProducer) {
        // Activation stages: lane 0 keeps the ring, lanes 0-1 issue the two
        // 64-wide k atoms of a stage in one instruction.
        int g = 0;
        bool ok = true;
        for (int64_t it = blockIdx.x; ok && it < items && !*abort_flag; it += gridDim.x) {
            const int4 tl = tiles[it / a.rblocks];
            const int npad = (tl.z + 15) & ~15;
            const CUtensorMap *xm = &x_maps.m[npad / 16 - 1];
            for (int ks = 0; ks < KS; ++ks, ++g) {
                const int xs = g % XS;
                if (lane == 0) {
                    ok = bar_wait(&sdone[xs], ((uint32_t)(g / XS) & 1u) ^ 1u, abort_flag);
                    if (ok) bar_expect_tx(&xfull[xs], (uint32_t)(2 * npad * 128));
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                const uint32_t st = smem_u + G.x + xs * x_slot_bytes(cap);
                if (lane < 2)
                    tma_2d(st + lane * xatom, xm, ks * kStageK + lane * 64, tl.y, &xfull[xs]);
            }
        }
        if (lane == 0) {
            if (!ok) give_up();
            // Drain: every copy issued must land before the CTA exits (bounded by time only).
            for (int d = 0; d < XS && d < g; ++d) {
                const int gg = g - 1 - d;
                if (!bar_wait(&xfull[gg % XS], (uint32_t)(gg / XS) & 1u, nullptr)) give_up();
            }
        }
        __syncwarp();
    } else if (warp == kCodeWarp) {
        // Code chunks (512 weights of all the item's rows) run ahead on their own ring.
        if (lane == 0) {
            int cchunk = 0;
            bool ok = true;
            for (int64_t it = blockIdx.x; ok && it < items && !*abort_flag; it += gridDim.x) {
                const int4 tl = tiles[it / a.rblocks];
                const int rb = (int)(it % a.rblocks);
                const int row0 = (int)((int64_t)tl.x * out + a.row0 + (int64_t)rb * kRows);
                for (int c = 0; c < KS / 4; ++c, ++cchunk) {
                    const int cs = cchunk % CS;
                    if (!bar_wait(&cempty[cs], ((uint32_t)(cchunk / CS) & 1u) ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    bar_expect_tx(&cfull[cs], kCodeSlot);
#pragma unroll
                    for (int j = 0; j < RB; ++j)
                        tma_2d(smem_u + G.code + cs * kCodeSlot + j * code_box(MEMBER), &qs_map,
                               c * (int)kCodeRow, row0 + j * kGroupRows, &cfull[cs]);
                }
            }
            if (!ok) give_up();
            for (int d = 0; d < CS && d < cchunk; ++d) {
                const int cc = cchunk - 1 - d;
                if (!bar_wait(&cfull[cc % CS], (uint32_t)(cc / CS) & 1u, nullptr)) give_up();
            }
        }
        __syncwarp();
    } else if (warp == kIssuer) {
        // The MMA issuer: per stage, RB x 8 MMAs (one activation stage, one A
        // buffer) into the RB accumulators, in stage order. The whole warp
        // runs the loop converged; one elected lane issues.
        int g = 0, item_i = 0;
        bool ok = true;
        for (int64_t it = blockIdx.x; ok && it < items && !*abort_flag;
             it += gridDim.x, ++item_i) {
            const int4 tl = tiles[it / a.rblocks];
            const int npad = (tl.z + 15) & ~15;
            const uint32_t idesc = idesc_f16(kGroupRows, npad);
            // accumulator set s (item parity) is free once the epilogue warps
            // read item i - 2's results from it
            const int sacc = item_i & 1;
            const uint32_t acc = tmem + (uint32_t)(sacc * RB) * 64u;
            if (item_i >= 2 &&
                !bar_wait(&dempty[sacc], ((uint32_t)(item_i >> 1) & 1u) ^ 1u, abort_flag)) {
                ok = false;
                break;
            }
            for (int ks = 0; ks < KS; ++ks, ++g) {
                const int xs = g % XS, b = g % kNumA;
                if (!bar_wait(&xfull[xs], (uint32_t)(g / XS) & 1u, abort_flag) ||
                    !bar_wait(&aready[b], (uint32_t)(g / kNumA) & 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t st = smem_u + G.x + xs * x_slot_bytes(cap);
                // elect.sync needs the whole warp converged: one lane issues.
                __syncwarp();
                if (elect_one()) {
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint64_t bdesc = sw128_desc(st + (kk >> 2) * xatom + (kk & 3) * 32);
#pragma unroll
                        for (int j = 0; j < RB; ++j)
                            tc_mma_ts(acc + (uint32_t)j * 64u,
                                      tmem + kACol + (uint32_t)(b * RB + j) * 64u + kk * 8, bdesc,
                                      idesc, (ks == 0 && kk == 0) ? 0u : 1u);
                    }
                    tc_commit(&sdone[xs]);
                    tc_commit(&afree[b]);
                }
                __syncwarp();
            }
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            if (elect_one()) tc_commit(&dfull[sacc]);
            __syncwarp();
        }
        if (!ok && lane == 0) give_up();
        __syncwarp();
        // Every MMA issued must finish before tensor memory is freed.
        if (elect_one()) tc_commit(drain);
        __syncwarp();
    } else if (warp >= kLoader0 && warp < kDq0) {
        const int t = threadIdx.x - 32 * kLoader0;  // 0..63
        int item_i = 0;
        for (int64_t it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x, ++item_i) {
            const int buf = item_i & 1;
            const uint32_t use = (uint32_t)(item_i >> 1);
            if (!bar_wait(&sempty[buf], (use & 1u) ^ 1u, abort_flag)) {
                give_up();
                break;
            }
            char *b = sbuf + buf * G.sb;
            uint32_t *sc = reinterpret_cast<uint32_t *>(b);
            float *rsc = reinterpret_cast<float *>(b + scale_words(MEMBER) * KS * kRows * 4);
            load_item_scales<MEMBER>(a, tiles[it / a.rblocks], (int)(it % a.rblocks), kRows, t,
                                     sc, rsc, reinterpret_cast<int32_t *>(rsc + kRows),
                                     rsc + kRows + kTok);
            bar_arrive(&sfull[buf]);
        }
    } else if (warp >= kDq0 && warp < kCodeWarp) {
        // dequant warp (q, j, kh): TMEM lane quarter q (fixed by the warp's
        // index mod 4), row half j, and k slice kh -- WPW of the stage's 8
        // code words (16 weights each) -- of every stage.
        constexpr int KH = 4 / RB, WPW = 8 / KH;
        const int dq = warp - kDq0;
        const int q = warp & 3;
        const int j = (dq >> 2) % RB, kh = (dq >> 2) / RB;
        const int rloc = kGroupRows * j + 32 * q + lane;  // item-local row
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        const uint32_t rsw = (uint32_t)(rloc & 7);  // 128-byte swizzle of this code row
        int g = 0, item_i = 0;
        for (int64_t it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x, ++item_i) {
            const int buf = item_i & 1;
            if (!bar_wait(&sfull[buf], (uint32_t)(item_i >> 1) & 1u, abort_flag)) {
                give_up();
                break;
            }
            const uint32_t *sc = reinterpret_cast<const uint32_t *>(sbuf + buf * G.sb);
            bool ok = true;
            for (int ks = 0; ks < KS; ++ks, ++g) {
                const int chunk = g >> 2, cs = chunk % CS, sub = g & 3, ab = g % kNumA;
                const uint32_t s0 = sc[ks * kRows + rloc];
                const uint32_t s1 = scale_words(MEMBER) == 2 ? sc[(KS + ks) * kRows + rloc] : 0u;
                if (!bar_wait(&cfull[cs], (uint32_t)(chunk / CS) & 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                // this warp's code words of the stage: word w of the stage is
                // word w % 4 of 16-byte chunk 2*sub + w / 4 of the row
                const uint32_t code_u = smem_u + G.code + cs * kCodeSlot + rloc * kCodeRow;
                uint32_t words[WPW];
                if (MEMBER == IQK_IQ1_S_R4) {
                    // the stage's 16 qs bytes (4 blocks) are 16-byte chunk `sub`
                    // of the row, 64-byte swizzled; this warp's code words
                    // kh*WPW .. are blocks kh*WPW/2 ..: one qs word per block
                    const uint32_t ch = code_u + (((uint32_t)sub ^ ((uint32_t)(rloc >> 1) & 3u)) << 4);
                    if (WPW == 4) {
                        const uint2 c = lds64(ch + (uint32_t)kh * 8u);
                        words[0] = c.x;
                        words[1] = c.y;
                    } else {
                        words[0] = lds32(ch + (uint32_t)kh * 4u);
                    }
                } else if (WPW == 4) {
                    const uint4 c = lds128(code_u + (((uint32_t)(2 * sub + kh) ^ rsw) << 4));
                    words[0] = c.x;
                    words[1] = c.y;
                    words[2 % WPW] = c.z;
                    words[3 % WPW] = c.w;
                } else {
                    const uint2 c = lds64(code_u + (((uint32_t)(2 * sub + (kh >> 1)) ^ rsw) << 4) +
                                          (uint32_t)(kh & 1) * 8u);
                    words[0] = c.x;
                    words[1] = c.y;
                }
                __syncwarp();
                // every warp reads every stage: the chunk's last stage releases it
                if (lane == 0 && sub == 3) bar_arrive(&cempty[cs]);
                // A buffer ab was last read by the MMAs of stage g - kNumA
                if (g >= kNumA &&
                    !bar_wait(&afree[ab], ((uint32_t)(g / kNumA) & 1u) ^ 1u, abort_flag)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t taddr = tmem + lane_base + kACol + (uint32_t)(ab * RB + j) * 64u +
                                       (uint32_t)(kh * WPW) * 8u;
                // IQ2_K: the super-block scale, f16 in both halves
                const uint32_t dsb2 = MEMBER == IQK_IQ2_K ? (s1 >> 16) * 0x10001u : 0u;
                uint32_t t01 = 0, t23 = 0, hs = 0, qw = 0;
#pragma unroll
                for (int wd = 0; wd < WPW; ++wd) {
                    const int wg = kh * WPW + wd;  // word of the stage
                    if (MEMBER == IQK_IQ1_S_R4) {
                        if ((wd & 1) == 0) {  // one 32-weight block per two code words
                            const int bl = wg >> 1;  // block of the stage
                            const uint32_t h = (((bl & 2) ? s1 : s0) >> (16 * (bl & 1))) & 0xffffu;
                            // the four 3-bit grid-index high parts, one per byte
                            hs = (((h & 0x1C7u) * 0x401u) & 0x00070007u) |
                                 (((h & 0xE38u) * 0x8020u) & 0x07000700u);
                            const uint2 t = gtab[(h >> 12) & 15u];
                            t01 = t.x;
                            t23 = t.y;
                            qw = words[wd >> 1];
                        }
                        // both grid indices of octets 2o, 2o+1: qs byte | high part << 8
                        const uint32_t v = prmt(qw, hs, (wd & 1) ? 0x7362u : 0x5140u);
                        const uint32_t cw = (uint32_t)grid[v & 0xffffu] |
                                            ((uint32_t)grid[v >> 16] << 16);
                        uint32_t r[8];
                        expand_word(cw, t01, t23, r);
                        tmem_st8(taddr + wd * 8, r);
                        continue;
                    }
                    if (MEMBER == IQK_IQ2_KS) {
                        if ((wd & 1) == 0) {  // one 32-weight group per two words
                            const uint2 t = gtab[prmt(s0, 0u, 0x4440u + (uint32_t)(wg >> 1))];
                            t01 = t.x;
                            t23 = t.y;
                        }
                    } else {
                        const uint32_t ti = ((s0 >> (4 * wg)) & 15u) | (((s1 >> wg) & 1u) << 4);
                        const uint2 t = gtab[ti];
                        t01 = hmul2_bits(t.x, dsb2);
                        t23 = hmul2_bits(t.y, dsb2);
                    }
                    uint32_t r[8];
                    expand_word(words[wd], t01, t23, r);
                    tmem_st8(taddr + wd * 8, r);
                }
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) bar_arrive(&aready[ab]);
            }
            if (!ok) {
                give_up();
                break;
            }
            if (*abort_flag) break;
            // this item's scale buffer is read (the epilogue warps release it too)
            __syncwarp();
            if (lane == 0) bar_arrive(&sempty[buf]);
        }
    } else if (warp >= kEpi0 && warp < kEpi0 + 4) {
        // Epilogue warp: TMEM lane quarter q of both row halves. Per item: copy
        // the column table and this thread's row scales out of the scale
        // buffer and release it at once (the loader refills it for item i + 2
        // during item i + 1); then, once the accumulators are final (dfull of
        // the item's parity), D rows are this thread's output rows, columns
        // the tile's tokens: row scale and 2^-S applied, stored to y; then the
        // accumulator set is released.
        const int q = warp & 3;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        uint4 *ecol = reinterpret_cast<uint4 *>(smem + G.bars + kEcolOff) + (warp - kEpi0) * kTok;
        int item_i = 0;
        for (int64_t it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x, ++item_i) {
            const int4 tl = tiles[it / a.rblocks];
            const int rb = (int)(it % a.rblocks);
            const int npad = (tl.z + 15) & ~15;
            const int buf = item_i & 1, sacc = item_i & 1;
            if (!bar_wait(&sfull[buf], (uint32_t)(item_i >> 1) & 1u, abort_flag)) {
                give_up();
                break;
            }
            const char *b = sbuf + buf * G.sb;
            const float *rsc =
                reinterpret_cast<const float *>(b + scale_words(MEMBER) * KS * kRows * 4);
            const int32_t *colp = reinterpret_cast<const int32_t *>(rsc + kRows);
            const float *colf = rsc + kRows + kTok;
            float rscale[RB];
#pragma unroll
            for (int j = 0; j < RB; ++j) rscale[j] = rsc[kGroupRows * j + 32 * q + lane];
#pragma unroll
            for (int h = 0; h < kTok / 32; ++h) {
                const int col = 32 * h + lane;
                const int64_t off = col < tl.z ? (int64_t)colp[col] * a.rows_out : 0;
                ecol[col] = make_uint4((uint32_t)off, (uint32_t)(off >> 32),
                                       __float_as_uint(colf[col]), 0u);
            }
            __syncwarp();
            if (lane == 0) bar_arrive(&sempty[buf]);
            if (!bar_wait(&dfull[sacc], (uint32_t)(item_i >> 1) & 1u, abort_flag)) {
                give_up();
                break;
            }
            tc_fence_after();
#pragma unroll
            for (int j = 0; j < RB; ++j) {
                const int64_t rlocal = (int64_t)rb * kRows + kGroupRows * j + 32 * q + lane;
                const bool row_ok = rlocal < a.rows_out;
                for (int c = 0; c < npad; c += 8) {
                    uint32_t d[8];
                    tmem_ld8(tmem + lane_base + (uint32_t)((sacc * RB + j) * 64 + c), d);
                    tc_wait_ld();
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const int col = c + k;
                        if (col < tl.z && row_ok) {
                            const uint4 e = ecol[col];
                            const int64_t o = (int64_t)(((uint64_t)e.y << 32) | e.x) + rlocal;
                            const float v = __uint_as_float(d[k]) * rscale[j] * __uint_as_float(e.z);
                            if (a.y_dtype == IQK_F32) store_out<float>(a.y, o, v);
                            else if (a.y_dtype == IQK_F16) store_out<__half>(a.y, o, v);
                            else store_out<__nv_bfloat16>(a.y, o, v);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(&dempty[sacc]);
        }
    }
    __syncthreads();
    if (warp == kTmemWarp) {
        if (lane == 0 && !bar_wait(drain, 0, nullptr)) give_up();
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

cudaError_t encode_map(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t inner,
                       uint64_t rows, uint64_t row_bytes, uint32_t box_inner, uint32_t box_rows,
                       CUtensorMapSwizzle swz) {
    using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static EncodeFn encode = nullptr;
    if (!encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
        if (err != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
        encode = reinterpret_cast<EncodeFn>(fn);
    }
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t estr[2] = {1u, 1u};
    const CUresult res = encode(map, dt, 2, const_cast<void *>(base), dims, strides, box, estr,
                                CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return res == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

}  // namespace

GroupedLayout grouped_layout(int64_t n, int64_t num_experts, int64_t pairs) {
    GroupedLayout L{};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off += (bytes + 255) & ~size_t(255);
        return at;
    };
    // 64-token tiles: the four per-group accumulators and A slots fill TMEM.
    L.tok_cap = kTok;
    L.max_tiles = (num_experts < pairs ? num_experts : pairs) + pairs / L.tok_cap + 1;
    L.hdr = take(64);
    L.order = take(sizeof(int32_t) * (size_t)(pairs + 1));
    L.pscale = take(sizeof(int32_t) * (size_t)(pairs + 1));
    L.tiles = take(16 * (size_t)L.max_tiles);
    L.xs = take(2 * (size_t)pairs * (size_t)n);
    L.total = off;
    return L;
}

cudaError_t launch_grouped_prepare(const void *x, int x_dtype, int64_t x_rows, int n,
                                   int64_t num_experts, const int32_t *sel, const int32_t *tok,
                                   int64_t pairs, void *ws, cudaStream_t stream, bool shard) {
    const GroupedLayout L = grouped_layout(n, num_experts, pairs);
    char *w = static_cast<char *>(ws);
    const size_t hist = sizeof(int32_t) * (size_t)num_experts;
    cudaError_t err = cudaSuccess;
    if (hist > 48 * 1024) {
        err = cudaFuncSetAttribute(grouped_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)hist);
        if (err != cudaSuccess) return err;
    }
    grouped_route_kernel<<<1, 1024, hist, stream>>>(sel, tok, (int)pairs, (int)x_rows,
                                                    (int)num_experts, shard ? 1 : 0, L, w);
    if ((err = cudaGetLastError()) != cudaSuccess) return err;
    const unsigned blocks = (unsigned)pairs;
#define IQK_CONV(T)                                                                         \
    grouped_convert_kernel<T><<<blocks, 256, 0, stream>>>(static_cast<const T *>(x), tok,    \
                                                          (int)pairs, (int)x_rows, n, L, w)
    if (x_dtype == IQK_F32) IQK_CONV(float);
    else if (x_dtype == IQK_F16) IQK_CONV(__half);
    else IQK_CONV(__nv_bfloat16);
#undef IQK_CONV
    return cudaGetLastError();
}

cudaError_t launch_grouped_run(int member, const void *const *streams, int64_t num_experts,
                               int64_t out_features, int n, int64_t pairs, void *y, int y_dtype,
                               const void *ws, cudaStream_t stream, int num_sms,
                               int64_t row_start, int64_t rows_out) {
    const GroupedLayout L = grouped_layout(n, num_experts, pairs);
    GroupedArgs ga{};
    const RowBytes rb = row_bytes(member, n);
    for (int i = 0; i < rb.count; ++i) ga.s[i] = streams[i];
    ga.out_features = out_features;
    ga.row0 = (int)row_start;
    ga.rows_out = (int)(rows_out < 0 ? out_features : rows_out);
    ga.n = n;
    ga.pairs = (int)pairs;
    ga.ws = static_cast<const char *>(ws);
    ga.L = L;
    ga.err = reinterpret_cast<int32_t *>(const_cast<char *>(ga.ws) + L.hdr);
    ga.y = y;
    ga.y_dtype = y_dtype;
    ga.tok_cap = L.tok_cap;
    // Items of 256 rows (two halves sharing each activation stage) when both
    // scale buffers fit beside two 32 KB code slots and four activation
    // slots; otherwise 128 rows.
    auto plan = [&](int rows, int &cslots, int &xslots, int &fixed) {
        for (cslots = kMaxCodeSlots; cslots >= 1; --cslots) {
            if (rows == 256 && cslots > 2) continue;
            fixed = 1024 + (int)gemm_smem(member, n, rows, 0, cslots).bars + bar_bytes(member);
            xslots = (kSmemCap - fixed) / x_slot_bytes(L.tok_cap);
            if (xslots >= kMinXSlots) break;
        }
        if (xslots > kMaxXSlots) xslots = kMaxXSlots;
        return cslots >= 1 && xslots >= kMinXSlots;
    };
    int cslots = 0, xslots = 0, fixed = 0, rows = 256;
    if (!plan(256, cslots, xslots, fixed)) {
        rows = 128;
        if (!plan(128, cslots, xslots, fixed)) return cudaErrorInvalidConfiguration;
    }
    ga.rblocks = (int)((ga.rows_out + rows - 1) / rows);
    ga.xslots = xslots;
    ga.cslots = cslots;
    const int smem = fixed + xslots * x_slot_bytes(L.tok_cap);
    CUtensorMap qmap;
    XMaps xmap{};
    // codes: [E * out rows, n / 4 bytes], 128 rows x 128 B boxes (512 weights), 128-byte
    // swizzle; IQ1_S_R4 [E * out rows, n / 8 bytes], 128 rows x 64 B, 64-byte swizzle
    const bool iq1 = member == IQK_IQ1_S_R4;
    const uint64_t qrow = iq1 ? (uint64_t)n / 8 : (uint64_t)n / 4;
    cudaError_t err = encode_map(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, streams[0], qrow,
                                 (uint64_t)(num_experts * out_features), qrow,
                                 iq1 ? kCodeK / 8 : kCodeK / 4, kGroupRows,
                                 iq1 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
    if (err != cudaSuccess) return err;
    // activations: [pairs rows, n] f16, boxes of 64 elements x (16 .. tok_cap) rows,
    // 128-byte swizzle
    for (int i = 0; i < L.tok_cap / 16; ++i) {
        err = encode_map(&xmap.m[i], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ga.ws + L.xs, (uint64_t)n,
                         (uint64_t)pairs, (uint64_t)n * 2, 64, 16 * (i + 1),
                         CU_TENSOR_MAP_SWIZZLE_128B);
        if (err != cudaSuccess) return err;
    }
    const int64_t max_items = L.max_tiles * ga.rblocks;
    int64_t blocks = max_items < num_sms ? max_items : num_sms;
    if (blocks < 1) blocks = 1;
    // The shared-memory opt-in (to the largest plan) is a per-device
    // function attribute: set once.
    static std::atomic<unsigned> attr_done[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = -1;
#define IQK_GG(M, R)                                                                           \
    do {                                                                                       \
        const unsigned bit = 1u << ((M) * 2 + (R) - 1);                                        \
        if (dev < 0 || !(attr_done[dev].load() & bit)) {                                       \
            err = cudaFuncSetAttribute(grouped_gemm_kernel<M, R>,                              \
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap); \
            if (err != cudaSuccess) return err;                                                \
            if (dev >= 0) attr_done[dev].fetch_or(bit);                                        \
        }                                                                                      \
        grouped_gemm_kernel<M, R><<<(unsigned)blocks, kThreadsG, smem, stream>>>(ga, qmap,     \
                                                                                 xmap);        \
    } while (0)
    if (member == IQK_IQ2_KS) {
        if (rows == 256) IQK_GG(IQK_IQ2_KS, 2);
        else IQK_GG(IQK_IQ2_KS, 1);
    } else if (member == IQK_IQ2_K) {
        if (rows == 256) IQK_GG(IQK_IQ2_K, 2);
        else IQK_GG(IQK_IQ2_K, 1);
    } else {
        if (rows == 256) IQK_GG(IQK_IQ1_S_R4, 2);
        else IQK_GG(IQK_IQ1_S_R4, 1);
    }
#undef IQK_GG
    return cudaGetLastError();
}

}  // namespace iqk
