// Grouped per-expert GEMM for the prefill route (sm_100a, tcgen05 + TMEM).
//
//   y[p, r] = sum_k W[sel[p], r, k] * x[tok[p], k]   for every routed pair p
//
// Reference: the prefill route of IqkSwitchLinear.__call__
// (src/mlx_iqk/nn.py:221-238): a full fp16 dequantization of the stacked
// experts followed by mx.gather_mm over (optionally sorted) indices. Here the
// weights are never materialised in HBM: each expert's relayout streams are
// read once per 128-token tile and dequantized tile by tile straight into
// tensor memory, where they are the A operand of tcgen05.mma.
//
// Numerics. Activations are scaled per row by a power of two 2^S (so the row
// maximum lies in [2^14, 2^15)) and converted to f16 -- exact for bf16 input.
// IQ2_KS weights enter the MMA as the exact small integers idx * value
// (|.| <= 496, exact in f16); the row's f16 scale is applied in the epilogue.
// IQ2_K weights enter as f16(d_sb * 2^-E * idx) * value with E the row's
// largest super-block exponent, so only two f16 roundings separate them from
// the CPU's float weights. Products are exact and accumulate in f32.
//
// Preparation (two launches): a single-block routing kernel counting-sorts
// the pairs by expert and cuts each expert's run into tiles of at most 128
// tokens; a conversion kernel writes each routed pair's scaled, permuted f16
// activation row in sorted order.
//
// GEMM kernel: persistent, one CTA per SM, 12 warps.
//   warp 0      TMA producer: per 128-weight k-stage, the 128 x 32 B code tile
//               (32-byte swizzle) and the tile's activation rows (two 64-wide
//               k atoms in the 128-byte swizzle, 16-row boxes)
//   warp 1      TMEM owner and MMA issuer (one thread): 8 x M128 N<=128 K16
//               MMAs per stage, A from TMEM, B from shared memory
//   warps 4-11  dequantize: two warps per TMEM lane quarter take alternate
//               stages; each thread expands its row's 128 codes into 64 f16x2
//               words with byte permutes on a per-group table of the four
//               alphabet products, and stores them to TMEM (tcgen05.st);
//               then the epilogue (tcgen05.ld of D, scale, store y)
// Work items are (tile, 128-row block), expert-major, so CTAs running at the
// same time share one expert's activation tile in L2.
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

#include "iqk_common.cuh"
#include "iqk_grouped.cuh"
#include "iqk_sync.cuh"

namespace iqk {
namespace {

using namespace dev;

constexpr int kThreadsG = 384;
constexpr int kProducer = 0, kIssuer = 1, kDq0 = 4;
constexpr int kStageK = 128;                        // weights per k-stage
constexpr int kStagesG = 4;
constexpr int kCodeTile = kGroupRows * kStageK / 4;  // 4 KB of 2-bit codes
constexpr int kXAtom = kGroupTok * 128;             // 16 KB: 128 rows x 64 f16
constexpr int kXTile = 2 * kXAtom;
constexpr int kStageBytesG = kXTile + kCodeTile;     // 36 KB, 1024-aligned
constexpr int kTmemCols = 512;
constexpr int kDCol = 0;                             // D: columns [0, 128)
constexpr int kACol = 128;                           // A: 4 stages x 64 columns
constexpr int kBarBytes = 8 * (3 * kStagesG + 3) + 16;
constexpr int kSmemG = 1024 + kStagesG * kStageBytesG + kBarBytes;

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
// most kGroupTok tokens. Shared memory: counts, then scatter cursors.
__global__ void __launch_bounds__(1024)
grouped_route_kernel(const int32_t *__restrict__ sel, const int32_t *__restrict__ tok, int pairs,
                     int x_rows, int num_experts, GroupedLayout L, char *ws) {
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
        if (e < 0 || e >= num_experts) err |= IQK_DEVERR_EXPERT;
        else if (t < 0 || t >= x_rows) err |= IQK_DEVERR_TOKEN;
        else atomicAdd(&cnt[e], 1);
    }
    if (err) atomicOr(&s_bad, err);
    __syncthreads();
    const int per = (num_experts + nt - 1) / nt;
    const int b0 = min(tid * per, num_experts), b1 = min(b0 + per, num_experts);
    int c_cnt = 0, c_tiles = 0;
    for (int e = b0; e < b1; ++e) {
        c_cnt += cnt[e];
        c_tiles += (cnt[e] + kGroupTok - 1) / kGroupTok;
    }
    int n_valid, n_tiles;
    int run = block_scan(c_cnt, warp_tot, &n_valid);
    int trun = block_scan(c_tiles, warp_tot, &n_tiles);
    for (int e = b0; e < b1; ++e) {
        const int c = cnt[e];
        for (int i = 0; i * kGroupTok < c; ++i)
            tiles[trun++] = make_int4(e, run + i * kGroupTok, min(kGroupTok, c - i * kGroupTok), 0);
        cnt[e] = run;  // becomes the scatter cursor
        run += c;
    }
    if (tid == 0) {
        hdr[0] = s_bad;
        hdr[1] = n_tiles;
        hdr[2] = n_valid;
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
    const int S = (bad || amax == 0.f) ? 0 : 14 - ilogbf(amax);
    if (tid == 0) {
        reinterpret_cast<int32_t *>(ws + L.pscale)[pos] = S;
        if (bad) atomicOr(reinterpret_cast<int32_t *>(ws + L.hdr), IQK_DEVERR_NONFINITE);
    }
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
        uint4 *dst = reinterpret_cast<uint4 *>(
            reinterpret_cast<__half *>(ws + L.xs) + (int64_t)pos * n + tid * 16);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
}

// ------------------------------------------------------------- GEMM kernel

struct GroupedArgs {
    const void *s[5];
    int64_t out_features;
    int n, pairs, rblocks;
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

template <int MEMBER>
__global__ void __launch_bounds__(kThreadsG, 1)
grouped_gemm_kernel(const GroupedArgs a, const __grid_constant__ CUtensorMap qs_map,
                    const __grid_constant__ CUtensorMap x_map) {
    extern __shared__ char smem_raw[];
    char *smem = smem_raw + ((1024u - (saddr(smem_raw) & 1023u)) & 1023u);
    const uint32_t stage_u = saddr(smem);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + kStagesG * kStageBytesG);
    uint64_t *aready = full + kStagesG;
    uint64_t *empty = aready + kStagesG;
    uint64_t *dfull = empty + kStagesG;
    uint64_t *dempty = dfull + 1;
    uint64_t *drain = dempty + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int32_t *hdr = reinterpret_cast<const int32_t *>(a.ws + a.L.hdr);
    const int4 *tiles = reinterpret_cast<const int4 *>(a.ws + a.L.tiles);
    const int32_t *order = reinterpret_cast<const int32_t *>(a.ws + a.L.order);
    const int32_t *pscale = reinterpret_cast<const int32_t *>(a.ws + a.L.pscale);
    const int n = a.n, KS = n / kStageK;
    const int64_t out = a.out_features;
    const int ntiles = hdr[1], n_valid = hdr[2];
    const int64_t items = (int64_t)ntiles * a.rblocks;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kStagesG; ++i) {
            bar_init(&full[i], 1);
            bar_init(&aready[i], 4);
            bar_init(&empty[i], 1);
        }
        bar_init(dfull, 1);
        bar_init(dempty, 8);
        bar_init(drain, 1);
        *abort_flag = 0;
        bar_fence_init();
    }
    if (warp == kIssuer) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
        tc_fence_before();
    }
    // Zero the outputs of unroutable pairs (bad expert or row index).
    {
        const int tail = a.pairs - n_valid;
        const int64_t total = (int64_t)tail * out;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
             i += (int64_t)gridDim.x * blockDim.x) {
            const int64_t p = order[n_valid + i / out];
            const int64_t r = i % out;
            if (a.y_dtype == IQK_F32) store_out<float>(a.y, p * out + r, 0.f);
            else if (a.y_dtype == IQK_F16) store_out<__half>(a.y, p * out + r, 0.f);
            else store_out<__nv_bfloat16>(a.y, p * out + r, 0.f);
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
        if (lane == 0) {
            int g = 0;
            for (int64_t it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x) {
                const int4 tl = tiles[it / a.rblocks];
                const int rb = (int)(it % a.rblocks);
                const int npad = (tl.z + 15) & ~15;
                const int row0 = (int)((int64_t)tl.x * out + (int64_t)rb * kGroupRows);
                const uint32_t bytes = (uint32_t)(kCodeTile + 2 * npad * 128);
                for (int ks = 0; ks < KS; ++ks, ++g) {
                    const int slot = g % kStagesG;
                    const uint32_t use = (uint32_t)(g / kStagesG);
                    if (!bar_wait(&empty[slot], (use & 1u) ^ 1u, abort_flag)) {
                        give_up();
                        break;
                    }
                    const uint32_t st = stage_u + slot * kStageBytesG;
                    bar_expect_tx(&full[slot], bytes);
                    tma_2d(st + kXTile, &qs_map, ks * (kStageK / 4), row0, &full[slot]);
#pragma unroll 1
                    for (int atom = 0; atom < 2; ++atom)
#pragma unroll 1
                        for (int b = 0; b < npad; b += 16)
                            tma_2d(st + atom * kXAtom + b * 128, &x_map,
                                   ks * kStageK + atom * 64, tl.y + b, &full[slot]);
                }
            }
            // Drain: the last stages' copies must land before the CTA exits,
            // aborted or not (bounded by time only).
            for (int d = 0; d < kStagesG && d < g; ++d) {
                const int gg = g - 1 - d;
                if (!bar_wait(&full[gg % kStagesG], (uint32_t)(gg / kStagesG) & 1u, nullptr))
                    give_up();
            }
        }
        __syncwarp();
    } else if (warp == kIssuer) {
        if (lane == 0) {
            int g = 0, item_i = 0;
            for (int64_t it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x, ++item_i) {
                const int4 tl = tiles[it / a.rblocks];
                const int npad = (tl.z + 15) & ~15;
                const uint32_t idesc = idesc_f16(kGroupRows, npad);
                if (item_i > 0 && !bar_wait(dempty, (uint32_t)(item_i - 1) & 1u, abort_flag)) {
                    give_up();
                    break;
                }
                tc_fence_after();
                bool ok = true;
                for (int ks = 0; ks < KS; ++ks, ++g) {
                    const int slot = g % kStagesG;
                    const uint32_t par = (uint32_t)(g / kStagesG) & 1u;
                    if (!bar_wait(&full[slot], par, abort_flag) ||
                        !bar_wait(&aready[slot], par, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t st = stage_u + slot * kStageBytesG;
#pragma unroll
                    for (int kk = 0; kk < 8; ++kk) {
                        const uint64_t bdesc = sw128_desc(st + (kk >> 2) * kXAtom + (kk & 3) * 32);
                        tc_mma_ts(tmem + kDCol, tmem + kACol + slot * 64 + kk * 8, bdesc, idesc,
                                  (ks | kk) != 0);
                    }
                    tc_commit(&empty[slot]);
                }
                if (!ok) {
                    give_up();
                    break;
                }
                tc_commit(dfull);
            }
            // Every MMA issued must finish before tensor memory is freed.
            tc_commit(drain);
            if (!bar_wait(drain, 0, nullptr)) give_up();
        }
        __syncwarp();
    } else if (warp >= kDq0) {
        const int dq = warp - kDq0;
        const int q = warp & 3;        // TMEM lane quarter this warp may access
        const int h = dq >> 2;         // stage parity this warp dequantizes
        const int rloc = 32 * q + lane;
        const uint32_t lane_base = (uint32_t)(32 * q) << 16;
        const uint32_t sw = (uint32_t)((rloc >> 2) & 1);  // 32-byte swizzle of this row
        int g = 0, item_i = 0;
        for (int64_t it = blockIdx.x; it < items && !*abort_flag; it += gridDim.x, ++item_i) {
            const int4 tl = tiles[it / a.rblocks];
            const int rb = (int)(it % a.rblocks);
            const int npad = (tl.z + 15) & ~15;
            const int64_t rlocal = (int64_t)rb * kGroupRows + rloc;
            const bool row_ok = rlocal < out;
            const int64_t row = (int64_t)tl.x * out + (row_ok ? rlocal : 0);
            float rscale;  // epilogue factor of this row (before 2^-S)
            float dnorm = 1.f;  // IQ2_K: 2^-E applied to the super-block scales
            if (MEMBER == IQK_IQ2_KS) {
                rscale = half_bits_to_float(static_cast<const uint16_t *>(a.s[4])[row]);
            } else {
                const uint16_t *dv = static_cast<const uint16_t *>(a.s[3]) + row * (n / 256);
                float m = 0.f;
                for (int i = 0; i < n / 256; ++i) m = fmaxf(m, fabsf(half_bits_to_float(dv[i])));
                const int E = m > 0.f ? ilogbf(m) + 1 : 0;
                dnorm = ldexpf(1.f, -E);
                rscale = ldexpf(1.f, E);
            }
            for (int ks = 0; ks < KS; ++ks, ++g) {
                if ((g & 1) != h) continue;
                const int slot = g % kStagesG;
                const uint32_t par = (uint32_t)(g / kStagesG) & 1u;
                // Scale bytes of this stage (global, cached in L1 across stages).
                uint32_t sc0, sc1;
                if (MEMBER == IQK_IQ2_KS) {
                    const uint8_t *scl = static_cast<const uint8_t *>(a.s[1]);
                    const uint8_t *sch = static_cast<const uint8_t *>(a.s[2]);
                    const uint8_t *sex = static_cast<const uint8_t *>(a.s[3]);
                    const int sh = 4 * (ks & 1);
                    sc0 = *reinterpret_cast<const uint16_t *>(scl + row * (n / 64) + 2 * ks);
                    sc1 = ((uint32_t)(sch[row * (n / 256) + (ks >> 1)] >> sh) & 15u) |
                          (((uint32_t)(sex[row * (n / 256) + (ks >> 1)] >> sh) & 15u) << 4);
                } else {
                    const uint8_t *scl = static_cast<const uint8_t *>(a.s[1]);
                    const uint8_t *sex = static_cast<const uint8_t *>(a.s[2]);
                    const uint16_t *dv = static_cast<const uint16_t *>(a.s[3]);
                    sc0 = *reinterpret_cast<const uint32_t *>(scl + row * (n / 32) + 4 * ks);
                    sc1 = (uint32_t)sex[row * (n / 128) + ks] |
                          ((uint32_t)dv[row * (n / 256) + (ks >> 1)] << 16);
                }
                if (!bar_wait(&full[slot], par, abort_flag) ||
                    !bar_wait(&empty[slot], par ^ 1u, abort_flag)) {
                    give_up();
                    break;
                }
                tc_fence_after();
                const uint32_t code_u = stage_u + slot * kStageBytesG + kXTile + rloc * 32;
                const uint4 c0 = lds128(code_u + ((0u ^ sw) << 4));
                const uint4 c1 = lds128(code_u + ((1u ^ sw) << 4));
                const uint32_t words[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                float dsb = 0.f;
                if (MEMBER == IQK_IQ2_K) dsb = half_bits_to_float((uint16_t)(sc1 >> 16)) * dnorm;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    uint32_t r[32];
#pragma unroll
                    for (int wi = 0; wi < 4; ++wi) {
                        const int wd = 4 * half + wi;  // word within the stage
                        uint32_t t01, t23;
                        if (MEMBER == IQK_IQ2_KS) {
                            const int gq = wd >> 1;    // 32-weight group within the stage
                            const int idx = (int)(((sc0 >> (4 * gq)) & 15u) |
                                                  (((sc1 >> gq) & 1u) << 4)) - 16;
                            const int alpha = (int)((sc1 >> (4 + gq)) & 1u);
                            const uint32_t hi = h2_bcast((float)idx);
                            t01 = hmul2_bits(hi, alpha ? kV01a1 : kV01a0);
                            t23 = hmul2_bits(hi, alpha ? kV23a1 : kV23a0);
                        } else {
                            const int idx = (int)((sc0 >> (4 * wd)) & 15u) - 8;
                            const int alpha = (int)((sc1 >> wd) & 1u);
                            const uint32_t hi = h2_bcast(dsb * (float)idx);
                            t01 = hmul2_bits(hi, alpha ? kV01a1 : kV01a0);
                            t23 = hmul2_bits(hi, alpha ? kV23a1 : kV23a0);
                        }
                        expand_word(words[wd], t01, t23, &r[8 * wi]);
                    }
                    tmem_st32(tmem + lane_base + kACol + slot * 64 + half * 32, r);
                }
                tc_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) bar_arrive(&aready[slot]);
            }
            if (*abort_flag) break;
            // Epilogue: D rows are this thread's output row, columns the tile's tokens.
            if (!bar_wait(dfull, (uint32_t)item_i & 1u, abort_flag)) {
                give_up();
                break;
            }
            tc_fence_after();
            for (int c = 8 * h; c < npad; c += 16) {
                uint32_t d[8];
                tmem_ld8(tmem + lane_base + kDCol + c, d);
                tc_wait_ld();
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int col = c + j;
                    if (col < tl.z && row_ok) {
                        const int64_t p = order[tl.y + col];
                        const int S = pscale[tl.y + col];
                        const float v = ldexpf(__uint_as_float(d[j]) * rscale, -S);
                        const int64_t o = p * out + rlocal;
                        if (a.y_dtype == IQK_F32) store_out<float>(a.y, o, v);
                        else if (a.y_dtype == IQK_F16) store_out<__half>(a.y, o, v);
                        else store_out<__nv_bfloat16>(a.y, o, v);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) bar_arrive(dempty);
        }
    }
    __syncthreads();
    if (warp == kIssuer) {
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
    L.max_tiles = (num_experts < pairs ? num_experts : pairs) + pairs / kGroupTok + 1;
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
                                   int64_t pairs, void *ws, cudaStream_t stream) {
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
                                                    (int)num_experts, L, w);
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
                               const void *ws, cudaStream_t stream, int num_sms) {
    const GroupedLayout L = grouped_layout(n, num_experts, pairs);
    GroupedArgs ga{};
    const RowBytes rb = row_bytes(member, n);
    for (int i = 0; i < rb.count; ++i) ga.s[i] = streams[i];
    ga.out_features = out_features;
    ga.n = n;
    ga.pairs = (int)pairs;
    ga.rblocks = (int)((out_features + kGroupRows - 1) / kGroupRows);
    ga.ws = static_cast<const char *>(ws);
    ga.L = L;
    ga.err = reinterpret_cast<int32_t *>(const_cast<char *>(ga.ws) + L.hdr);
    ga.y = y;
    ga.y_dtype = y_dtype;
    CUtensorMap qmap, xmap;
    // codes: [E * out rows, n / 4 bytes], 128 rows x 32 B boxes, 32-byte swizzle
    cudaError_t err = encode_map(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, streams[0], (uint64_t)n / 4,
                                 (uint64_t)(num_experts * out_features), (uint64_t)n / 4,
                                 kStageK / 4, kGroupRows, CU_TENSOR_MAP_SWIZZLE_32B);
    if (err != cudaSuccess) return err;
    // activations: [pairs rows, n] f16, 16 rows x 64 elements, 128-byte swizzle
    err = encode_map(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ga.ws + L.xs, (uint64_t)n,
                     (uint64_t)pairs, (uint64_t)n * 2, 64, 16, CU_TENSOR_MAP_SWIZZLE_128B);
    if (err != cudaSuccess) return err;
    const int64_t max_items = L.max_tiles * ga.rblocks;
    int64_t blocks = max_items < num_sms ? max_items : num_sms;
    if (blocks < 1) blocks = 1;
#define IQK_GG(M)                                                                              \
    do {                                                                                       \
        err = cudaFuncSetAttribute(grouped_gemm_kernel<M>,                                     \
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemG);       \
        if (err != cudaSuccess) return err;                                                    \
        grouped_gemm_kernel<M><<<(unsigned)blocks, kThreadsG, kSmemG, stream>>>(ga, qmap, xmap); \
    } while (0)
    if (member == IQK_IQ2_KS) IQK_GG(IQK_IQ2_KS);
    else if (member == IQK_IQ2_K) IQK_GG(IQK_IQ2_K);
    else return cudaErrorInvalidValue;
#undef IQK_GG
    return cudaGetLastError();
}

}  // namespace iqk
