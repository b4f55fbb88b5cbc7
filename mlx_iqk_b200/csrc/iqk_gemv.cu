// Fused relayout-stream dequant + GEMV for few-token decode (sm_100a).
//
// y[p, r] = sum_k W[sel[p], r, k] * x[tok[p], k]    for every pair p.
//
// Reference: the Metal decode GEMVs (src/mlx_iqk/kernels.py:332-572,
// launched at src/mlx_iqk/nn.py:240-333). This is not a translation of them;
// the arithmetic is organised for integer tensor cores:
//
// * Activations are prepared once per call (prep kernel): each row x[t] is
//   scaled by a power of two 2^S_t so max|x| < 2^22, rounded to an integer,
//   and split into three signed 8-bit digit planes (x_int = 65536*h + 256*m
//   + l), stored in the B-operand order of the MMA below.
// * Weights are never materialised. Each 2-bit code (or ternary grid value)
//   becomes its int8 alphabet value through a byte permute whose selector
//   nibble is (code | 4*alphabet), straight into an mma.sync.m16n8k32 s8 A
//   fragment; the digit planes are the B operand. The tensor core returns
//   exact int32 sums per 32-weight group, scaled by the group's integer scale
//   index with IMAD: the whole reduction is exact integer arithmetic until
//   one final double-precision multiply by the fp16 row (or super-block)
//   scale and 2^-S_t.
// * So every output is independent of reduction order and of how pairs are
//   grouped: a sorted or unioned call is bit-identical to the per-pair call,
//   and the only approximation is x's 22-bit rounding.
// * Routing is on the device: pairs are bucketed by expert, so the work tiles
//   of one expert are adjacent and the CTAs that run them at the same time
//   read the expert's rows from DRAM once (the later reads hit L2). This
//   covers the reference's sorted and "union" formulations
//   (src/mlx_iqk/kernels.py:404-572) for every member.
//
// Run kernel layout. A CTA item is (pair, 64-row block): four compute warps
// each own 16 rows for all of k, one producer warp streams the item through
// a four-stage ring of TMA boxes (16 rows x 128 code bytes per warp and
// round) plus the round's slice of activation planes, and the item's scale
// streams arrive in one of two double-buffered scale slots. Per round each
// warp expands its rows' group metadata (alphabet mask, integer scale) into
// shared memory, then runs 8 MMA pairs of 64 weights; the metadata of round
// r+1 is built during round r (two buffers per warp) so its shared-memory
// latency overlaps the MMA work. The operand build is bound by the integer
// ALU pipe (byte permutes and logic ops, issued every other cycle per
// scheduler), so the shift by two of each code word goes through mul.hi on
// the FMA pipe and the metadata is expanded four groups at a time with
// byte-SIMD multiplies. Items are split evenly over one persistent wave of
// CTAs (as many per SM as shared memory and registers allow).
#include <cuda.h>

#include <atomic>

#include "iqk_common.cuh"
#include "iqk_gemv.cuh"
#include "iqk_tables.cuh"

namespace iqk {

// ------------------------------------------------------------------ helpers

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void mma_s8(int32_t d[4], const uint32_t a[4], uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}

// Programmatic dependent launch (PTX griddepcontrol). Both decode kernels are
// launched with programmatic stream serialization: a kernel may start while
// the previous kernel of the stream is still draining, does its shared-memory
// set-up, then waits for that kernel's completion (and its memory) before it
// reads or writes any global memory, and at once lets the next kernel start.
__device__ __forceinline__ void grid_dep_wait() {
    asm volatile("griddepcontrol.wait;\n" ::: "memory");
}
__device__ __forceinline__ void grid_dep_launch() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// ------------------------------------------------------------- prep kernel

// One block per activation row: digit planes, block sums and the exponent.
// Row layout in the workspace: planes [n/64 pairs][4 code words][3 planes]
// [16 bytes] -- for the 16 weights of a code word: bytes 0-3 the even k of
// its first 8, 4-7 the odd k, 8-11 / 12-15 the same for its last 8 -- then
// block sums [n/32][4] int32 (per 32-weight block, planes 0..2, 0).
template <typename XT>
__device__ void prep_row(const XT *__restrict__ x, int n, int row, const GemvLayout &L,
                         char *ws) {
    __shared__ float red_max[32];
    __shared__ int red_bad[32];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int noct = n / 8;  // octets: (k-step s = q / 4, lane-in-quad = q % 4)
    const XT *xr = x + (int64_t)row * n;
    float v[2][8];
    float amax = 0.f;
    int bad = 0;
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        const int q = tid + it * blockDim.x;
        if (q < noct) {
            // one octet = 8 consecutive activations: 16 or 32 bytes, vector loads
            if (sizeof(XT) == 2) {
                const uint4 u = *reinterpret_cast<const uint4 *>(xr + q * 8);
                const XT *h = reinterpret_cast<const XT *>(&u);
#pragma unroll
                for (int j = 0; j < 8; ++j) v[it][j] = to_float<XT>(h[j]);
            } else {
                const float4 a = *reinterpret_cast<const float4 *>(xr + q * 8);
                const float4 b = *reinterpret_cast<const float4 *>(xr + q * 8 + 4);
                v[it][0] = a.x; v[it][1] = a.y; v[it][2] = a.z; v[it][3] = a.w;
                v[it][4] = b.x; v[it][5] = b.y; v[it][6] = b.z; v[it][7] = b.w;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float f = v[it][j];
                if (!isfinite(f)) bad = 1;
                else amax = fmaxf(amax, fabsf(f));
            }
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        bad |= __shfl_xor_sync(0xffffffffu, bad, o);
    }
    if (lane == 0) {
        red_max[wid] = amax;
        red_bad[wid] = bad;
    }
    __syncthreads();
    if (wid == 0) {
        const int nw = blockDim.x / 32;
        amax = lane < nw ? red_max[lane] : 0.f;
        bad = lane < nw ? red_bad[lane] : 0;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            bad |= __shfl_xor_sync(0xffffffffu, bad, o);
        }
        if (lane == 0) {
            red_max[0] = amax;
            red_bad[0] = bad;
        }
    }
    __syncthreads();
    amax = red_max[0];
    bad = red_bad[0];
    // |x| * 2^S < 2^22 keeps the top digit inside int8 after the balanced split.
    const int S = amax > 0.f ? 21 - ilogbf(amax) : 0;
    if (tid == 0) {
        int32_t *xs = reinterpret_cast<int32_t *>(ws + L.xscale);
        xs[row] = bad ? kScaleNonFinite : S;
    }
    int8_t *xb = reinterpret_cast<int8_t *>(ws + L.xbuf) + (int64_t)row * L.xrow_bytes;
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        const int q = tid + it * blockDim.x;
        if (q >= noct) continue;  // uniform per warp: noct is a multiple of 256
        const int s = q >> 2, tig = q & 3;
        uint32_t planes[3][2] = {{0, 0}, {0, 0}, {0, 0}};
        int bsum[3] = {0, 0, 0};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int xi = bad ? 0 : __float2int_rn(ldexpf(v[it][j], S));
            const int lo = ((xi + 128) & 255) - 128;
            const int r1 = (xi - lo) >> 8;
            const int mid = ((r1 + 128) & 255) - 128;
            const int hi = (r1 - mid) >> 8;
            const int dig[3] = {hi, mid, lo};
#pragma unroll
            for (int p = 0; p < 3; ++p) {
                planes[p][j & 1] |= (uint32_t)(uint8_t)(int8_t)dig[p] << (8 * (j >> 1));
                bsum[p] += dig[p];
            }
        }
        // pair of groups (64 weights) q/8, code word (16 weights) (q/2)%4, half q%2
        int8_t *dst = xb + (int64_t)(q >> 3) * 192 + ((q >> 1) & 3) * 48 + (q & 1) * 8;
#pragma unroll
        for (int p = 0; p < 3; ++p)
            *reinterpret_cast<uint2 *>(dst + p * 16) = make_uint2(planes[p][0], planes[p][1]);
        // Block sums over the 32 weights of k-step s: reduce across the quad.
#pragma unroll
        for (int p = 0; p < 3; ++p) {
            bsum[p] += __shfl_xor_sync(0xffffffffu, bsum[p], 1);
            bsum[p] += __shfl_xor_sync(0xffffffffu, bsum[p], 2);
        }
        if (tig == 0)
            *reinterpret_cast<int4 *>(xb + 3 * (int64_t)n + (int64_t)s * 16) =
                make_int4(bsum[0], bsum[1], bsum[2], 0);
    }
}

// Block-wide exclusive scan of one int per thread (warp shuffles + one
// shared array of warp totals). Returns the exclusive prefix; *total = sum.
__device__ __forceinline__ int block_exclusive_scan(int v, int *warp_tot, int *total) {
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
        if (lane < nw) warp_tot[lane] = winc - w;  // exclusive warp offsets
        if (lane == nw - 1) warp_tot[32] = winc;
    }
    __syncthreads();
    const int excl = warp_tot[wid] + inc - v;
    *total = warp_tot[32];
    __syncthreads();
    return excl;
}

// Route the pairs: bucket by expert (counting sort in shared memory) and lay
// out the work tiles -- one per routable pair, grouped by expert -- written
// directly by the thread that places each pair. Pairs whose expert or row
// index is out of range go to the tail of `order` (the run kernel zeroes
// their outputs) and set the device error word.
// Shared memory: per-expert counts, then scatter cursors (num_experts ints).
__device__ void route_pairs(const int32_t *__restrict__ sel, const int32_t *__restrict__ tok,
                            int pairs, int x_rows, int num_experts, const GemvLayout &L,
                            char *ws) {
    extern __shared__ int32_t cur[];
    __shared__ int32_t warp_tot[33];
    __shared__ int32_t s_bad, s_tail;
    const int tid = threadIdx.x, nt = blockDim.x;
    int32_t *hdr = reinterpret_cast<int32_t *>(ws + L.hdr);
    int32_t *order = reinterpret_cast<int32_t *>(ws + L.order);
    TileRef *tiles = reinterpret_cast<TileRef *>(ws + L.tiles1);
    for (int e = tid; e < num_experts; e += nt) cur[e] = 0;
    if (tid == 0) s_bad = 0;
    __syncthreads();
    const int dims = tok ? 1 : pairs / x_rows;
    int err = 0;
    for (int p = tid; p < pairs; p += nt) {
        const int e = sel[p];
        const int t = tok ? tok[p] : p / dims;
        if (e < 0 || e >= num_experts) err |= IQK_DEVERR_EXPERT;
        else if (t < 0 || t >= x_rows) err |= IQK_DEVERR_TOKEN;
        else atomicAdd(&cur[e], 1);
    }
    if (err) atomicOr(&s_bad, err);
    __syncthreads();
    // thread-contiguous bins; exclusive scan of the per-expert counts
    const int per = (num_experts + nt - 1) / nt;
    const int b0 = min(tid * per, num_experts), b1 = min(b0 + per, num_experts);
    int c_cnt = 0;
    for (int e = b0; e < b1; ++e) c_cnt += cur[e];
    int n_valid;
    int run = block_exclusive_scan(c_cnt, warp_tot, &n_valid);
    for (int e = b0; e < b1; ++e) {
        const int c = cur[e];
        cur[e] = run;
        run += c;
    }
    if (tid == 0) {
        hdr[0] = s_bad;
        hdr[3] = n_valid;  // work tiles == routable pairs
        s_tail = n_valid;
    }
    __syncthreads();
    for (int p = tid; p < pairs; p += nt) {
        const int e = sel[p];
        const int t = tok ? tok[p] : p / dims;
        const bool ok = e >= 0 && e < num_experts && t >= 0 && t < x_rows;
        if (!ok) {
            order[atomicAdd(&s_tail, 1)] = p;
            continue;
        }
        const int pos = atomicAdd(&cur[e], 1);
        order[pos] = p;
        tiles[pos] = TileRef{e, p, -1, t, -1, 0, 0, 1};
    }
}

template <typename XT>
__global__ void __launch_bounds__(256)
gemv_prep_kernel(const XT *__restrict__ x, int n, int x_rows, const int32_t *__restrict__ sel,
                 const int32_t *__restrict__ tok, int pairs, int num_experts, GemvLayout L,
                 char *__restrict__ ws) {
    grid_dep_wait();
    grid_dep_launch();
    if ((int)blockIdx.x < x_rows) {
        prep_row<XT>(x, n, blockIdx.x, L, ws);
    } else {
        if (threadIdx.x == 0) {
            int32_t *h = reinterpret_cast<int32_t *>(ws + L.hdr);
            h[8] = 0;  // the run kernels' work counter (items claimed)
            h[9] = 0;  // and the count of their CTAs done (the last one resets both)
        }
        route_pairs(sel, tok, pairs, x_rows, num_experts, L, ws);
    }
}

// -------------------------------------------------------------- run kernel

constexpr int kConsumers = 4;                 // compute warps: 16 rows x all of k each
constexpr int kThreads = (kConsumers + 1) * 32;  // + one producer warp
constexpr int kItemRows = 16 * kConsumers;    // 64 rows per CTA item
constexpr int kChunkK = 512;                  // weights per row per round and warp
constexpr int kPairsPerRound = kChunkK / 64;  // MMA pairs (64 weights per row) per round
constexpr int kMaxTiles = 64;                 // tile entries cached in shared memory
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // bounded mbarrier waits (2 s)

// One work tile is one pair (expert, activation row). A warp's 16 rows x 64
// weights form an "MMA pair": two m16n8k32 products whose A fragments come
// from one 32-bit code word per lane and row.
template <int MEMBER> struct Geo {
    // Four-stage rings; three CTAs per SM (two for IQ2_K, whose scale
    // streams and metadata are twice as large). IQ1_S_R4, whose scale slots
    // are the largest and whose grid table also sits in shared memory, takes
    // three stages and a 32-entry tile cache, so that three CTAs fit.
    static constexpr int kStages = MEMBER == IQK_IQ1_S_R4 ? 3 : 4;
    static constexpr int kTileCache = MEMBER == IQK_IQ1_S_R4 ? 32 : kMaxTiles;
    static constexpr int kMinBlocks = MEMBER == IQK_IQ2_K ? 2 : 3;
    static constexpr int kRowChunk = MEMBER == IQK_IQ1_S_R4 ? 64 : 128;   // qs bytes per round
    static constexpr int kWBox = 16 * kRowChunk;                         // one warp's TMA box
    static constexpr int kWBytes = kConsumers * kWBox;
    static constexpr int kXPlanes = kPairsPerRound * 192;                  // 3 planes
    static constexpr int kXSums = MEMBER == IQK_IQ1_S_R4 ? kPairsPerRound * 32 : 0;
    static constexpr int kXBlock = kXPlanes + kXSums;                      // per round
    static constexpr int kMetaSides = MEMBER == IQK_IQ2_K ? 4 : 2;
    static constexpr int kMetaBytes = kPairsPerRound * kMetaSides * 8 * 16;  // per warp
};

// The scale streams of one member at width N: bytes per row of stream si
// (1 .. kCount-1, component order after qs) and each stream's offset inside
// an item's scale slot (ROWS rows of every stream, back to back).
template <int MEMBER, int N, int ROWS = kItemRows> struct Streams {
    static constexpr int kCount = MEMBER == IQK_IQ2_KS ? 5 : MEMBER == IQK_IQ2_K ? 4 : 3;
    static constexpr __host__ __device__ int b(int si) {
        return MEMBER == IQK_IQ2_KS ? (si == 1 ? N / 64 : si == 4 ? 2 : N / 256)
               : MEMBER == IQK_IQ2_K ? (si == 1 ? N / 32 : si == 2 ? N / 128 : 2 * (N / 256))
                                     : (si == 1 ? N / 16 : 2);
    }
    static constexpr __host__ __device__ int off(int si) {
        return si <= 1 ? 0 : off(si - 1) + ROWS * b(si - 1);
    }
    static constexpr int kSlot = off(kCount);
};

// Stage: [weights: kConsumers TMA boxes][activation slices of KQ chunks],
// released every round. An item's scale streams sit in one of two scale
// slots for the whole item.
template <int MEMBER, int KQ = 1> __host__ __device__ constexpr int stage_bytes() {
    return (Geo<MEMBER>::kWBytes + KQ * Geo<MEMBER>::kXBlock + 1023) / 1024 * 1024;
}
template <int MEMBER, int N, int ROWS = kItemRows> __host__ __device__ constexpr int sslot_bytes() {
    return (Streams<MEMBER, N, ROWS>::kSlot + 127) / 128 * 128;
}

// Two item shapes. Wide: 64 rows x all of k, each compute warp 16 rows x all
// of k. Narrow (few items, e.g. one token): 16 rows x all of k, the four
// compute warps take a quarter of every round's k each and their exact
// partial sums meet in shared memory -- four times the items, so small
// decode batches still reach every SM.
// GLU (wide items only): a SwitchGLU's gate and up together -- an item is
// 32 rows of one pair, warps 0-1 on the gate's rows, warps 2-3 on the same
// rows of up; at item end the up warps hand their results to the gate warps,
// which store h = silu(gate) * up * router weight.
template <int MEMBER, bool NARROW, bool GLU = false> struct Shape {
    static constexpr int kRows = NARROW ? 16 : GLU ? kItemRows / 2 : kItemRows;  // rows per item
    static constexpr int KQ = NARROW ? kConsumers : 1;        // k chunks per round
    static constexpr int kStages = NARROW ? 3 : Geo<MEMBER>::kStages;
    static constexpr int kRedBytes = NARROW ? 2 * kConsumers * 32 * 16 : GLU ? 2 * 2 * 8 * 8 : 0;
    static constexpr int kProj = GLU ? 2 : 1;  // projections whose scale streams fill a slot
};

template <int MEMBER, int N, bool NARROW, bool GLU = false>
__host__ __device__ constexpr int gemv_smem_bytes() {
    using G = Geo<MEMBER>;
    using SH = Shape<MEMBER, NARROW, GLU>;
    return 1024 /* alignment slack */ + SH::kStages * stage_bytes<MEMBER, SH::KQ>() +
           2 * SH::kProj * sslot_bytes<MEMBER, N, SH::kRows>() + 2 * kConsumers * G::kMetaBytes +
           G::kTileCache * (int)sizeof(TileRef) + (MEMBER == IQK_IQ1_S_R4 ? 4096 : 0) +
           2 * SH::kStages * 8 + 8 * 8 + 16 +
           kPairsPerRound * 192 + SH::kRedBytes;
}

struct GemvArgs {
    const void *s[5];
    const void *s2[5];  // GLU: the up projection's streams
    const float *rw;    // GLU: router weight per pair, or null (1)
    int out_features;  // experts x out_features <= 2^30 (checked by the C ABI)
    int pairs;
    uint32_t one;      // 1: source of the mul.hi shift multipliers (see below)
    GemvLayout L;
    const char *ws;
    int32_t *err;  // device error word (workspace header)
    int dynamic;   // 1: CTAs claim whole items from the workspace's work counter
    void *y;
    int y_dtype;
};

__device__ __forceinline__ uint32_t lds_u16(const void *p) {
    return *reinterpret_cast<const uint16_t *>(p);
}
__device__ __forceinline__ uint32_t lds_u32(const void *p) {
    return *reinterpret_cast<const uint32_t *>(p);
}
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// Explicit shared-space accesses on 32-bit addresses.
__device__ __forceinline__ uint32_t ld_s32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];\n" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 ld_s64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 ld_s128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ void st_s128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w)
                 : "memory");
}

// The operand build is bound by the integer ALU pipe (byte permutes, logic
// ops). The code word's shift by two is a plain shift: a multiply-high on the
// FMA pipe issues at a quarter of the ALU's rate on B200 (measured: 0.95
// against 1.84 warp instructions per SM cycle), and the whole kernel measured
// 3 % faster with the shift (38.1 against 39.2 us, IQ2_KS gate at B = 8).
// mulhi stays for the metadata's byte-SIMD spreads.
__device__ __forceinline__ uint32_t mulhi(uint32_t x, uint32_t m) { return __umulhi(x, m); }
__device__ __forceinline__ uint32_t shr2(uint32_t x, uint32_t) { return x >> 2; }
__device__ __forceinline__ uint32_t shr16(uint32_t x) { return x >> 16; }

// d += A * B (int8 m16n8k32, accumulating in place).
__device__ __forceinline__ void mma_s8_acc(int32_t d[4], const uint32_t a[4], uint32_t b0,
                                           uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---- mbarrier / bulk-copy primitives (PTX ISA: mbarrier, cp.async.bulk)
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
                 "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}
// Wait for a phase with a wall-clock bound; false means it timed out.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity,
                                          unsigned long long limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_ns() - t0 > limit_ns) return false;
    return true;
}

// The expiry path of the bounded wait above, on demand: one warp waits on a
// shared-memory mbarrier that nothing ever arrives on, with the given limit,
// and records IQK_DEVERR_TIMEOUT when the wait gives up. No copy is in
// flight and nothing else waits, so the kernel simply returns.
__global__ void __launch_bounds__(32) bounded_wait_check_kernel(unsigned long long limit_ns,
                                                              int32_t *flags) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    __syncwarp();
    const bool ok = mbar_wait(&bar, 0, limit_ns);
    if (!ok && threadIdx.x == 0) atomicOr(flags, IQK_DEVERR_TIMEOUT);
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// 2^k as a double, for |k| < 1000 (exact scaling, same result as ldexp).
__device__ __forceinline__ double pow2(int k) {
    return __longlong_as_double((long long)(k + 1023) << 52);
}

// FLOOR: the address floor of this kernel (the reference's deleted-decode
// floor, bench/floors.py:1-17): the same launch, producer and copies, so
// the same bytes cross from HBM into shared memory, and the compute warps read
// the same code words and activation planes, but fold them into an integer
// accumulator instead of decoding; the folded value reaches y, so no copy
// or read can be dropped. Only the benchmark's floor entry point uses it.
template <int MEMBER, int N, bool NARROW, bool FLOOR = false, bool GLU = false>
__global__ void __launch_bounds__(kThreads, Geo<MEMBER>::kMinBlocks)
gemv_kernel(GemvArgs a, const __grid_constant__ CUtensorMap qs_map,
            const __grid_constant__ CUtensorMap qs_map2) {
    extern __shared__ char smem_raw[];
    using G = Geo<MEMBER>;
    using SH = Shape<MEMBER, NARROW, GLU>;
    static_assert(!(GLU && (NARROW || FLOOR)), "the GLU shape is wide and decodes");
    constexpr int kRows = SH::kRows, KQ = SH::KQ, kStages = SH::kStages;
    using SS = Streams<MEMBER, N, kRows>;
    constexpr int CPW = N / kChunkK;  // 512-weight chunks per row: 8 (n=4096) or 4 (2048)
    constexpr int RPI = CPW / KQ;     // rounds per item
    static_assert(RPI % 2 == 0, "metadata buffers alternate by round parity");
    constexpr int SSB = sslot_bytes<MEMBER, N, kRows>();
    constexpr int STB = stage_bytes<MEMBER, KQ>();
    char *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const int out = a.out_features;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;

    char *stages = smem;
    char *sslots = stages + kStages * STB;  // two item scale slots
    char *metas = sslots + 2 * SH::kProj * SSB;  // slot o: projection q at (o * kProj + q) * SSB
    TileRef *tcache = reinterpret_cast<TileRef *>(metas + 2 * kConsumers * G::kMetaBytes);
    char *tail = reinterpret_cast<char *>(tcache + G::kTileCache);
    uint16_t *grid = reinterpret_cast<uint16_t *>(tail);   // IQ1_S_R4
    uint64_t *full = reinterpret_cast<uint64_t *>(tail + (MEMBER == IQK_IQ1_S_R4 ? 4096 : 0));
    uint64_t *empty = full + kStages;
    uint64_t *sfull = empty + kStages;  // [2] item scale slots
    uint64_t *sempty = sfull + 2;       // [2]
    uint64_t *rfull = sempty + 2;       // [2] narrow: warps 1-3 handed in their partials
    uint64_t *rempty = rfull + 2;       // [2] narrow: warp 0 read them
    int *abort_flag = reinterpret_cast<int *>(rempty + 2);
    char *zeros = reinterpret_cast<char *>(abort_flag) + 16;  // kPairsPerRound * 192 zero bytes
    char *red = zeros + kPairsPerRound * 192;  // narrow: [2][kConsumers][32 lanes][16 B]

    const int32_t *hdr = reinterpret_cast<const int32_t *>(a.ws + a.L.hdr);
    const int32_t *order = reinterpret_cast<const int32_t *>(a.ws + a.L.order);
    const int32_t *xscale = reinterpret_cast<const int32_t *>(a.ws + a.L.xscale);
    const TileRef *tlist = reinterpret_cast<const TileRef *>(a.ws + a.L.tiles1);
    const char *xbuf = a.ws + a.L.xbuf;
    const int64_t xrow = a.L.xrow_bytes;

    // Shared-memory set-up first: it overlaps the previous kernel's drain.
    if (MEMBER == IQK_IQ1_S_R4)
        for (int i = tid; i < 2048; i += blockDim.x) grid[i] = g_iq1s_grid[i];
    for (int i = tid; i < kPairsPerRound * 192 / 4; i += blockDim.x)
        reinterpret_cast<uint32_t *>(zeros)[i] = 0u;
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumers);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&sfull[s], 1);
            mbar_init(&sempty[s], kConsumers);
            mbar_init(&rfull[s], GLU ? 2 : kConsumers - 1);
            mbar_init(&rempty[s], GLU ? 2 : 1);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
    // From here on the workspace and the outputs: the previous kernel is done.
    grid_dep_wait();
    grid_dep_launch();

    const int ntiles = hdr[3];
    const int rblocks = (out + kRows - 1) / kRows;
    const int items = ntiles * rblocks;  // < 2^31 (checked by the C ABI)

    if (blockIdx.x == 0) {
        // zero the outputs of unroutable pairs (the tail of order)
        const int elem = a.y_dtype == IQK_F32 ? 4 : 2;
        const int row_words = out * elem / 4;
        for (int q = ntiles; q < a.pairs; ++q) {
            int32_t *yr = reinterpret_cast<int32_t *>(static_cast<char *>(a.y) +
                                                      (int64_t)order[q] * out * elem);
            for (int i = tid; i < row_words; i += blockDim.x) yr[i] = 0;
        }
    }
    // Work division: whole items. With more than two items per CTA they are
    // claimed dynamically: CTA b takes item b, then its producer claims the next one
    // from a counter in the workspace header and hands it to the compute warps
    // beside the item's scale slot. The schedulers favour low warp slots
    // (measured: warps in slots 0-3 run a round in 0.89 us, slots 12-15 in
    // 1.17 us), so a static division leaves the CTAs on high slots finishing
    // alone (30 % after the rest); claimed items keep every CTA busy until the
    // work runs out. The last CTA to finish resets the counter for the next
    // run on the workspace (runs on one workspace are stream-ordered). Each
    // item's rows are computed by one CTA with exact integer sums, so the
    // output does not depend on which CTA ran it.
    // (claiming pays for itself only with several items per CTA: with one or
    // two, every CTA's closing claim and count would only lengthen the launch)
    const bool dyn = a.dynamic && items > 2 * (int)gridDim.x;
    int32_t *work_ctr = reinterpret_cast<int32_t *>(const_cast<char *>(a.ws) + a.L.hdr) + 8;
    int32_t *done_ctr = work_ctr + 1;
    int *sitem = abort_flag + 1;  // [2] the item of scale slot 0 / 1 (-1: no more)
    const int i0 = dyn ? 0 : (int)((int64_t)items * blockIdx.x / gridDim.x);
    const int i1 = dyn ? items : (int)((int64_t)items * (blockIdx.x + 1) / gridDim.x);
    if (i0 >= i1) return;  // uniform over the CTA (a dynamic launch has items > 0)
    const int t0 = i0 / rblocks, t1 = (i1 - 1) / rblocks;
    const bool cached = !dyn && t1 - t0 < G::kTileCache;
    auto load_tile = [&](int t) -> TileRef {
        TileRef r = tlist[t];
        r.sh0 = xscale[r.tok0];
        return r;
    };
    if (cached)
        for (int t = tid; t <= t1 - t0; t += blockDim.x) tcache[t] = load_tile(t0 + t);
    __syncthreads();
    auto tile_of = [&](int t) -> TileRef { return cached ? tcache[t - t0] : load_tile(t); };
    const int n_items = i1 - i0;

    if (wid == kConsumers) {
        // ================= producer warp: TMA / bulk copies into the ring
        int ti = i0 / rblocks, rb = i0 % rblocks;
        int issued = 0, sissued = 0;
        bool ok = true;
        // this lane's scale stream (lanes 1 .. kCount-1; GLU: lanes 17 .. for
        // up's): bytes per row, slot offset
        const int sproj = GLU && lane >= 16 ? 1 : 0;
        const int sl = lane - 16 * sproj;
        const int si = sl >= 1 && sl < SS::kCount ? sl : 0;
        const int s_rowb = si ? SS::b(si) : 0, s_off = si ? sproj * SSB + SS::off(si) : 0;
        const void *const *sstreams = sproj ? a.s2 : a.s;
        for (int o = 0; ok; ++o) {
            int item;
            if (dyn) {
                if (o == 0) {
                    item = (int)blockIdx.x;
                } else {
                    if (lane == 0) item = (int)gridDim.x + atomicAdd(work_ctr, 1);
                    item = __shfl_sync(0xffffffffu, item, 0);
                }
            } else {
                if (o >= n_items) break;
                item = i0 + o;
            }
            // the item's scale streams (all rows, all of k) into scale slot o % 2
            const int ss = o & 1;
            if (o >= 2 && !mbar_wait(&sempty[ss], ((o >> 1) & 1) ^ 1)) {
                ok = false;
                break;
            }
            if (dyn && item >= items) {
                // no more work: the compute warps learn it from the slot
                if (lane == 0) {
                    sitem[ss] = -1;
                    mbar_arrive(&sfull[ss]);
                }
                sissued = o + 1;
                break;
            }
            if (dyn && lane == 0) sitem[ss] = item;
            ti = item / rblocks;
            rb = item - ti * rblocks;
            const TileRef T = tile_of(ti);
            const int r0 = rb * kRows;
            const int rows_valid = min(kRows, out - r0);
            if (lane == 0)
                mbar_arrive_expect_tx(&sfull[ss],
                                      (uint32_t)(SH::kProj * rows_valid * (SS::kSlot / kRows)));
            __syncwarp();
            if (si)
                bulk_load(sslots + ss * SH::kProj * SSB + s_off,
                          static_cast<const char *>(sstreams[si]) + ((int64_t)T.e * out + r0) * s_rowb,
                          (uint32_t)(rows_valid * s_rowb), &sfull[ss]);
            sissued = o + 1;
            // wide: warp w's box is rows 16w.., chunk r; narrow: all warps the
            // item's 16 rows, warp w chunk KQ*r + w
            const int wrow = T.e * out + r0 + (NARROW ? 0 : 16 * (GLU ? (lane & 1) : lane));
            const char *xb = xbuf + T.tok0 * xrow;
            for (int r = 0; r < RPI; ++r) {
                const int j = o * RPI + r;
                const int slot = j % kStages;
                if (j >= kStages && !mbar_wait(&empty[slot], ((j / kStages) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
                char *st = stages + slot * STB;
                if (lane == 0) mbar_arrive_expect_tx(&full[slot], (uint32_t)(G::kWBytes + KQ * G::kXBlock));
                __syncwarp();
                if (lane < kConsumers) {
                    // weights: one 16-row x kRowChunk-byte box per compute warp
                    tma_load_2d(st + lane * G::kWBox, GLU && lane >= 2 ? &qs_map2 : &qs_map,
                                (KQ * r + (NARROW ? lane : 0)) * G::kRowChunk, wrow, &full[slot]);
                } else if (lane == kConsumers) {
                    // activation digit planes (+ IQ1 block sums) of this round's
                    // KQ chunks: contiguous in the prepared row
                    char *xs = st + G::kWBytes;
                    bulk_load(xs, xb + (int64_t)r * KQ * G::kXPlanes, KQ * G::kXPlanes, &full[slot]);
                    if (G::kXSums)
                        bulk_load(xs + KQ * G::kXPlanes,
                                  xb + 3 * (int64_t)N + (int64_t)r * KQ * G::kXSums,
                                  KQ * G::kXSums, &full[slot]);
                }
                issued = j + 1;
            }
        }
        if (!ok && lane == 0) {
            atomicOr(a.err, IQK_DEVERR_TIMEOUT);
            atomicExch(abort_flag, 1);
        }
        // Drain: never leave the CTA with bulk copies still in flight. In
        // normal operation the consumers already waited on every stage; after
        // an abort this waits (bounded) for the copies issued last.
        for (int j = issued - 1; j >= 0 && j >= issued - kStages; --j)
            mbar_wait(&full[j % kStages], (j / kStages) & 1);
        for (int q = sissued - 1; q >= 0 && q >= sissued - 2; --q)
            mbar_wait(&sfull[q & 1], (q >> 1) & 1);
        if (dyn && lane == 0) {
            // the last CTA done resets the counters (every CTA has claimed its
            // last item before it counts itself done)
            __threadfence();
            if (atomicAdd(done_ctr, 1) == (int)gridDim.x - 1) {
                atomicExch(work_ctr, 0);
                atomicExch(done_ctr, 0);
            }
        }
        return;
    }

    // ===================== compute warps
    const int g = lane >> 2, tig = lane & 3;
    // first item-local row of this warp (GLU: within its projection)
    const int rbase = NARROW ? 0 : 16 * (GLU ? (wid & 1) : wid);
    const int proj = GLU ? (wid >> 1) : 0;  // GLU: 0 gate, 1 up
    const uint32_t meta_u = smem_u32(metas + wid * 2 * G::kMetaBytes);  // two round buffers
    const int side = tig >> 1;  // IQ2_KS, IQ1_S_R4: which 32-weight group of an MMA pair
    // Activation plane of B column g (or -1: a zero block). IQ2_KS and IQ1_S_R4
    // have two sides (columns 4s .. 4s+2: planes 0-2 of side s, lanes tig >> 1
    // == s supplying its k). IQ2_K has four, one per 16-weight sub-block = code
    // word tig: product a, columns 2s and 2s+1 = planes 0 and 1 of side s;
    // product b, column 2s = plane 2. Every column of a lane then belongs to
    // its own sub-block and takes that sub-block's integer scale.
    int bplane, bplane2 = -1;
    if (MEMBER == IQK_IQ2_K) {
        bplane = (g >> 1) == tig ? (g & 1) : -1;
        bplane2 = g == 2 * tig ? 2 : -1;
    } else {
        bplane = ((g & 3) < 3 && (g >> 2) == side) ? (g & 3) : -1;
    }
    // swizzled offsets of this lane's code words (rows g and g+8 of its box)
    uint32_t woff;
    if (MEMBER == IQK_IQ1_S_R4) woff = g * 64 + ((((uint32_t)g >> 1) & 3u) << 4) + side * 4;
    else woff = g * 128 + ((uint32_t)(g & 7) << 4) + tig * 4;
    // this lane's metadata entry within a pair: [pair][row pair g][side or word]
    const uint32_t moff = MEMBER == IQK_IQ2_K ? (g * 4 + tig) * 16 : (g * 2 + side) * 16;
    const uint32_t zero_u = smem_u32(zeros);
    const uint32_t m30 = a.one << 30;  // mulhi(x, m30) == x >> 2
    // metadata lanes: (mg, mq) owns row pair (mg, mg + 8) and 128 weights a round
    const int mg = lane & 7, mq = lane >> 3;
    const int mra = rbase + mg;  // item-local row (and mra + 8)
    // IQ2_KS group bits of (mg, mq) sit at bit msh of the sch / sex bytes
    const uint32_t msh = (uint32_t)(mq & 1) * 4u;
    const uint32_t hmask = 0xFu << msh;
    const uint32_t hmul = 0x02040810u >> msh;                 // bit msh+u -> bit 8u+4
    const uint32_t amul = msh ? 0x01020408u : 0x10204080u;    // bit msh+u -> bit 8u+7
    const uint32_t a44 = a.one * 0x88000000u;                 // mulhi: t>>1 | t>>5
    // IQ1_S_R4 grid-index permute: bytes (qs 2h, high 2h, qs 2h+1, high 2h+1), h = tig & 1
    const uint32_t isel = 0x5140u + 0x2222u * (uint32_t)(tig & 1);

    // Group metadata of round r (this warp's 16 rows x 512 weights) into the
    // metadata buffer at mb.
    // this warp's 512-weight chunk of round r
    auto chunk_of = [&](int r) { return KQ * r + (NARROW ? wid : 0); };
    auto build_meta = [&](const char *sd, int c, uint32_t mb) {
        if (MEMBER == IQK_IQ2_KS) {
            // Four groups of rows mra and mra + 8 at once, one byte per
            // group: scale index (low nibble | high bit << 4) and the
            // alphabet mask (0x44 when the group uses the second one).
            const int s0 = c * 16 + mq * 4;  // first of 4 groups (2 pairs)
            const uint8_t *scl = reinterpret_cast<const uint8_t *>(sd);
            const uint8_t *sch = scl + SS::off(2) + (s0 >> 3);
            const uint8_t *sex = scl + SS::off(3) + (s0 >> 3);
            scl += s0 >> 1;
            const uint32_t la = lds_u16(scl + mra * (N / 64));
            const uint32_t lb = lds_u16(scl + (mra + 8) * (N / 64));
            const uint32_t ha = sch[mra * (N / 256)], hb = sch[(mra + 8) * (N / 256)];
            const uint32_t xa = sex[mra * (N / 256)], xb = sex[(mra + 8) * (N / 256)];
            const uint32_t pa = prmt(la, 0u, 0x4140u), pb = prmt(lb, 0u, 0x4140u);
            const uint32_t va = ((pa | (pa << 4)) & 0x0F0F0F0Fu) | (((ha & hmask) * hmul) & 0x10101010u);
            const uint32_t vb = ((pb | (pb << 4)) & 0x0F0F0F0Fu) | (((hb & hmask) * hmul) & 0x10101010u);
            const uint32_t aa = mulhi(((xa & hmask) * amul) & 0x80808080u, a44);
            const uint32_t ab = mulhi(((xb & hmask) * amul) & 0x80808080u, a44);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int ia = (int)prmt(va, 0u, 0x4440u + u) - 16;
                const int ib = (int)prmt(vb, 0u, 0x4440u + u) - 16;
                const uint32_t ama = prmt(aa, 0u, 0x1111u * u);
                const uint32_t amb = prmt(ab, 0u, 0x1111u * u);
                const int pr = mq * 2 + (u >> 1), sd2 = u & 1;  // pair, side
                st_s128(mb + pr * 256 + (mg * 2 + sd2) * 16, ama, amb, (uint32_t)ia,
                        (uint32_t)ib);
            }
        } else if (MEMBER == IQK_IQ2_K) {
            // Eight 16-weight sub-blocks of rows mra and mra + 8, by byte
            // permutes: the alphabet mask (0x44 per byte for the second
            // alphabet; extra bit u spread to bit 7 of byte u & 3 by one
            // multiply, then 0x80 -> 0x44 by mul.hi) and the scale
            // 16 * (nibble - 8): nibble ^ 8 is nibble - 8 as a signed 4-bit
            // value, moved to the top of a byte and sign-extended by the permute.
            const int b0 = c * 32 + mq * 8;  // first of 8 sub-blocks (2 pairs)
            const uint8_t *scl = reinterpret_cast<const uint8_t *>(sd);
            const uint8_t *sex = scl + SS::off(2) + (b0 >> 3);
            scl += b0 >> 1;
            const uint32_t la = lds_u32(scl + mra * (N / 32)) ^ 0x88888888u;
            const uint32_t lb = lds_u32(scl + (mra + 8) * (N / 32)) ^ 0x88888888u;
            const uint32_t xa = sex[mra * (N / 128)], xb = sex[(mra + 8) * (N / 128)];
            const uint32_t ea[2] = {(la << 4) & 0xF0F0F0F0u, la & 0xF0F0F0F0u};  // even, odd u
            const uint32_t eb[2] = {(lb << 4) & 0xF0F0F0F0u, lb & 0xF0F0F0F0u};
            const uint32_t ma[2] = {mulhi(((xa & 0x0Fu) * 0x10204080u) & 0x80808080u, a44),
                                    mulhi(((xa & 0xF0u) * 0x01020408u) & 0x80808080u, a44)};
            const uint32_t mb2[2] = {mulhi(((xb & 0x0Fu) * 0x10204080u) & 0x80808080u, a44),
                                     mulhi(((xb & 0xF0u) * 0x01020408u) & 0x80808080u, a44)};
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const uint32_t bsel = 0x1111u * (u & 3);                  // replicate byte
                const uint32_t ssel = 0x8880u + 0x1111u * (u >> 1);       // sign-extend byte
                const int pr = mq * 2 + (u >> 2), wd = u & 3;  // pair, word
                st_s128(mb + pr * 512 + (mg * 4 + wd) * 16, prmt(ma[u >> 2], 0u, bsel),
                        prmt(mb2[u >> 2], 0u, bsel), prmt(ea[u & 1], 0u, ssel),
                        prmt(eb[u & 1], 0u, ssel));
            }
        } else {
            // Per block and row: the four octets' 3-bit grid-index high parts
            // spread to one byte each (fields 0, 2 and 1, 3 moved apart by
            // one multiply each, no overlapping bits), and the signed shift
            // term (sign of the block's delta) x its scale 2s+1.
            const int s0 = c * 16 + mq * 4;  // first of 4 blocks (2 pairs)
            const uint16_t *qh = reinterpret_cast<const uint16_t *>(sd) + s0;
            auto spread3 = [](uint32_t h) {
                return (((h & 0x1C7u) * 0x401u) & 0x00070007u) | (((h & 0xE38u) * 0x8020u) & 0x07000700u);
            };
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t ha = qh[mra * (N / 32) + u], hb = qh[(mra + 8) * (N / 32) + u];
                const int sa = 2 * (int)((ha >> 12) & 7u) + 1, sb = 2 * (int)((hb >> 12) & 7u) + 1;
                const int pr = mq * 2 + (u >> 1), sd2 = u & 1;
                st_s128(mb + pr * 256 + (mg * 2 + sd2) * 16, spread3(ha), spread3(hb),
                        (uint32_t)((ha & 0x8000u) ? -sa : sa), (uint32_t)((hb & 0x8000u) ? -sb : sb));
            }
        }
    };

    int ti = i0 / rblocks, rb = i0 % rblocks;
    bool prebuilt = false;  // this item's first-round metadata was built during the last item
    for (int o = 0; dyn || o < n_items; ++o) {
        // the item's scale streams (and, claimed dynamically, the item itself)
        if (!mbar_wait(&sfull[o & 1], (o >> 1) & 1)) {
            if (lane == 0) {
                atomicOr(a.err, IQK_DEVERR_TIMEOUT);
                atomicExch(abort_flag, 1);
            }
            break;
        }
        if (*(volatile int *)abort_flag) break;
        const int item = dyn ? *(volatile int *)&sitem[o & 1] : i0 + o;
        if (item < 0) break;  // no more work
        ti = item / rblocks;
        rb = item - ti * rblocks;
        const TileRef T = tile_of(ti);
        const int r0 = rb * kRows;
        const bool live = NARROW || rbase < out - r0;  // this warp's row tile exists
        // the next item's row tile, for building its first-round metadata early
        // (wide items only: in a two-round narrow item the extra wait measured
        // slower); claimed dynamically, it is known once its slot is full
        const bool nlive = !NARROW && (dyn || (o + 1 < n_items &&
                           rbase < out - (rb + 1 == rblocks ? 0 : rb + 1) * kRows));
        const char *sd = sslots + ((o & 1) * SH::kProj + proj) * SSB;
        // metadata buffer of round r: r & 1
        if (!FLOOR && live && !prebuilt) build_meta(sd, chunk_of(0), meta_u);
        prebuilt = false;
        __syncwarp();
        uint32_t facc = 0u;  // FLOOR: every word this warp would decode, folded
        int32_t tot[4] = {0, 0, 0, 0};
        int32_t tb[2] = {0, 0};        // IQ2_K: plane 2 (product b), rows g, g+8
        double dacc[2] = {0.0, 0.0};  // IQ2_K: rows g, g+8, this lane's sub-blocks
        bool ok = true;
#pragma unroll 1
        for (int r = 0; r < RPI; ++r) {
            const int j = o * RPI + r;
            const int slot = j % kStages;
            if (!mbar_wait(&full[slot], (j / kStages) & 1)) {
                ok = false;
                break;
            }
            const char *st = stages + slot * STB;
            if (FLOOR && live) {
                // the round's code words and activation planes (the loads of
                // the MMA-pair loop) plus the scale-slot words its metadata
                // reads, folded with distinct odd multipliers
                const uint32_t wb_u = smem_u32(st + wid * G::kWBox);
                const uint32_t xs_u = smem_u32(st + G::kWBytes + (NARROW ? wid * G::kXPlanes : 0));
                const uint32_t wl = wb_u | woff;
#pragma unroll
                for (int pr = 0; pr < kPairsPerRound; ++pr) {
                    uint32_t w0, w1;
                    if (MEMBER == IQK_IQ1_S_R4) {
                        const uint32_t wo = (wl ^ (uint32_t)((pr >> 1) << 4)) + (uint32_t)((pr & 1) << 3);
                        w0 = ld_s32(wo);
                        w1 = ld_s32(wo + 512);
                        // the grid gathers are addressing, not decode: kept
                        w0 += 131u * grid[w0 & 0x7ffu] + 137u * grid[(w1 >> 8) & 0x7ffu];
                    } else {
                        const uint32_t wo = wl ^ (uint32_t)(pr << 4);
                        w0 = ld_s32(wo);
                        w1 = ld_s32(wo + 1024);
                    }
                    const uint4 bv = ld_s128(xs_u + tig * 48 + pr * 192);
                    facc += w0 + 3u * w1 + 5u * bv.x + 7u * bv.y + 11u * bv.z + 13u * bv.w;
                }
                const uint32_t* sw = reinterpret_cast<const uint32_t *>(sd);
                facc += 17u * sw[(lane + 32 * (chunk_of(r) & 7)) % (SS::kSlot / 4)];
            } else if (live) {
                // ---- 8 MMA pairs, all shared-memory addresses 32-bit and the
                // per-pair offsets compile-time immediates.
                const uint32_t wb_u = smem_u32(st + wid * G::kWBox);
                // this warp's chunk: activation planes, and (IQ1) block sums
                const uint32_t xs_u = smem_u32(st + G::kWBytes + (NARROW ? wid * G::kXPlanes : 0));
                const uint32_t xsum_u = smem_u32(st + G::kWBytes + KQ * G::kXPlanes +
                                                 (NARROW ? wid * G::kXSums : 0));
                // B: live lanes read their plane's 16 bytes; the others a zero block
                const uint32_t xl_u = bplane >= 0 ? xs_u + tig * 48 + bplane * 16 : zero_u;
                const uint32_t xl2_u = bplane2 >= 0 ? xs_u + tig * 48 + bplane2 * 16 : zero_u;
                const uint32_t mrow = meta_u + (r & 1) * G::kMetaBytes + moff;
                const uint32_t wl = wb_u | woff;  // box is 1024-aligned, woff < 1024
#pragma unroll
                for (int pr = 0; pr < kPairsPerRound; ++pr) {
                    const uint4 bv = ld_s128(xl_u + pr * 192);
                    uint32_t A[4];
                    if (MEMBER == IQK_IQ2_KS) {
                        const uint32_t wo = wl ^ (uint32_t)(pr << 4);
                        const uint32_t wg = ld_s32(wo);
                        const uint32_t wg8 = ld_s32(wo + 1024);
                        const uint4 m = ld_s128(mrow + pr * 256);
                        const uint32_t s0g = (wg & 0x33333333u) | m.x;
                        const uint32_t s1g = (shr2(wg, m30) & 0x33333333u) | m.x;
                        const uint32_t s0h = (wg8 & 0x33333333u) | m.y;
                        const uint32_t s1h = (shr2(wg8, m30) & 0x33333333u) | m.y;
                        int32_t d[4];
                        A[0] = prmt(kIq2Tab0, kIq2Tab1, s0g);
                        A[1] = prmt(kIq2Tab0, kIq2Tab1, s0h);
                        A[2] = prmt(kIq2Tab0, kIq2Tab1, s1g);
                        A[3] = prmt(kIq2Tab0, kIq2Tab1, s1h);
                        mma_s8(d, A, bv.x, bv.y);
                        A[0] = prmt(kIq2Tab0, kIq2Tab1, shr16(s0g));
                        A[1] = prmt(kIq2Tab0, kIq2Tab1, shr16(s0h));
                        A[2] = prmt(kIq2Tab0, kIq2Tab1, shr16(s1g));
                        A[3] = prmt(kIq2Tab0, kIq2Tab1, shr16(s1h));
                        mma_s8_acc(d, A, bv.z, bv.w);
                        tot[0] += (int)m.z * d[0];
                        tot[1] += (int)m.z * d[1];
                        tot[2] += (int)m.w * d[2];
                        tot[3] += (int)m.w * d[3];
                    } else if (MEMBER == IQK_IQ2_K) {
                        const uint32_t wo = wl ^ (uint32_t)(pr << 4);
                        const uint32_t wg = ld_s32(wo);
                        const uint32_t wg8 = ld_s32(wo + 1024);
                        const uint4 m = ld_s128(mrow + pr * 512);  // masks g, g+8; scales g, g+8
                        const uint4 bw = ld_s128(xl2_u + pr * 192);
                        const uint32_t s0g = (wg & 0x33333333u) | m.x;
                        const uint32_t s1g = (shr2(wg, m30) & 0x33333333u) | m.x;
                        const uint32_t s0h = (wg8 & 0x33333333u) | m.y;
                        const uint32_t s1h = (shr2(wg8, m30) & 0x33333333u) | m.y;
                        int32_t d[4], e[4];
                        A[0] = prmt(kIq2Tab0, kIq2Tab1, s0g);
                        A[1] = prmt(kIq2Tab0, kIq2Tab1, s0h);
                        A[2] = prmt(kIq2Tab0, kIq2Tab1, s1g);
                        A[3] = prmt(kIq2Tab0, kIq2Tab1, s1h);
                        mma_s8(d, A, bv.x, bv.y);
                        mma_s8(e, A, bw.x, bw.y);
                        A[0] = prmt(kIq2Tab0, kIq2Tab1, shr16(s0g));
                        A[1] = prmt(kIq2Tab0, kIq2Tab1, shr16(s0h));
                        A[2] = prmt(kIq2Tab0, kIq2Tab1, shr16(s1g));
                        A[3] = prmt(kIq2Tab0, kIq2Tab1, shr16(s1h));
                        mma_s8_acc(d, A, bv.z, bv.w);
                        mma_s8_acc(e, A, bw.z, bw.w);
                        tot[0] += (int)m.z * d[0];
                        tot[1] += (int)m.z * d[1];
                        tot[2] += (int)m.w * d[2];
                        tot[3] += (int)m.w * d[3];
                        tb[0] += (int)m.z * e[0];
                        tb[1] += (int)m.w * e[2];
                        if ((pr & 3) == 3) {
                            // end of a 256-weight super-block: fold in its fp16
                            // scale (exact products; |tot| < 2^26 per super-block)
                            const int sbi = (chunk_of(r) * kChunkK + pr * 64) >> 8;
                            const uint16_t *dvp = reinterpret_cast<const uint16_t *>(sd + SS::off(3));
                            const int ra = rbase + g;
                            const double Tg = (double)tot[0] * 65536.0 + (double)tot[1] * 256.0 + (double)tb[0];
                            const double Th = (double)tot[2] * 65536.0 + (double)tot[3] * 256.0 + (double)tb[1];
                            dacc[0] += (double)half_bits_to_float(dvp[ra * (N / 256) + sbi]) * Tg;
                            dacc[1] += (double)half_bits_to_float(dvp[(ra + 8) * (N / 256) + sbi]) * Th;
                            tot[0] = tot[1] = tot[2] = tot[3] = 0;
                            tb[0] = tb[1] = 0;
                        }
                    } else {
                        // IQ1_S_R4: this lane covers sub-groups 2h, 2h+1 of block 2*pr+side
                        const int hsel = tig & 1;
                        const uint32_t wo = (wl ^ (uint32_t)((pr >> 1) << 4)) + (uint32_t)((pr & 1) << 3);
                        const uint32_t qg = ld_s32(wo);
                        const uint32_t qg8 = ld_s32(wo + 512);
                        const uint4 m = ld_s128(mrow + pr * 256);  // high parts g, g+8; shift terms
                        // both grid indices of a row (octets 2h, 2h+1: qs byte | high part << 8)
                        // from one byte permute
                        const uint32_t wig = prmt(qg, m.x, isel), wih = prmt(qg8, m.y, isel);
                        const uint32_t ga = grid[wig & 0xffffu], gb = grid[wig >> 16];
                        const uint32_t ha = grid[wih & 0xffffu], hb = grid[wih >> 16];
                        const uint32_t vg = prmt(ga, gb, 0x5410u), vh = prmt(ha, hb, 0x5410u);
                        const uint32_t s0g = vg & 0x33333333u, s1g = shr2(vg, m30) & 0x33333333u;
                        const uint32_t s0h = vh & 0x33333333u, s1h = shr2(vh, m30) & 0x33333333u;
                        int32_t d[4];
                        A[0] = prmt(kTernTab, 0u, s0g);
                        A[1] = prmt(kTernTab, 0u, s0h);
                        A[2] = prmt(kTernTab, 0u, s1g);
                        A[3] = prmt(kTernTab, 0u, s1h);
                        mma_s8(d, A, bv.x, bv.y);
                        A[0] = prmt(kTernTab, 0u, shr16(s0g));
                        A[1] = prmt(kTernTab, 0u, shr16(s0h));
                        A[2] = prmt(kTernTab, 0u, shr16(s1g));
                        A[3] = prmt(kTernTab, 0u, shr16(s1h));
                        mma_s8_acc(d, A, bv.z, bv.w);
                        // block sums of this lane's two C columns (block 2*pr+side,
                        // planes 2*(tig&1) and +1; plane 3 reads the stored zero)
                        const uint2 xsum = ld_s64(xsum_u + (pr * 2 + side) * 16 + hsel * 8);
                        const int sy = (int)m.z, sz = (int)m.w;  // +-(2s+1)
                        const int ma = abs(sy), mb = abs(sz);
                        tot[0] += ma * 8 * d[0] + sy * (int)xsum.x;
                        tot[1] += ma * 8 * d[1] + sy * (int)xsum.y;
                        tot[2] += mb * 8 * d[2] + sz * (int)xsum.x;
                        tot[3] += mb * 8 * d[3] + sz * (int)xsum.y;
                    }
                }
                // Next round's metadata into the other buffer, after the pair
                // loop in program order so its loads and arithmetic can fill
                // the loop's latency gaps. After a wide item's last round: the
                // next item's first round, from its scale slot, into buffer 0
                // (RPI is even, so this round reads buffer 1).
                if (FLOOR) {
                } else if (r + 1 < RPI) {
                    build_meta(sd, chunk_of(r + 1), meta_u + ((r + 1) & 1) * G::kMetaBytes);
                } else if (nlive && (r & 1) && mbar_wait(&sfull[(o + 1) & 1], ((o + 1) >> 1) & 1)) {
                    const int nitem = dyn ? *(volatile int *)&sitem[(o + 1) & 1] : item + 1;
                    if (nitem >= 0 && rbase < out - (nitem % rblocks) * kRows) {
                        build_meta(sslots + (((o + 1) & 1) * SH::kProj + proj) * SSB, chunk_of(0),
                                   meta_u);
                        prebuilt = true;
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);  // this round's stage
        }
        if (!ok) {
            if (lane == 0) {
                atomicOr(a.err, IQK_DEVERR_TIMEOUT);
                atomicExch(abort_flag, 1);
            }
            break;
        }

        if (FLOOR) {
            // the folds travel like the partial sums: through the narrow
            // shape's exchange area to warp 0
            tot[0] = (int32_t)facc;
            dacc[0] = (double)facc;
        }
        if (NARROW) {
            // ---- combine the four k quarters in warp 0: warps 1-3 hand over
            // their partials (exact integers; IQ2_K doubles, added in warp
            // order), through a double-buffered exchange area per item parity.
            const int rbuf = o & 1;
            char *area = red + (rbuf * kConsumers * 32 + lane) * 16;  // + warp * 512
            bool rok = true;
            if (wid != 0) {
                if (o >= 2 && !mbar_wait(&rempty[rbuf], ((o >> 1) & 1) ^ 1)) rok = false;
                if (rok) {
                    char *mine = area + wid * 32 * 16;
                    if (MEMBER == IQK_IQ2_K)
                        *reinterpret_cast<double2 *>(mine) = make_double2(dacc[0], dacc[1]);
                    else
                        *reinterpret_cast<int4 *>(mine) = make_int4(tot[0], tot[1], tot[2], tot[3]);
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&rfull[rbuf]);
                }
            } else {
                if (!mbar_wait(&rfull[rbuf], (o >> 1) & 1)) rok = false;
                if (rok) {
#pragma unroll
                    for (int w = 1; w < kConsumers; ++w) {
                        const char *theirs = area + w * 32 * 16;
                        if (MEMBER == IQK_IQ2_K) {
                            const double2 v = *reinterpret_cast<const double2 *>(theirs);
                            dacc[0] += v.x;
                            dacc[1] += v.y;
                        } else {
                            const int4 v = *reinterpret_cast<const int4 *>(theirs);
                            tot[0] += v.x;
                            tot[1] += v.y;
                            tot[2] += v.z;
                            tot[3] += v.w;
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&rempty[rbuf]);
                }
            }
            if (!rok) {
                if (lane == 0) {
                    atomicOr(a.err, IQK_DEVERR_TIMEOUT);
                    atomicExch(abort_flag, 1);
                }
                break;
            }
        }

        if (live && (!NARROW || wid == 0)) {
            // ---- item end: this warp holds the whole k range of its 16 rows.
            const int ra = rbase + g;  // item-local row
            double yg, yg8;
            if (FLOOR) {
                uint32_t f = MEMBER == IQK_IQ2_K ? (uint32_t)(long long)dacc[0] : (uint32_t)tot[0];
#pragma unroll
                for (int o2 = 1; o2 < 32; o2 <<= 1) f += __shfl_xor_sync(0xffffffffu, f, o2);
                yg = (double)(f & 0xffu);
                yg8 = (double)((f >> 8) & 0xffu);
            } else if (MEMBER == IQK_IQ2_K) {
                // the quad's four sub-block sides, in a fixed order
                yg = dacc[0] + __shfl_xor_sync(0xffffffffu, dacc[0], 1);
                yg8 = dacc[1] + __shfl_xor_sync(0xffffffffu, dacc[1], 1);
                yg += __shfl_xor_sync(0xffffffffu, yg, 2);
                yg8 += __shfl_xor_sync(0xffffffffu, yg8, 2);
            } else {
                int32_t s4[4] = {tot[0], tot[1], tot[2], tot[3]};
                // lanes tig 0/2 hold planes (0,1) of the two sides, 1/3 plane 2
#pragma unroll
                for (int k = 0; k < 4; ++k) s4[k] += __shfl_down_sync(0xffffffffu, s4[k], 2);
                const int32_t n0 = __shfl_down_sync(0xffffffffu, s4[0], 1);
                const int32_t n2 = __shfl_down_sync(0xffffffffu, s4[2], 1);
                const double Tg = (double)s4[0] * 65536.0 + (double)s4[1] * 256.0 + (double)n0;
                const double Tg8 = (double)s4[2] * 65536.0 + (double)s4[3] * 256.0 + (double)n2;
                const uint16_t *dvp = reinterpret_cast<const uint16_t *>(sd + SS::off(SS::kCount - 1));
                yg = (double)half_bits_to_float(dvp[ra]) * Tg;
                yg8 = (double)half_bits_to_float(dvp[ra + 8]) * Tg8;
            }
            float vg = 0.f, vg8 = 0.f;
            const int64_t o0 = (int64_t)T.pair0 * out + r0 + ra;
            const bool ok8 = r0 + ra + 8 < out;
            if (tig == 0) {
                const int S = T.sh0;
                if (S == kScaleNonFinite) {
                    vg = vg8 = __int_as_float(0x7fc00000);
                } else {
                    const double sc = pow2(-S - (MEMBER == IQK_IQ1_S_R4 ? 3 : MEMBER == IQK_IQ2_K ? 4 : 0));
                    vg = (float)(yg * sc);
                    vg8 = (float)(yg8 * sc);
                }
            }
            if (GLU) {
                // up warps hand rows (g, g + 8) of their row pair to the gate
                // warp of the same rows through a double-buffered exchange
                // (by item parity); the gate warp stores
                // h = silu(gate) * up * router weight
                const int rbuf = o & 1;
                float2 *xa = reinterpret_cast<float2 *>(red) + (rbuf * 2 + (wid & 1)) * 8;
                bool gok = true;
                if (proj == 1) {
                    if (o >= 2 && !mbar_wait(&rempty[rbuf], ((o >> 1) & 1) ^ 1)) gok = false;
                    if (gok && tig == 0) xa[g] = make_float2(vg, vg8);
                    __syncwarp();
                    if (gok && lane == 0) mbar_arrive(&rfull[rbuf]);
                } else {
                    if (!mbar_wait(&rfull[rbuf], (o >> 1) & 1)) gok = false;
                    if (gok && tig == 0) {
                        const float2 u = xa[g];
                        const float w = a.rw ? a.rw[T.pair0] : 1.f;
                        float *y = static_cast<float *>(a.y);
                        y[o0] = vg / (1.0f + expf(-vg)) * u.x * w;
                        if (ok8) y[o0 + 8] = vg8 / (1.0f + expf(-vg8)) * u.y * w;
                    }
                    __syncwarp();
                    if (gok && lane == 0) mbar_arrive(&rempty[rbuf]);
                }
                if (!gok) {
                    if (lane == 0) {
                        atomicOr(a.err, IQK_DEVERR_TIMEOUT);
                        atomicExch(abort_flag, 1);
                    }
                    break;
                }
            } else if (tig == 0) {
                if (a.y_dtype == IQK_F32) {
                    float *y = static_cast<float *>(a.y);
                    y[o0] = vg;
                    if (ok8) y[o0 + 8] = vg8;
                } else if (a.y_dtype == IQK_F16) {
                    __half *y = static_cast<__half *>(a.y);
                    y[o0] = __float2half_rn(vg);
                    if (ok8) y[o0 + 8] = __float2half_rn(vg8);
                } else {
                    __nv_bfloat16 *y = static_cast<__nv_bfloat16 *>(a.y);
                    y[o0] = __float2bfloat16_rn(vg);
                    if (ok8) y[o0 + 8] = __float2bfloat16_rn(vg8);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&sempty[o & 1]);  // the item's scale slot
    }
}


// ------------------------------------------------------------------- host

cudaError_t launch_bounded_wait_check(int64_t limit_ns, int32_t *flags, cudaStream_t stream) {
    bounded_wait_check_kernel<<<1, 32, 0, stream>>>((unsigned long long)limit_ns, flags);
    return cudaGetLastError();
}

GemvLayout gemv_layout(int member, int64_t n, int64_t x_rows, int64_t pairs) {
    GemvLayout L{};
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t at = off;
        off += (bytes + 255) & ~size_t(255);
        return at;
    };
    (void)member;
    L.hdr = take(64);
    L.order = take(sizeof(int32_t) * (pairs + 1));
    L.ptok = take(sizeof(int32_t) * (pairs + 1));
    L.tiles1 = take(sizeof(TileRef) * (pairs + 1));
    L.xscale = take(sizeof(int32_t) * (x_rows + 1));
    L.xrow_bytes = 3 * n + n / 2;  // planes [n/64][4][3][16] + block sums [n/32][4] int32
    L.xbuf = take((size_t)(x_rows * L.xrow_bytes));
    L.total = off;
    return L;
}

using GemvFn = void (*)(GemvArgs, CUtensorMap, CUtensorMap);

// Kernel variants: the decode, its address floor, and the SwitchGLU pair.
enum GemvVariant { kVarDecode = 0, kVarFloor = 1, kVarGlu = 2 };

// The narrow shape exists at in_features 4096 only (decode and floor).
template <bool FLOOR, bool GLU> static GemvFn gemv_fn_t(int member, int n, bool narrow) {
#define IQK_FN(M, NN) (narrow && !GLU ? (GemvFn)gemv_kernel<M, NN, true, FLOOR, false> \
                                      : (GemvFn)gemv_kernel<M, NN, false, FLOOR, GLU>)
    if (n == 2048)
        return member == IQK_IQ2_KS ? (GemvFn)gemv_kernel<IQK_IQ2_KS, 2048, false, FLOOR, GLU>
               : member == IQK_IQ2_K ? (GemvFn)gemv_kernel<IQK_IQ2_K, 2048, false, FLOOR, GLU>
                                     : (GemvFn)gemv_kernel<IQK_IQ1_S_R4, 2048, false, FLOOR, GLU>;
    return member == IQK_IQ2_KS ? IQK_FN(IQK_IQ2_KS, 4096)
           : member == IQK_IQ2_K ? IQK_FN(IQK_IQ2_K, 4096) : IQK_FN(IQK_IQ1_S_R4, 4096);
#undef IQK_FN
}
static GemvFn gemv_fn(int member, int n, bool narrow, int variant) {
    return variant == kVarFloor ? gemv_fn_t<true, false>(member, n, narrow)
           : variant == kVarGlu ? gemv_fn_t<false, true>(member, n, false)
                                : gemv_fn_t<false, false>(member, n, narrow);
}

static int gemv_smem_for(int member, int n, bool narrow, bool glu) {
#define IQK_SM(M, NN) (glu ? gemv_smem_bytes<M, NN, false, true>()                 \
                           : narrow ? gemv_smem_bytes<M, NN, true>() : gemv_smem_bytes<M, NN, false>())
    if (n == 2048)
        return member == IQK_IQ2_KS ? IQK_SM(IQK_IQ2_KS, 2048)
               : member == IQK_IQ2_K ? IQK_SM(IQK_IQ2_K, 2048) : IQK_SM(IQK_IQ1_S_R4, 2048);
    return member == IQK_IQ2_KS ? IQK_SM(IQK_IQ2_KS, 4096)
           : member == IQK_IQ2_K ? IQK_SM(IQK_IQ2_K, 4096) : IQK_SM(IQK_IQ1_S_R4, 4096);
#undef IQK_SM
}
int gemv_smem_for(int member, int n, bool narrow) { return gemv_smem_for(member, n, narrow, false); }

// Launch configuration with programmatic stream serialization (the kernel
// waits with griddepcontrol.wait before its first global-memory access).
struct PdlLaunch {
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    PdlLaunch(unsigned grid, unsigned block, size_t smem, cudaStream_t stream) {
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(block);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
};

cudaError_t launch_gemv_prepare(const void *x, int x_dtype, int64_t x_rows, int n,
                                int64_t num_experts, const int32_t *sel, const int32_t *tok,
                                int64_t pairs, void *ws, cudaStream_t stream) {
    const GemvLayout L = gemv_layout(0, n, x_rows, pairs);
    char *w = static_cast<char *>(ws);
    const size_t hist_bytes = sizeof(int32_t) * (size_t)num_experts;
    cudaError_t err = cudaSuccess;
    if (hist_bytes > 48 * 1024) {
        err = cudaFuncSetAttribute(gemv_prep_kernel<float>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hist_bytes);
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(gemv_prep_kernel<__half>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hist_bytes);
        if (err == cudaSuccess)
            err = cudaFuncSetAttribute(gemv_prep_kernel<__nv_bfloat16>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)hist_bytes);
        if (err != cudaSuccess) return err;
    }
    const unsigned pblocks = (unsigned)x_rows + 1;
    PdlLaunch pl(pblocks, 256, hist_bytes, stream);
#define IQK_PREP(T)                                                                          \
    err = cudaLaunchKernelEx(&pl.cfg, gemv_prep_kernel<T>, static_cast<const T *>(x), n,      \
                             (int)x_rows, sel, tok, (int)pairs, (int)num_experts, L, w)
    if (x_dtype == IQK_F32) IQK_PREP(float);
    else if (x_dtype == IQK_F16) IQK_PREP(__half);
    else IQK_PREP(__nv_bfloat16);
#undef IQK_PREP
    if (err != cudaSuccess) return err;
    return cudaGetLastError();
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link).
static cudaError_t encode_qs_map(CUtensorMap *map, const void *qs, int64_t rows, int64_t row_bytes,
                                 int box_bytes, bool swizzle128) {
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
    const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)box_bytes, 16u};
    const cuuint32_t estr[2] = {1u, 1u};
    const CUresult res = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(qs), dims,
                                strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return res == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_gemv_run(int member, const void *const *streams, int64_t num_experts,
                            int64_t out_features, int n, int64_t x_rows, int64_t pairs, void *y,
                            int y_dtype, const void *ws, cudaStream_t stream, int num_sms,
                            bool floor, const void *const *up_streams, const float *router_weight) {
    const int variant = up_streams ? kVarGlu : floor ? kVarFloor : kVarDecode;
    const GemvLayout L = gemv_layout(member, n, x_rows, pairs);
    GemvArgs ga{};
    const RowBytes rb = row_bytes(member, n);
    for (int i = 0; i < rb.count; ++i) {
        ga.s[i] = streams[i];
        ga.s2[i] = up_streams ? up_streams[i] : streams[i];
    }
    ga.rw = router_weight;
    ga.out_features = (int)out_features;
    ga.pairs = (int)pairs;
    ga.one = 1u;
    ga.L = L;
    ga.ws = static_cast<const char *>(ws);
    ga.err = reinterpret_cast<int32_t *>(const_cast<char *>(ga.ws) + L.hdr);
    ga.y = y;
    ga.y_dtype = y_dtype;
    CUtensorMap map, map2;
    const bool iq1 = member == IQK_IQ1_S_R4;
    cudaError_t err = encode_qs_map(&map, streams[0], num_experts * out_features,
                                    iq1 ? n / 8 : n / 4, iq1 ? 64 : 128, !iq1);
    if (err != cudaSuccess) return err;
    map2 = map;
    if (up_streams) {
        err = encode_qs_map(&map2, up_streams[0], num_experts * out_features, iq1 ? n / 8 : n / 4,
                            iq1 ? 64 : 128, !iq1);
        if (err != cudaSuccess) return err;
    }
    // One persistent wave: as many CTAs as fit on every SM at once (shared
    // memory and registers decide; cached per member, width and shape). The
    // shared-memory opt-in is a per-device function attribute: set once.
    // The floor variant runs with the decode kernel's grid (its own occupancy
    // could differ), so the two launches issue the same copies from the same
    // number of CTAs; the GLU variant has its own.
    static std::atomic<int> resident[2][3][2][2];
    static std::atomic<unsigned> attr_done[3][64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = -1;
    const bool glu = variant == kVarGlu;
    auto setup = [&](bool narrow, int &per_sm) -> cudaError_t {
        const int smem = gemv_smem_for(member, n, narrow, glu);
        const unsigned bit = 1u << ((member * 2 + (n == 4096)) * 2 + (narrow ? 1 : 0));
        for (int v = 0; v < 3; ++v) {
            if (v != kVarDecode && v != variant) continue;
            if (dev < 0 || !(attr_done[v][dev].load() & bit)) {
                const cudaError_t e = cudaFuncSetAttribute(
                    gemv_fn(member, n, narrow, v), cudaFuncAttributeMaxDynamicSharedMemorySize,
                    gemv_smem_for(member, n, narrow, v == kVarGlu));
                if (e != cudaSuccess) return e;
                if (dev >= 0) attr_done[v][dev].fetch_or(bit);
            }
        }
        const GemvFn fn = gemv_fn(member, n, narrow, glu ? kVarGlu : kVarDecode);
        std::atomic<int> &r = resident[glu][member][n == 4096][narrow ? 1 : 0];
        if (r.load() == 0) {
            int nb = 0;
            const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, fn, kThreads, smem);
            if (e != cudaSuccess) return e;
            r.store(nb > 0 ? nb : 1);
        }
        per_sm = r.load();
        return cudaSuccess;
    };
    int per_sm = 0;
    err = setup(false, per_sm);
    if (err != cudaSuccess) return err;
    // Upper bound on items: every pair its own tile of every row block. Fewer
    // wide items than resident CTAs (e.g. one token) take the narrow shape.
    const int64_t wide_items = pairs * ((out_features + kItemRows - 1) / kItemRows);
    // (At in_features 2048 an item is only four rounds wide already, and a
    // narrow item's single round does not pay for its set-up: measured.)
    const bool narrow = !glu && n == 4096 && wide_items < (int64_t)num_sms * per_sm;
    if (narrow) {
        err = setup(true, per_sm);
        if (err != cudaSuccess) return err;
    }
    const int64_t rows = narrow ? 16 : glu ? kItemRows / 2 : kItemRows;
    const int64_t max_items = pairs * ((out_features + rows - 1) / rows);
    const int64_t cap = (int64_t)num_sms * per_sm;
    int64_t blocks = max_items < cap ? max_items : cap;
    if (blocks < 1) blocks = 1;
    ga.dynamic = 1;
    PdlLaunch pl((unsigned)blocks, kThreads, gemv_smem_for(member, n, narrow, glu), stream);
    err = cudaLaunchKernelEx(&pl.cfg, gemv_fn(member, n, narrow, variant), ga, map, map2);
    if (err != cudaSuccess) return err;
    return cudaGetLastError();
}

}  // namespace iqk
