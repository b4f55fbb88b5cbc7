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
// * Routing is on the device: pairs are bucketed by expert and each distinct
//   expert's rows are streamed once for all pairs that selected it (the
//   reference's "union" formulation, src/mlx_iqk/kernels.py:484-572, for
//   every member).
//
// Run kernel layout. A CTA item is (expert, 32-row block, pair tile of 2
// pairs -- 1 for IQ2_K, whose two 16-weight sub-blocks per k-step occupy two
// operand columns each). The 8 warps split it 2 row tiles x 4 k-quarters, so
// small decode batches still spread over every SM. Each "round" moves, for
// every warp, one 512-weight chunk of its 16 rows plus the matching slice of
// the activation planes into a 4-stage cp.async ring; the first round of an
// item also brings the item's scale streams. Per round each warp expands the
// group metadata (alphabet nibble mask, scale indices) into shared memory
// once, then runs 16 MMA k-steps. Partials of the 4 k-quarters are summed in
// a fixed order, so results stay deterministic.
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

// ------------------------------------------------------------- prep kernel

// One block per activation row: digit planes, block sums and the exponent.
// Row layout in the workspace: planes [n/32 k-steps][3][4 lanes][8 bytes]
// (bytes 0-3: the lane's even k, 4-7: odd k), then block sums [n/32][4] int32.
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
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float f = to_float<XT>(xr[q * 8 + j]);
                v[it][j] = f;
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
        int8_t *dst = xb + (int64_t)s * 96;
#pragma unroll
        for (int p = 0; p < 3; ++p)
            *reinterpret_cast<uint2 *>(dst + p * 32 + tig * 8) = make_uint2(planes[p][0], planes[p][1]);
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

// Route the pairs: bucket by expert (counting sort in shared memory), then
// lay out two tile lists -- pairs grouped two by two per expert (IQ2_KS,
// IQ1_S_R4) and one by one (IQ2_K). Pairs whose expert or row index is out of
// range go to the tail of `order` (the run kernel zeroes their outputs) and
// set the device error word.
__device__ void route_pairs(const int32_t *__restrict__ sel, const int32_t *__restrict__ tok,
                            int pairs, int x_rows, int num_experts, const GemvLayout &L,
                            char *ws) {
    extern __shared__ int32_t hist[];  // [num_experts]
    __shared__ int32_t warp_tot[33];
    __shared__ int32_t s_bad, s_tail;
    const int tid = threadIdx.x, nt = blockDim.x;
    int32_t *hdr = reinterpret_cast<int32_t *>(ws + L.hdr);
    int32_t *order = reinterpret_cast<int32_t *>(ws + L.order);
    int32_t *ptok = reinterpret_cast<int32_t *>(ws + L.ptok);
    TileRef *tiles2 = reinterpret_cast<TileRef *>(ws + L.tiles2);
    TileRef *tiles1 = reinterpret_cast<TileRef *>(ws + L.tiles1);
    for (int e = tid; e < num_experts; e += nt) hist[e] = 0;
    if (tid == 0) s_bad = 0;
    __syncthreads();
    const int dims = tok ? 1 : pairs / x_rows;
    int err = 0;
    for (int p = tid; p < pairs; p += nt) {
        const int e = sel[p];
        const int t = tok ? tok[p] : p / dims;
        ptok[p] = t;
        if (e < 0 || e >= num_experts) err |= IQK_DEVERR_EXPERT;
        else if (t < 0 || t >= x_rows) err |= IQK_DEVERR_TOKEN;
        else atomicAdd(&hist[e], 1);
    }
    if (err) atomicOr(&s_bad, err);
    __syncthreads();
    // Thread-contiguous bins; scans of (routable pairs, tiles of 2).
    const int per = (num_experts + nt - 1) / nt;
    const int b0 = min(tid * per, num_experts), b1 = min(b0 + per, num_experts);
    int c_cnt = 0, c_t2 = 0;
    for (int e = b0; e < b1; ++e) {
        const int c = hist[e];
        c_cnt += c;
        c_t2 += (c + 1) >> 1;
    }
    int n_valid, n_t2;
    const int base_cnt = block_exclusive_scan(c_cnt, warp_tot, &n_valid);
    const int base_t2 = block_exclusive_scan(c_t2, warp_tot, &n_t2);
    // scatter cursors: first position of each expert's pairs
    {
        int run = base_cnt;
        for (int e = b0; e < b1; ++e) {
            const int c = hist[e];
            hist[e] = run;
            run += c;
        }
    }
    if (tid == 0) {
        hdr[0] = s_bad;
        hdr[2] = n_t2;     // tiles of 2 pairs (IQ2_KS, IQ1_S_R4)
        hdr[3] = n_valid;  // tiles of 1 pair (IQ2_K) == routable pairs
        s_tail = n_valid;
    }
    __syncthreads();
    for (int p = tid; p < pairs; p += nt) {
        const int e = sel[p];
        const int t = ptok[p];
        const bool ok = e >= 0 && e < num_experts && t >= 0 && t < x_rows;
        const int pos = ok ? atomicAdd(&hist[e], 1) : atomicAdd(&s_tail, 1);
        order[pos] = p;
    }
    __syncthreads();
    // Tile lists, expert by expert (each thread owns its bin range again;
    // hist[e] now holds the end of expert e's segment).
    {
        int run = base_cnt, run2 = base_t2;
        for (int e = b0; e < b1; ++e) {
            const int end = hist[e];
            for (int q = run; q < end; ++q) {
                const int p = order[q];
                tiles1[q] = TileRef{e, p, -1, ptok[p], -1, 0, 0, 1};
            }
            for (int q = run; q < end; q += 2) {
                const int p0 = order[q];
                const int p1 = q + 1 < end ? order[q + 1] : -1;
                tiles2[run2++] = TileRef{e, p0, p1, ptok[p0], p1 >= 0 ? ptok[p1] : -1, 0, 0,
                                         p1 >= 0 ? 2 : 1};
            }
            run = end;
        }
    }
}

template <typename XT>
__global__ void __launch_bounds__(256)
gemv_prep_kernel(const XT *__restrict__ x, int n, int x_rows, const int32_t *__restrict__ sel,
                 const int32_t *__restrict__ tok, int pairs, int num_experts, GemvLayout L,
                 char *__restrict__ ws) {
    if ((int)blockIdx.x < x_rows) {
        prep_row<XT>(x, n, blockIdx.x, L, ws);
    } else {
        route_pairs(sel, tok, pairs, x_rows, num_experts, L, ws);
    }
}

// -------------------------------------------------------------- run kernel

constexpr int kWarps = 8;
constexpr int kKSplit = 4;                    // warps sharing one row tile along k
constexpr int kRowTiles = kWarps / kKSplit;   // 16-row tiles per CTA item
constexpr int kItemRows = 16 * kRowTiles;     // 32
constexpr int kStages = 4;
constexpr int kChunkK = 512;                  // weights per row per round and warp
constexpr int kSteps = kChunkK / 32;          // MMA k-steps per round
constexpr int kMaxTiles = 256;                // tile entries cached in shared memory

template <int MEMBER> struct Geo {
    static constexpr int kPpt = MEMBER == IQK_IQ2_K ? 1 : 2;                 // pairs per tile
    static constexpr int kRowChunk = MEMBER == IQK_IQ1_S_R4 ? 64 : 128;      // qs bytes
    static constexpr int kRowStride = MEMBER == IQK_IQ1_S_R4 ? 80 : 144;     // bank-staggered
    static constexpr int kWBytes = kWarps * 16 * kRowStride;
    static constexpr int kXPlanes = kSteps * 96;                             // 3 planes
    static constexpr int kXSums = MEMBER == IQK_IQ1_S_R4 ? kSteps * 16 : 0;  // block sums
    static constexpr int kXBlock = kXPlanes + kXSums;                        // per (ks, pair)
    static constexpr int kStageBytes = kWBytes + kKSplit * kPpt * kXBlock;
    static constexpr int kMetaEntry = MEMBER == IQK_IQ2_K ? 32 : 16;
    static constexpr int kMetaBytes = kSteps * 8 * kMetaEntry;               // per warp
};

// Scale streams of one CTA item (kItemRows rows, whole k), all but qs.
template <int MEMBER> __host__ __device__ constexpr int slot_bytes(int n) {
    return MEMBER == IQK_IQ2_KS ? kItemRows * (n / 64 + n / 256 + n / 256) + 2 * kItemRows
           : MEMBER == IQK_IQ2_K ? kItemRows * (n / 32 + n / 128 + n / 128)
                                 : kItemRows * (n / 16) + 2 * kItemRows;
}

template <int MEMBER> __host__ __device__ constexpr int gemv_smem_bytes(int n) {
    using G = Geo<MEMBER>;
    return kStages * G::kStageBytes + kStages * slot_bytes<MEMBER>(n) + kWarps * G::kMetaBytes +
           kWarps * 32 * 4 * 4 + kWarps * 32 * 2 * 8 + kMaxTiles * (int)sizeof(TileRef) +
           (MEMBER == IQK_IQ1_S_R4 ? 4096 : 0);
}

struct GemvArgs {
    const void *s[5];
    int64_t out_features;
    int n;
    int pairs;
    GemvLayout L;
    const char *ws;
    void *y;
    int y_dtype;
};

__device__ __forceinline__ uint32_t lds_u16(const void *p) {
    return *reinterpret_cast<const uint16_t *>(p);
}

template <int MEMBER>
__global__ void __launch_bounds__(kWarps * 32, 1)
gemv_kernel(GemvArgs a) {
    extern __shared__ __align__(128) char smem[];
    using G = Geo<MEMBER>;
    constexpr int ppt = G::kPpt;
    const int n = a.n;
    const int64_t out = a.out_features;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int g = lane >> 2, tig = lane & 3;
    const int rt = wid / kKSplit, ks = wid % kKSplit;
    const int cpw = n / (kChunkK * kKSplit);  // rounds per item: 2 (n=4096) or 1 (2048)
    const int SB = slot_bytes<MEMBER>(n);

    char *stages = smem;
    char *slots = stages + kStages * G::kStageBytes;
    char *metas = slots + kStages * SB;
    int32_t *red_i = reinterpret_cast<int32_t *>(metas + kWarps * G::kMetaBytes);
    double *red_d = reinterpret_cast<double *>(red_i + kWarps * 32 * 4);
    TileRef *tcache = reinterpret_cast<TileRef *>(red_d + kWarps * 32 * 2);
    uint16_t *grid = reinterpret_cast<uint16_t *>(tcache + kMaxTiles);
    char *meta = metas + wid * G::kMetaBytes;

    const int32_t *hdr = reinterpret_cast<const int32_t *>(a.ws + a.L.hdr);
    const int32_t *order = reinterpret_cast<const int32_t *>(a.ws + a.L.order);
    const int32_t *xscale = reinterpret_cast<const int32_t *>(a.ws + a.L.xscale);
    const TileRef *tlist = reinterpret_cast<const TileRef *>(a.ws + (ppt == 2 ? a.L.tiles2 : a.L.tiles1));
    const char *xbuf = a.ws + a.L.xbuf;
    const int64_t xrow = a.L.xrow_bytes;

    const int ntiles = ppt == 2 ? hdr[2] : hdr[3];
    const int rblocks = (int)((out + kItemRows - 1) / kItemRows);
    const int items = ntiles * rblocks;

    if (blockIdx.x == 0) {
        // zero the outputs of unroutable pairs (the tail of order)
        const int nvalid = hdr[3];
        const int elem = a.y_dtype == IQK_F32 ? 4 : 2;
        const int row_words = (int)(out * elem / 4);
        for (int q = nvalid; q < a.pairs; ++q) {
            int32_t *yr = reinterpret_cast<int32_t *>(static_cast<char *>(a.y) +
                                                      (int64_t)order[q] * out * elem);
            for (int i = tid; i < row_words; i += blockDim.x) yr[i] = 0;
        }
    }
    const int i0 = (int)((int64_t)items * blockIdx.x / gridDim.x);
    const int i1 = (int)((int64_t)items * (blockIdx.x + 1) / gridDim.x);
    if (i0 >= i1) return;  // uniform over the CTA
    const int t0 = i0 / rblocks, t1 = (i1 - 1) / rblocks;
    const bool cached = t1 - t0 < kMaxTiles;
    auto load_tile = [&](int t) -> TileRef {
        TileRef r = tlist[t];
        r.sh0 = xscale[r.tok0];
        r.sh1 = r.tok1 >= 0 ? xscale[r.tok1] : 0;
        return r;
    };
    if (cached)
        for (int t = tid; t <= t1 - t0; t += blockDim.x) tcache[t] = load_tile(t0 + t);
    if (MEMBER == IQK_IQ1_S_R4)
        for (int i = tid; i < 2048; i += blockDim.x) grid[i] = g_iq1s_grid[i];
    __syncthreads();
    auto tile_of = [&](int t) -> TileRef { return cached ? tcache[t - t0] : load_tile(t); };

    const char *qs = static_cast<const char *>(a.s[0]);
    const int64_t qrow = MEMBER == IQK_IQ1_S_R4 ? n / 8 : n / 4;  // qs bytes per row
    const RowBytes rbs = row_bytes(MEMBER, n);

    // Issue round j: every warp's chunk of weights, the activation slices,
    // and (first round of an item) the item's scale streams.
    auto issue = [&](int j) {
        const int o = j / cpw, r = j - o * cpw, i = i0 + o;
        const TileRef T = tile_of(i / rblocks);
        const int64_t r0 = (int64_t)(i % rblocks) * kItemRows;
        const int rows_valid = (int)min((int64_t)kItemRows, out - r0);
        char *st = stages + (j % kStages) * G::kStageBytes;
        constexpr int per_row = G::kRowChunk / 16;
        for (int q = tid; q < kWarps * 16 * per_row; q += blockDim.x) {
            const int w = q / (16 * per_row), rem = q - w * 16 * per_row;
            const int row = rem / per_row, part = rem - row * per_row;
            const int lr = 16 * (w / kKSplit) + row;
            if (lr >= rows_valid) continue;
            const int c = (w % kKSplit) * cpw + r;
            cp_async16(st + (w * 16 + row) * G::kRowStride + part * 16,
                       qs + ((int64_t)T.e * out + r0 + lr) * qrow + c * G::kRowChunk + part * 16);
        }
        char *xs = st + G::kWBytes;
        constexpr int xparts = G::kXBlock / 16;
        for (int q = tid; q < kKSplit * ppt * xparts; q += blockDim.x) {
            const int blk = q / xparts, part = q - blk * xparts;
            const int ksx = blk / ppt, t = blk - ksx * ppt;
            const int tk = t == 0 ? T.tok0 : T.tok1;
            if (tk < 0) continue;
            const int c = ksx * cpw + r;
            const char *src = part < G::kXPlanes / 16
                                  ? xbuf + tk * xrow + (int64_t)c * G::kXPlanes + part * 16
                                  : xbuf + tk * xrow + 3 * (int64_t)n + (int64_t)c * kSteps * 16 +
                                        (part - G::kXPlanes / 16) * 16;
            cp_async16(xs + blk * G::kXBlock + part * 16, src);
        }
        if (r == 0) {
            char *sd = slots + (o % kStages) * SB;
            int off = 0;
            for (int si = 1; si < rbs.count; ++si) {
                const int bytes = (int)(rows_valid * rbs.b[si]);
                const char *src = static_cast<const char *>(a.s[si]) + ((int64_t)T.e * out + r0) * rbs.b[si];
                for (int q = tid * 16; q < bytes; q += blockDim.x * 16) cp_async16(sd + off + q, src + q);
                off += (int)(kItemRows * rbs.b[si]);
            }
        }
    };

    const int total_rounds = (i1 - i0) * cpw;
#pragma unroll 1
    for (int j = 0; j < kStages - 1; ++j) {
        if (j < total_rounds) issue(j);
        cp_async_commit();
    }

    int32_t tot[4] = {0, 0, 0, 0};
    double dacc[2] = {0.0, 0.0};  // IQ2_K: rows g, g+8 (lanes with tig == 0)

#pragma unroll 1
    for (int j = 0; j < total_rounds; ++j) {
        const int o = j / cpw, r = j - o * cpw, i = i0 + o;
        const TileRef T = tile_of(i / rblocks);
        const int64_t r0 = (int64_t)(i % rblocks) * kItemRows;
        cp_async_wait<kStages - 2>();
        __syncthreads();
        if (j + kStages - 1 < total_rounds) issue(j + kStages - 1);
        cp_async_commit();
        if (r == 0) {
            tot[0] = tot[1] = tot[2] = tot[3] = 0;
            dacc[0] = dacc[1] = 0.0;
        }
        const bool live = 16 * rt < out - r0;  // this warp's row tile exists
        const char *st = stages + (j % kStages) * G::kStageBytes;
        const char *sd = slots + (o % kStages) * SB;
        const int c = ks * cpw + r;  // chunk of this warp
        if (live) {
            // ---- expand group metadata for this warp's 16 rows x 16 k-steps
            {
                const int mg = lane & 7, mq = lane >> 3;  // row pair, quad of k-steps
                const int ra = 16 * rt + mg, rb = ra + 8;  // item-local rows g, g+8
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int ls = mq * 4 + u;
                    const int s = c * kSteps + ls;  // global k-step
                    if (MEMBER == IQK_IQ2_KS) {
                        const uint8_t *scl = reinterpret_cast<const uint8_t *>(sd);
                        const uint8_t *sch = scl + kItemRows * (n / 64);
                        const uint8_t *sex = sch + kItemRows * (n / 256);
                        const int sh = (s & 1) * 4, bi = s >> 3, bb = s & 7;
                        const int ia = (((scl[ra * (n / 64) + (s >> 1)] >> sh) & 15) |
                                        (((sch[ra * (n / 256) + bi] >> bb) & 1) << 4)) - 16;
                        const int ib = (((scl[rb * (n / 64) + (s >> 1)] >> sh) & 15) |
                                        (((sch[rb * (n / 256) + bi] >> bb) & 1) << 4)) - 16;
                        const uint32_t am = (((sex[ra * (n / 256) + bi] >> bb) & 1) ? 0x4444u : 0u) |
                                            (((sex[rb * (n / 256) + bi] >> bb) & 1) ? 0x44440000u : 0u);
                        *reinterpret_cast<int4 *>(meta + (ls * 8 + mg) * 16) =
                            make_int4((int)am, ia, ib, 0);
                    } else if (MEMBER == IQK_IQ2_K) {
                        const uint8_t *scl = reinterpret_cast<const uint8_t *>(sd);
                        const uint8_t *sex = scl + kItemRows * (n / 32);
                        const int ba = scl[ra * (n / 32) + s], bbv = scl[rb * (n / 32) + s];
                        const int xa = sex[ra * (n / 128) + (s >> 2)] >> ((2 * s) & 7);
                        const int xb = sex[rb * (n / 128) + (s >> 2)] >> ((2 * s) & 7);
                        const uint32_t am0 = ((xa & 1) ? 0x4444u : 0u) | ((xb & 1) ? 0x44440000u : 0u);
                        const uint32_t am1 = ((xa & 2) ? 0x4444u : 0u) | ((xb & 2) ? 0x44440000u : 0u);
                        int4 *m = reinterpret_cast<int4 *>(meta + (ls * 8 + mg) * 32);
                        m[0] = make_int4((int)am0, (int)am1, 0, 0);
                        m[1] = make_int4((ba & 15) - 8, (ba >> 4) - 8, (bbv & 15) - 8, (bbv >> 4) - 8);
                    } else {
                        const uint16_t *qh = reinterpret_cast<const uint16_t *>(sd);
                        const uint32_t ha = qh[ra * (n / 32) + s], hb = qh[rb * (n / 32) + s];
                        const int ma = 2 * (int)((ha >> 12) & 7u) + 1, mb = 2 * (int)((hb >> 12) & 7u) + 1;
                        *reinterpret_cast<int4 *>(meta + (ls * 8 + mg) * 16) =
                            make_int4((int)(ha | (hb << 16)), ma, mb,
                                      ((ha & 0x8000u) ? 1 : 0) | ((hb & 0x8000u) ? 2 : 0));
                    }
                }
            }
            __syncwarp();

            // ---- 16 MMA k-steps
            const char *wb = st + wid * 16 * G::kRowStride;
            const char *xs = st + G::kWBytes + ks * ppt * G::kXBlock;
            int bt, bp;
            bool blive;
            if (MEMBER == IQK_IQ2_K) {
                bt = 0;
                bp = g >> 1;
                blive = bp < 3 && (g & 1) == (tig >> 1);
            } else {
                bt = g >> 2;
                bp = g & 3;
                blive = bp < 3 && (bt == 0 ? T.tok0 : T.tok1) >= 0;
            }
            const char *xl = xs + bt * G::kXBlock + bp * 32 + tig * 8;
#pragma unroll 4
            for (int ls = 0; ls < kSteps; ++ls) {
                uint32_t A[4];
                uint2 bv = make_uint2(0u, 0u);
                if (blive) bv = *reinterpret_cast<const uint2 *>(xl + ls * 96);
                int32_t d[4];
                if (MEMBER == IQK_IQ1_S_R4) {
                    const int4 m = *reinterpret_cast<const int4 *>(meta + (ls * 8 + g) * 16);
                    const uint32_t qg = *reinterpret_cast<const uint32_t *>(wb + g * G::kRowStride + ls * 4);
                    const uint32_t qg8 = *reinterpret_cast<const uint32_t *>(wb + (g + 8) * G::kRowStride + ls * 4);
                    const uint32_t h = (uint32_t)m.x;
                    const uint32_t ig = ((qg >> (8 * tig)) & 0xffu) | (((h >> (3 * tig)) & 7u) << 8);
                    const uint32_t ig8 = ((qg8 >> (8 * tig)) & 0xffu) | (((h >> (16 + 3 * tig)) & 7u) << 8);
                    const uint32_t v = (uint32_t)grid[ig] | ((uint32_t)grid[ig8] << 16);
                    const uint32_t s0 = v & 0x33333333u;
                    const uint32_t s1 = (v >> 2) & 0x33333333u;
                    A[0] = prmt(kTernTab, 0u, s0);
                    A[1] = prmt(kTernTab, 0u, s0 >> 16);
                    A[2] = prmt(kTernTab, 0u, s1);
                    A[3] = prmt(kTernTab, 0u, s1 >> 16);
                    mma_s8(d, A, bv.x, bv.y);
                    // block sums of this lane's C columns: token tig>>1,
                    // planes 2*(tig&1) and +1 (plane 3 is the stored zero)
                    const int ct = tig >> 1, cp = 2 * (tig & 1);
                    const int2 xb = *reinterpret_cast<const int2 *>(
                        xs + ct * G::kXBlock + G::kXPlanes + ls * 16 + cp * 4);
                    const int sa = (m.w & 1) ? -1 : 1, sb = (m.w & 2) ? -1 : 1;
                    tot[0] += m.y * (8 * d[0] + sa * xb.x);
                    tot[1] += m.y * (8 * d[1] + sa * xb.y);
                    tot[2] += m.z * (8 * d[2] + sb * xb.x);
                    tot[3] += m.z * (8 * d[3] + sb * xb.y);
                } else {
                    const uint32_t hg = lds_u16(wb + g * G::kRowStride + ls * 8 + tig * 2);
                    const uint32_t hg8 = lds_u16(wb + (g + 8) * G::kRowStride + ls * 8 + tig * 2);
                    const uint32_t v = hg | (hg8 << 16);
                    uint32_t am;
                    int4 ix;
                    if (MEMBER == IQK_IQ2_KS) {
                        const int4 m = *reinterpret_cast<const int4 *>(meta + (ls * 8 + g) * 16);
                        am = (uint32_t)m.x;
                        ix = make_int4(m.y, m.y, m.z, m.z);
                    } else {
                        const char *mp = meta + (ls * 8 + g) * 32;
                        am = *reinterpret_cast<const uint32_t *>(mp + 4 * (tig >> 1));
                        ix = *reinterpret_cast<const int4 *>(mp + 16);
                    }
                    const uint32_t s0 = (v & 0x33333333u) | am;
                    const uint32_t s1 = ((v >> 2) & 0x33333333u) | am;
                    A[0] = prmt(kIq2Tab0, kIq2Tab1, s0);
                    A[1] = prmt(kIq2Tab0, kIq2Tab1, s0 >> 16);
                    A[2] = prmt(kIq2Tab0, kIq2Tab1, s1);
                    A[3] = prmt(kIq2Tab0, kIq2Tab1, s1 >> 16);
                    mma_s8(d, A, bv.x, bv.y);
                    tot[0] += ix.x * d[0];
                    tot[1] += ix.y * d[1];
                    tot[2] += ix.z * d[2];
                    tot[3] += ix.w * d[3];
                    if (MEMBER == IQK_IQ2_K && (ls & 7) == 7) {
                        // end of a 256-weight super-block: fold in its fp16 scale
                        const int s = c * kSteps + ls;
                        const uint16_t *dvp = reinterpret_cast<const uint16_t *>(
                            sd + kItemRows * (n / 32) + kItemRows * (n / 128));
                        const int32_t pg = tot[0] + tot[1], pg8 = tot[2] + tot[3];
                        const int32_t p1g = __shfl_down_sync(0xffffffffu, pg, 1);
                        const int32_t p2g = __shfl_down_sync(0xffffffffu, pg, 2);
                        const int32_t p1g8 = __shfl_down_sync(0xffffffffu, pg8, 1);
                        const int32_t p2g8 = __shfl_down_sync(0xffffffffu, pg8, 2);
                        if (tig == 0) {
                            const int ra = 16 * rt + g;
                            const double Tg = (double)pg * 65536.0 + (double)p1g * 256.0 + (double)p2g;
                            const double Tg8 = (double)pg8 * 65536.0 + (double)p1g8 * 256.0 + (double)p2g8;
                            dacc[0] += (double)half_bits_to_float(dvp[ra * (n / 256) + (s >> 3)]) * Tg;
                            dacc[1] += (double)half_bits_to_float(dvp[(ra + 8) * (n / 256) + (s >> 3)]) * Tg8;
                        }
                        tot[0] = tot[1] = tot[2] = tot[3] = 0;
                    }
                }
            }
        }

        if (r == cpw - 1) {
            // ---- item end: k-quarter partials -> shared, fixed-order sum, epilogue
            *reinterpret_cast<int4 *>(red_i + (wid * 32 + lane) * 4) = make_int4(tot[0], tot[1], tot[2], tot[3]);
            if (MEMBER == IQK_IQ2_K) {
                red_d[(wid * 32 + lane) * 2] = dacc[0];
                red_d[(wid * 32 + lane) * 2 + 1] = dacc[1];
            }
            __syncthreads();
            if (ks == 0 && live) {
                const int ra = 16 * rt + g;  // item-local row
                double yg = 0.0, yg8 = 0.0;
                int t_out;
                bool writer;
                if (MEMBER == IQK_IQ2_K) {
                    for (int k = 0; k < kKSplit; ++k) {
                        yg += red_d[((rt * kKSplit + k) * 32 + lane) * 2];
                        yg8 += red_d[((rt * kKSplit + k) * 32 + lane) * 2 + 1];
                    }
                    t_out = 0;
                    writer = tig == 0;
                } else {
                    int32_t s4[4] = {0, 0, 0, 0};
                    for (int k = 0; k < kKSplit; ++k) {
                        const int4 pv = *reinterpret_cast<const int4 *>(red_i + ((rt * kKSplit + k) * 32 + lane) * 4);
                        s4[0] += pv.x;
                        s4[1] += pv.y;
                        s4[2] += pv.z;
                        s4[3] += pv.w;
                    }
                    // even-tig lanes hold planes (0,1) of token tig>>1, odd lanes (2, pad)
                    const int32_t n0 = __shfl_down_sync(0xffffffffu, s4[0], 1);
                    const int32_t n2 = __shfl_down_sync(0xffffffffu, s4[2], 1);
                    const double Tg = (double)s4[0] * 65536.0 + (double)s4[1] * 256.0 + (double)n0;
                    const double Tg8 = (double)s4[2] * 65536.0 + (double)s4[3] * 256.0 + (double)n2;
                    const uint16_t *dvp = reinterpret_cast<const uint16_t *>(
                        sd + (MEMBER == IQK_IQ2_KS ? kItemRows * (n / 64 + n / 256 + n / 256)
                                                   : kItemRows * (n / 16)));
                    yg = (double)half_bits_to_float(dvp[ra]) * Tg;
                    yg8 = (double)half_bits_to_float(dvp[ra + 8]) * Tg8;
                    t_out = tig >> 1;
                    writer = (tig & 1) == 0;
                }
                const int pair = t_out == 0 ? T.pair0 : T.pair1;
                if (writer && pair >= 0) {
                    const int S = t_out == 0 ? T.sh0 : T.sh1;
                    const int shift = -S - (MEMBER == IQK_IQ1_S_R4 ? 3 : 0);
                    float vg, vg8;
                    if (S == kScaleNonFinite) {
                        vg = vg8 = __int_as_float(0x7fc00000);
                    } else {
                        vg = (float)ldexp(yg, shift);
                        vg8 = (float)ldexp(yg8, shift);
                    }
                    const int64_t o0 = (int64_t)pair * out + r0 + ra;
                    if (a.y_dtype == IQK_F32) {
                        float *y = static_cast<float *>(a.y);
                        y[o0] = vg;
                        y[o0 + 8] = vg8;
                    } else if (a.y_dtype == IQK_F16) {
                        __half *y = static_cast<__half *>(a.y);
                        y[o0] = __float2half_rn(vg);
                        y[o0 + 8] = __float2half_rn(vg8);
                    } else {
                        __nv_bfloat16 *y = static_cast<__nv_bfloat16 *>(a.y);
                        y[o0] = __float2bfloat16_rn(vg);
                        y[o0 + 8] = __float2bfloat16_rn(vg8);
                    }
                }
            }
        }
    }
    cp_async_wait<0>();
}

// ------------------------------------------------------------------- host

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
    L.tiles2 = take(sizeof(TileRef) * (pairs + 1));
    L.tiles1 = take(sizeof(TileRef) * (pairs + 1));
    L.xscale = take(sizeof(int32_t) * (x_rows + 1));
    L.xrow_bytes = 3 * n + n / 2;  // planes [n/32][3][4][8] + block sums [n/32][4] int32
    L.xbuf = take((size_t)(x_rows * L.xrow_bytes));
    L.total = off;
    return L;
}

int gemv_smem_for(int member, int n) {
    if (member == IQK_IQ2_KS) return gemv_smem_bytes<IQK_IQ2_KS>(n);
    if (member == IQK_IQ2_K) return gemv_smem_bytes<IQK_IQ2_K>(n);
    return gemv_smem_bytes<IQK_IQ1_S_R4>(n);
}

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
#define IQK_PREP(T)                                                                          \
    gemv_prep_kernel<T><<<pblocks, 256, hist_bytes, stream>>>(                               \
        static_cast<const T *>(x), n, (int)x_rows, sel, tok, (int)pairs, (int)num_experts, L, w)
    if (x_dtype == IQK_F32) IQK_PREP(float);
    else if (x_dtype == IQK_F16) IQK_PREP(__half);
    else IQK_PREP(__nv_bfloat16);
#undef IQK_PREP
    return cudaGetLastError();
}

cudaError_t launch_gemv_run(int member, const void *const *streams, int64_t out_features, int n,
                            int64_t x_rows, int64_t pairs, void *y, int y_dtype, const void *ws,
                            cudaStream_t stream, int num_sms) {
    const GemvLayout L = gemv_layout(member, n, x_rows, pairs);
    GemvArgs ga{};
    const RowBytes rb = row_bytes(member, n);
    for (int i = 0; i < rb.count; ++i) ga.s[i] = streams[i];
    ga.out_features = out_features;
    ga.n = n;
    ga.pairs = (int)pairs;
    ga.L = L;
    ga.ws = static_cast<const char *>(ws);
    ga.y = y;
    ga.y_dtype = y_dtype;
    const int smem = gemv_smem_for(member, n);
    // Upper bound on CTA items: every pair its own tile of every row block.
    const int64_t max_items = pairs * ((out_features + kItemRows - 1) / kItemRows);
    int64_t blocks = max_items < num_sms ? max_items : num_sms;
    if (blocks < 1) blocks = 1;
    cudaError_t err = cudaSuccess;
#define IQK_GEMV(M)                                                                          \
    do {                                                                                     \
        err = cudaFuncSetAttribute(gemv_kernel<M>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                   smem);                                                    \
        if (err != cudaSuccess) return err;                                                  \
        gemv_kernel<M><<<(unsigned)blocks, kWarps * 32, smem, stream>>>(ga);                 \
    } while (0)
    if (member == IQK_IQ2_KS) IQK_GEMV(IQK_IQ2_KS);
    else if (member == IQK_IQ2_K) IQK_GEMV(IQK_IQ2_K);
    else IQK_GEMV(IQK_IQ1_S_R4);
#undef IQK_GEMV
    return cudaGetLastError();
}

}  // namespace iqk
