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
//   + l). The planes are stored in the operand order of the MMA below.
// * Weights are never materialised. Each 2-bit code (or ternary grid value)
//   is turned into its int8 alphabet value with a byte permute straight into
//   an mma.sync.m16n8k32 s8 A fragment; the digit planes are the B operand.
//   The tensor core returns exact int32 sums per 32-weight group, which are
//   scaled by the group's integer scale index with IMAD -- so the whole
//   reduction is exact integer arithmetic until one final double-precision
//   multiply by the fp16 row (or super-block) scale and 2^-S_t.
// * Consequently every output is independent of reduction order and of how
//   pairs are grouped: a sorted or unioned call is bit-identical to the
//   per-pair call, and the only approximation is x's 22-bit rounding.
// * Routing is on the device: pairs are bucketed by expert, and each distinct
//   expert's weight rows are streamed once for all pairs that selected it
//   (the reference's "union" formulation, src/mlx_iqk/kernels.py:484-572,
//   for every member).
//
// Work unit: one warp owns a 16-row tile of one expert for one "pair tile"
// (2 pairs for IQ2_KS / IQ1_S_R4, 1 pair for IQ2_K whose two 16-weight
// sub-blocks per k-step occupy two operand columns each). Weight streams go
// through a per-warp cp.async ring in shared memory; activation planes are
// read through L1.
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

__device__ __forceinline__ uint2 ldg_nc_u2(const void *p) {
    uint2 v;
    asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

// ------------------------------------------------------------- prep kernel

// One block per activation row: digit planes + block sums + exponent.
// The last block routes the pairs.
template <typename XT>
__device__ void prep_row(const XT *__restrict__ x, int n, int row, const GemvLayout &L,
                         char *ws) {
    __shared__ float red_max[32];
    __shared__ int red_bad[32];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int noct = n / 8;  // octets: (k-step s = q / 4, tig = q % 4)
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
        if (bad) atomicOr(reinterpret_cast<int32_t *>(ws + L.hdr), IQK_DEVERR_NONFINITE);
    }
    int8_t *xb = reinterpret_cast<int8_t *>(ws + L.xbuf) + (int64_t)row * L.xrow_bytes;
#pragma unroll
    for (int it = 0; it < 2; ++it) {
        const int q = tid + it * blockDim.x;
        if (q >= noct) continue;  // uniform per quad: noct is a multiple of 4
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
            // byte j/2 of word (j & 1): even k in word 0, odd k in word 1
#pragma unroll
            for (int p = 0; p < 3; ++p) {
                planes[p][j & 1] |= (uint32_t)(uint8_t)(int8_t)dig[p] << (8 * (j >> 1));
                bsum[p] += dig[p];
            }
        }
        int8_t *dst = xb + (int64_t)s * 128;
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
            *reinterpret_cast<int4 *>(dst + 96) = make_int4(bsum[0], bsum[1], bsum[2], 0);
        else if (tig == 2)
            *reinterpret_cast<int4 *>(dst + 112) = make_int4(0, 0, 0, 0);
    }
}

// Route the pairs: bucket by expert (counting sort in shared memory), list
// distinct experts, and lay out the warp work items.
__device__ void route_pairs(const int32_t *__restrict__ sel, const int32_t *__restrict__ tok,
                            int pairs, int x_rows, int num_experts, int out_features,
                            int ppt, const GemvLayout &L, char *ws, void *y, int y_elem) {
    extern __shared__ int32_t hist[];  // [num_experts]
    __shared__ int32_t s_part[1024];
    __shared__ int32_t s_total[2];
    const int tid = threadIdx.x, nt = blockDim.x;
    int32_t *hdr = reinterpret_cast<int32_t *>(ws + L.hdr);
    int32_t *uniq = reinterpret_cast<int32_t *>(ws + L.uniq);
    int32_t *seg = reinterpret_cast<int32_t *>(ws + L.seg);
    int32_t *ubase = reinterpret_cast<int32_t *>(ws + L.ubase);
    int32_t *order = reinterpret_cast<int32_t *>(ws + L.order);
    int32_t *ptok = reinterpret_cast<int32_t *>(ws + L.ptok);
    for (int e = tid; e < num_experts; e += nt) hist[e] = 0;
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
        if (e < 0 || e >= num_experts || t < 0 || t >= x_rows) {
            // zero the output row of an unroutable pair
            char *yr = static_cast<char *>(y) + (int64_t)p * out_features * y_elem;
            for (int i = 0; i < out_features * y_elem; i += 4)
                *reinterpret_cast<int32_t *>(yr + i) = 0;
        }
    }
    if (err) atomicOr(&hdr[0], err);
    __syncthreads();
    // Exclusive scans over experts of (count) and (distinct flag) and of the
    // item count ceil(count / ppt); thread-contiguous bins, then a block scan.
    const int per = (num_experts + nt - 1) / nt;
    const int b0 = tid * per, b1 = min(b0 + per, num_experts);
    int c_cnt = 0, c_u = 0, c_items = 0;
    for (int e = b0; e < b1; ++e) {
        const int c = hist[e];
        c_cnt += c;
        c_u += c > 0;
        c_items += (c + ppt - 1) / ppt;
    }
    // pack three sums: do the scan three times through s_part (simple, once per call)
    int scans[3] = {c_cnt, c_u, c_items};
    int excl[3];
    for (int k = 0; k < 3; ++k) {
        s_part[tid] = scans[k];
        __syncthreads();
        for (int off = 1; off < nt; off <<= 1) {
            const int add = tid >= off ? s_part[tid - off] : 0;
            __syncthreads();
            s_part[tid] += add;
            __syncthreads();
        }
        excl[k] = s_part[tid] - scans[k];
        if (tid == nt - 1) {
            if (k == 1) s_total[0] = s_part[tid];
            if (k == 2) s_total[1] = s_part[tid];
        }
        __syncthreads();
    }
    const int rtiles = out_features / 16;
    int run_cnt = excl[0], run_u = excl[1], run_items = excl[2];
    for (int e = b0; e < b1; ++e) {
        const int c = hist[e];
        if (c > 0) {
            uniq[run_u] = e;
            seg[run_u] = run_cnt;
            ubase[run_u] = run_items * rtiles;
            ++run_u;
        }
        hist[e] = run_cnt;  // becomes the scatter cursor
        run_cnt += c;
        run_items += (c + ppt - 1) / ppt;
    }
    __syncthreads();
    if (tid == nt - 1) {
        // the last thread's running count is the number of routable pairs
        const int U = s_total[0];
        const int items = s_total[1] * rtiles;
        hdr[1] = U;
        hdr[2] = items;
        seg[U] = run_cnt;
        ubase[U] = items;
    }
    __syncthreads();
    for (int p = tid; p < pairs; p += nt) {
        const int e = sel[p];
        const int t = ptok[p];
        if (e >= 0 && e < num_experts && t >= 0 && t < x_rows) {
            const int pos = atomicAdd(&hist[e], 1);
            order[pos] = p;
        }
    }
}

template <typename XT>
__global__ void __launch_bounds__(256)
gemv_prep_kernel(const XT *__restrict__ x, int n, int x_rows, const int32_t *__restrict__ sel,
                 const int32_t *__restrict__ tok, int pairs, int num_experts,
                 int out_features, int ppt, GemvLayout L, char *__restrict__ ws, void *y,
                 int y_elem) {
    if ((int)blockIdx.x < x_rows) {
        prep_row<XT>(x, n, blockIdx.x, L, ws);
    } else {
        route_pairs(sel, tok, pairs, x_rows, num_experts, out_features, ppt, L, ws, y, y_elem);
    }
}

// ------------------------------------------------------------- gemv kernel

constexpr int kWarps = 8;
constexpr int kStages = 4;
constexpr int kChunkK = 512;         // weights per row per ring stage
constexpr int kStepsPerChunk = 16;   // 32-weight k-steps per stage

template <int MEMBER> struct Geo {
    // ring stage: 16 rows of the main code stream for kChunkK weights
    static constexpr int kRowChunkBytes = MEMBER == IQK_IQ1_S_R4 ? 64 : 128;
    static constexpr int kRowStride = MEMBER == IQK_IQ1_S_R4 ? 80 : 144;  // bank-staggered
    static constexpr int kStageBytes = 16 * kRowStride;
};

// Per-warp scale-stream block for one 16-row tile, all streams but qs.
template <int MEMBER> __host__ __device__ constexpr int scale_block_bytes(int n) {
    return MEMBER == IQK_IQ2_KS ? 16 * (n / 64 + n / 256 + n / 256) + 32
           : MEMBER == IQK_IQ2_K ? 16 * (n / 32 + n / 128 + n / 128)
                                 : 16 * (n / 16) + 32;
}

template <int MEMBER>
__host__ __device__ constexpr int gemv_smem_bytes(int n) {
    return kWarps * (kStages * Geo<MEMBER>::kStageBytes + 2 * scale_block_bytes<MEMBER>(n)) +
           (MEMBER == IQK_IQ1_S_R4 ? 4096 : 0);
}

struct GemvArgs {
    const void *s[5];
    int64_t out_features;
    int n;
    int x_rows;
    GemvLayout L;
    const char *ws;
    void *y;
    int y_dtype;
};

template <int MEMBER>
__global__ void __launch_bounds__(kWarps * 32, 1)
gemv_kernel(GemvArgs a) {
    extern __shared__ __align__(16) char smem[];
    using G = Geo<MEMBER>;
    const int n = a.n;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int g = lane >> 2, tig = lane & 3;
    const int sbb = scale_block_bytes<MEMBER>(n);
    char *wsm = smem + wid * (kStages * G::kStageBytes + 2 * sbb);
    char *ring = wsm;
    char *scal = wsm + kStages * G::kStageBytes;
    uint16_t *grid = reinterpret_cast<uint16_t *>(smem + kWarps * (kStages * G::kStageBytes + 2 * sbb));
    if (MEMBER == IQK_IQ1_S_R4) {
        for (int i = threadIdx.x; i < 2048; i += blockDim.x) grid[i] = g_iq1s_grid[i];
        __syncthreads();
    }

    const int32_t *hdr = reinterpret_cast<const int32_t *>(a.ws + a.L.hdr);
    const int32_t *uniq = reinterpret_cast<const int32_t *>(a.ws + a.L.uniq);
    const int32_t *seg = reinterpret_cast<const int32_t *>(a.ws + a.L.seg);
    const int32_t *ubase = reinterpret_cast<const int32_t *>(a.ws + a.L.ubase);
    const int32_t *order = reinterpret_cast<const int32_t *>(a.ws + a.L.order);
    const int32_t *ptok = reinterpret_cast<const int32_t *>(a.ws + a.L.ptok);
    const int32_t *xscale = reinterpret_cast<const int32_t *>(a.ws + a.L.xscale);
    const int8_t *xbuf = reinterpret_cast<const int8_t *>(a.ws + a.L.xbuf);

    const int U = hdr[1];
    const int items = hdr[2];
    const int nwarps = gridDim.x * kWarps;
    const int gw = blockIdx.x * kWarps + wid;
    const int i0 = (int)((int64_t)items * gw / nwarps);
    const int i1 = (int)((int64_t)items * (gw + 1) / nwarps);
    if (i0 >= i1) return;
    const int chunks = n / kChunkK;
    const int rtiles = (int)(a.out_features / 16);
    constexpr int ppt = MEMBER == IQK_IQ2_K ? 1 : 2;

    // Resolve an item into (expert, first row, pair tile) -------------------
    struct Item {
        int e, r0, pfirst, npair;
    };
    auto resolve = [&](int i) -> Item {
        int lo = 0, hi = U;  // ubase[lo] <= i < ubase[hi]
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (ubase[mid] <= i) lo = mid;
            else hi = mid;
        }
        const int cnt = seg[lo + 1] - seg[lo];
        const int ntile = (cnt + ppt - 1) / ppt;
        const int local = i - ubase[lo];
        const int rt = local / ntile, pt = local - rt * ntile;
        Item it;
        it.e = uniq[lo];
        it.r0 = rt * 16;
        it.pfirst = seg[lo] + pt * ppt;
        it.npair = min(ppt, cnt - pt * ppt);
        return it;
    };

    // Issue one ring stage (item, chunk); chunk 0 also brings the scale block.
    auto issue = [&](int stage_idx, const Item &it, int item_ord, int c) {
        const int64_t rowbase = (int64_t)it.e * a.out_features + it.r0;
        char *dst = ring + (stage_idx % kStages) * G::kStageBytes;
        const char *qs = static_cast<const char *>(a.s[0]);
        const int qrow = MEMBER == IQK_IQ1_S_R4 ? n / 8 : n / 4;  // bytes per qs row
        constexpr int per_row = G::kRowChunkBytes / 16;
        for (int i = lane; i < 16 * per_row; i += 32) {
            const int r = i / per_row, q = i - r * per_row;
            cp_async16(dst + r * G::kRowStride + q * 16,
                       qs + (rowbase + r) * qrow + (int64_t)c * G::kRowChunkBytes + q * 16);
        }
        if (c == 0) {
            char *sd = scal + (item_ord & 1) * sbb;
            int off = 0;
            const RowBytes rb = row_bytes(MEMBER, n);
            for (int si = 1; si < rb.count; ++si) {
                const int bytes = (int)(16 * rb.b[si]);
                const char *src = static_cast<const char *>(a.s[si]) + rowbase * rb.b[si];
                for (int i = lane * 16; i < bytes; i += 32 * 16) cp_async16(sd + off + i, src + i);
                off += bytes;
            }
        }
    };

    const int total_stages = (i1 - i0) * chunks;
    // stage index j -> (item ordinal j / chunks, chunk j % chunks)
    Item it_issue = resolve(i0);
    int issue_ord = 0;
#pragma unroll 1
    for (int j = 0; j < kStages - 1; ++j) {
        if (j < total_stages) {
            const int ord = j / chunks, c = j - ord * chunks;
            if (ord != issue_ord) {
                issue_ord = ord;
                it_issue = resolve(i0 + ord);
            }
            issue(j, it_issue, ord, c);
        }
        cp_async_commit();
    }

    // Per-item state
    Item it{};
    int32_t tot[4] = {0, 0, 0, 0};
    double acc_g[2] = {0.0, 0.0}, acc_g8[2] = {0.0, 0.0};  // IQ2_K super-block sums
    const int8_t *xcol = nullptr;  // activation planes for this lane's B column
    bool col_live = false;
    int tok_t[2] = {-1, -1};
    int pair_t[2] = {-1, -1};

#pragma unroll 1
    for (int j = 0; j < total_stages; ++j) {
        const int ord = j / chunks, c = j - ord * chunks;
        if (c == 0) {
            it = resolve(i0 + ord);
            for (int t = 0; t < 2; ++t) {
                pair_t[t] = t < it.npair ? order[it.pfirst + t] : -1;
                tok_t[t] = pair_t[t] >= 0 ? ptok[pair_t[t]] : -1;
            }
            // B column of this lane: IQ2_KS / IQ1: col g = 4*t + plane;
            // IQ2_K: col g = 2*plane + half (1 pair per tile).
            int t, p;
            if (MEMBER == IQK_IQ2_K) {
                t = 0;
                p = g >> 1;
                col_live = p < 3 && (g & 1) == (tig >> 1) && tok_t[0] >= 0;
            } else {
                t = g >> 2;
                p = g & 3;
                col_live = p < 3 && tok_t[t] >= 0;
            }
            xcol = col_live ? xbuf + (int64_t)tok_t[t] * a.L.xrow_bytes + p * 32 + tig * 8 : nullptr;
            tot[0] = tot[1] = tot[2] = tot[3] = 0;
            acc_g[0] = acc_g[1] = acc_g8[0] = acc_g8[1] = 0.0;
        }
        cp_async_wait<kStages - 2>();
        __syncwarp();
        // Refill the slot consumed in the previous iteration, S-1 stages ahead.
        {
            const int jn = j + kStages - 1;
            if (jn < total_stages) {
                const int ordn = jn / chunks, cn = jn - ordn * chunks;
                if (ordn != issue_ord) {
                    issue_ord = ordn;
                    it_issue = resolve(i0 + ordn);
                }
                issue(jn, it_issue, ordn, cn);
            }
            cp_async_commit();
        }

        const char *st = ring + (j % kStages) * G::kStageBytes;
        const char *sd = scal + (ord & 1) * sbb;
        // B fragments for the 16 k-steps of this chunk
        uint32_t bf[kStepsPerChunk][2];
#pragma unroll
        for (int ls = 0; ls < kStepsPerChunk; ++ls) {
            if (col_live) {
                const uint2 v = ldg_nc_u2(xcol + (int64_t)(c * kStepsPerChunk + ls) * 128);
                bf[ls][0] = v.x;
                bf[ls][1] = v.y;
            } else {
                bf[ls][0] = bf[ls][1] = 0;
            }
        }
        // IQ1_S_R4: block sums of this lane's two C columns (token tig>>1,
        // planes 2*(tig&1) and +1; plane 3 reads the stored zero).
        int32_t xbs[MEMBER == IQK_IQ1_S_R4 ? kStepsPerChunk : 1][2];
        if (MEMBER == IQK_IQ1_S_R4) {
            const int ct = tig >> 1, cp = 2 * (tig & 1);
#pragma unroll
            for (int ls = 0; ls < kStepsPerChunk; ++ls) {
                if (tok_t[ct] >= 0) {
                    const uint2 v = ldg_nc_u2(xbuf + (int64_t)tok_t[ct] * a.L.xrow_bytes +
                                              (int64_t)(c * kStepsPerChunk + ls) * 128 + 96 + cp * 4);
                    xbs[ls][0] = (int32_t)v.x;
                    xbs[ls][1] = (int32_t)v.y;
                } else {
                    xbs[ls][0] = xbs[ls][1] = 0;
                }
            }
        }

#pragma unroll
        for (int ls = 0; ls < kStepsPerChunk; ++ls) {
            const int s = c * kStepsPerChunk + ls;  // global k-step (32 weights)
            uint32_t A[4];
            if (MEMBER == IQK_IQ1_S_R4) {
                const uint32_t qg = *reinterpret_cast<const uint32_t *>(st + g * G::kRowStride + ls * 4);
                const uint32_t qg8 = *reinterpret_cast<const uint32_t *>(st + (g + 8) * G::kRowStride + ls * 4);
                const uint16_t *qh = reinterpret_cast<const uint16_t *>(sd);
                const uint32_t hg = qh[g * (n / 32) + s];
                const uint32_t hg8 = qh[(g + 8) * (n / 32) + s];
                const uint32_t ig = ((qg >> (8 * tig)) & 0xffu) | (((hg >> (3 * tig)) & 7u) << 8);
                const uint32_t ig8 = ((qg8 >> (8 * tig)) & 0xffu) | (((hg8 >> (3 * tig)) & 7u) << 8);
                const uint32_t v = (uint32_t)grid[ig] | ((uint32_t)grid[ig8] << 16);
                const uint32_t s0 = v & 0x33333333u;
                const uint32_t s1 = (v >> 2) & 0x33333333u;
                A[0] = prmt(kTernTab, 0u, s0);
                A[1] = prmt(kTernTab, 0u, s0 >> 16);
                A[2] = prmt(kTernTab, 0u, s1);
                A[3] = prmt(kTernTab, 0u, s1 >> 16);
                int32_t d[4];
                mma_s8(d, A, bf[ls][0], bf[ls][1]);
                const int xb0 = xbs[MEMBER == IQK_IQ1_S_R4 ? ls : 0][0];
                const int xb1 = xbs[MEMBER == IQK_IQ1_S_R4 ? ls : 0][1];
                const int mg = 2 * (int)((hg >> 12) & 7u) + 1;
                const int mg8 = 2 * (int)((hg8 >> 12) & 7u) + 1;
                const int sg = (hg & 0x8000u) ? -1 : 1;
                const int sg8 = (hg8 & 0x8000u) ? -1 : 1;
                tot[0] += mg * (8 * d[0] + sg * xb0);
                tot[1] += mg * (8 * d[1] + sg * xb1);
                tot[2] += mg8 * (8 * d[2] + sg8 * xb0);
                tot[3] += mg8 * (8 * d[3] + sg8 * xb1);
            } else {
                const uint32_t wg = *reinterpret_cast<const uint32_t *>(
                    st + g * G::kRowStride + (2 * ls + (tig >> 1)) * 4);
                const uint32_t wg8 = *reinterpret_cast<const uint32_t *>(
                    st + (g + 8) * G::kRowStride + (2 * ls + (tig >> 1)) * 4);
                const uint32_t v = prmt(wg, wg8, (tig & 1) ? 0x7632u : 0x5410u);
                int alpha_g, alpha_g8, idx_g0, idx_g1, idx_g80, idx_g81;
                if (MEMBER == IQK_IQ2_KS) {
                    const uint8_t *scl = reinterpret_cast<const uint8_t *>(sd);
                    const uint8_t *sch = scl + 16 * (n / 64);
                    const uint8_t *sex = sch + 16 * (n / 256);
                    const int sb = (s & 1) * 4;
                    const int lo_g = (scl[g * (n / 64) + (s >> 1)] >> sb) & 15;
                    const int lo_g8 = (scl[(g + 8) * (n / 64) + (s >> 1)] >> sb) & 15;
                    const int hi_g = (sch[g * (n / 256) + (s >> 3)] >> (s & 7)) & 1;
                    const int hi_g8 = (sch[(g + 8) * (n / 256) + (s >> 3)] >> (s & 7)) & 1;
                    alpha_g = (sex[g * (n / 256) + (s >> 3)] >> (s & 7)) & 1;
                    alpha_g8 = (sex[(g + 8) * (n / 256) + (s >> 3)] >> (s & 7)) & 1;
                    idx_g0 = idx_g1 = (lo_g | (hi_g << 4)) - 16;
                    idx_g80 = idx_g81 = (lo_g8 | (hi_g8 << 4)) - 16;
                } else {
                    const uint8_t *scl = reinterpret_cast<const uint8_t *>(sd);
                    const uint8_t *sex = scl + 16 * (n / 32);
                    const int sbk = 2 * s + (tig >> 1);  // sub-block of this lane's codes
                    alpha_g = (sex[g * (n / 128) + (sbk >> 3)] >> (sbk & 7)) & 1;
                    alpha_g8 = (sex[(g + 8) * (n / 128) + (sbk >> 3)] >> (sbk & 7)) & 1;
                    const int bg = scl[g * (n / 32) + s];
                    const int bg8 = scl[(g + 8) * (n / 32) + s];
                    idx_g0 = (bg & 15) - 8;
                    idx_g1 = (bg >> 4) - 8;
                    idx_g80 = (bg8 & 15) - 8;
                    idx_g81 = (bg8 >> 4) - 8;
                }
                const uint32_t tab_g = alpha_g ? kIq2Tab1 : kIq2Tab0;
                const uint32_t tab_g8 = alpha_g8 ? kIq2Tab1 : kIq2Tab0;
                const uint32_t s0 = (v & 0x33333333u) | 0x44440000u;
                const uint32_t s1 = ((v >> 2) & 0x33333333u) | 0x44440000u;
                A[0] = prmt(tab_g, tab_g8, s0);
                A[1] = prmt(tab_g, tab_g8, s0 >> 16);
                A[2] = prmt(tab_g, tab_g8, s1);
                A[3] = prmt(tab_g, tab_g8, s1 >> 16);
                int32_t d[4];
                mma_s8(d, A, bf[ls][0], bf[ls][1]);
                tot[0] += idx_g0 * d[0];
                tot[1] += idx_g1 * d[1];
                tot[2] += idx_g80 * d[2];
                tot[3] += idx_g81 * d[3];
                if (MEMBER == IQK_IQ2_K && (s & 7) == 7) {
                    // end of a 256-weight super-block: fold in its fp16 scale
                    const int sbi = s >> 3;
                    const uint16_t *dvp = reinterpret_cast<const uint16_t *>(
                        sd + 16 * (n / 32) + 16 * (n / 128));
                    const int32_t pg = tot[0] + tot[1], pg8 = tot[2] + tot[3];
                    const int32_t p1g = __shfl_down_sync(0xffffffffu, pg, 1);
                    const int32_t p2g = __shfl_down_sync(0xffffffffu, pg, 2);
                    const int32_t p1g8 = __shfl_down_sync(0xffffffffu, pg8, 1);
                    const int32_t p2g8 = __shfl_down_sync(0xffffffffu, pg8, 2);
                    if (tig == 0) {
                        const double Tg = (double)pg * 65536.0 + (double)p1g * 256.0 + (double)p2g;
                        const double Tg8 = (double)pg8 * 65536.0 + (double)p1g8 * 256.0 + (double)p2g8;
                        acc_g[0] += (double)half_bits_to_float(dvp[g * (n / 256) + sbi]) * Tg;
                        acc_g8[0] += (double)half_bits_to_float(dvp[(g + 8) * (n / 256) + sbi]) * Tg8;
                    }
                    tot[0] = tot[1] = tot[2] = tot[3] = 0;
                }
            }
        }
        __syncwarp();

        if (c == chunks - 1) {
            // ---- item epilogue: combine digit planes, scale, store
            const char *sdd = sd;
            double yg[2], yg8[2];
            int nt_out;
            if (MEMBER == IQK_IQ2_K) {
                nt_out = 1;
                yg[0] = acc_g[0];
                yg8[0] = acc_g8[0];
            } else {
                // lanes with even tig hold planes (0,1) of token tig>>1; odd hold (2, pad)
                const int32_t n0 = __shfl_down_sync(0xffffffffu, tot[0], 1);
                const int32_t n2 = __shfl_down_sync(0xffffffffu, tot[2], 1);
                nt_out = 2;
                const double Tg = (double)tot[0] * 65536.0 + (double)tot[1] * 256.0 + (double)n0;
                const double Tg8 = (double)tot[2] * 65536.0 + (double)tot[3] * 256.0 + (double)n2;
                const uint16_t *dvp = reinterpret_cast<const uint16_t *>(
                    sdd + (MEMBER == IQK_IQ2_KS ? 16 * (n / 64 + n / 256 + n / 256) : 16 * (n / 16)));
                const double dg = half_bits_to_float(dvp[g]);
                const double dg8 = half_bits_to_float(dvp[g + 8]);
                yg[0] = dg * Tg;
                yg8[0] = dg8 * Tg8;
            }
            const bool writer = MEMBER == IQK_IQ2_K ? tig == 0 : (tig & 1) == 0;
            const int t = MEMBER == IQK_IQ2_K ? 0 : tig >> 1;
            if (writer && t < nt_out && pair_t[t] >= 0) {
                const int S = xscale[tok_t[t]];
                const int sh = -S - (MEMBER == IQK_IQ1_S_R4 ? 3 : 0);
                float vg, vg8;
                if (S == kScaleNonFinite) {
                    vg = vg8 = __int_as_float(0x7fc00000);
                } else {
                    vg = (float)ldexp(yg[0], sh);
                    vg8 = (float)ldexp(yg8[0], sh);
                }
                const int64_t o0 = (int64_t)pair_t[t] * a.out_features + it.r0 + g;
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
    L.uniq = take(sizeof(int32_t) * (pairs + 1));
    L.seg = take(sizeof(int32_t) * (pairs + 2));
    L.ubase = take(sizeof(int32_t) * (pairs + 2));
    L.order = take(sizeof(int32_t) * (pairs + 1));
    L.ptok = take(sizeof(int32_t) * (pairs + 1));
    L.xscale = take(sizeof(int32_t) * (x_rows + 1));
    L.xrow_bytes = 4 * n;  // (n/32 k-steps) x (4 planes) x (4 lanes) x 8 bytes
    L.xbuf = take((size_t)(x_rows * L.xrow_bytes));
    L.total = off;
    return L;
}

int gemv_smem_for(int member, int n) {
    if (member == IQK_IQ2_KS) return gemv_smem_bytes<IQK_IQ2_KS>(n);
    if (member == IQK_IQ2_K) return gemv_smem_bytes<IQK_IQ2_K>(n);
    return gemv_smem_bytes<IQK_IQ1_S_R4>(n);
}

cudaError_t launch_gemv(int member, const void *x, int x_dtype, int64_t x_rows,
                        const void *const *streams, int64_t num_experts,
                        int64_t out_features, int n, const int32_t *sel,
                        const int32_t *tok, int64_t pairs, void *y, int y_dtype,
                        void *ws, cudaStream_t stream, int num_sms) {
    const GemvLayout L = gemv_layout(member, n, x_rows, pairs);
    char *w = static_cast<char *>(ws);
    cudaError_t err = cudaMemsetAsync(w + L.hdr, 0, 64, stream);
    if (err != cudaSuccess) return err;
    const int ppt = member == IQK_IQ2_K ? 1 : 2;
    const int y_elem = y_dtype == IQK_F32 ? 4 : 2;
    const size_t hist_bytes = sizeof(int32_t) * (size_t)num_experts;
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
#define IQK_PREP(T)                                                                       \
    gemv_prep_kernel<T><<<pblocks, 256, hist_bytes, stream>>>(                            \
        static_cast<const T *>(x), n, (int)x_rows, sel, tok, (int)pairs, (int)num_experts, \
        (int)out_features, ppt, L, w, y, y_elem)
    if (x_dtype == IQK_F32) IQK_PREP(float);
    else if (x_dtype == IQK_F16) IQK_PREP(__half);
    else IQK_PREP(__nv_bfloat16);
#undef IQK_PREP
    err = cudaGetLastError();
    if (err != cudaSuccess) return err;

    GemvArgs ga{};
    const RowBytes rb = row_bytes(member, n);
    for (int i = 0; i < rb.count; ++i) ga.s[i] = streams[i];
    ga.out_features = out_features;
    ga.n = n;
    ga.x_rows = (int)x_rows;
    ga.L = L;
    ga.ws = w;
    ga.y = y;
    ga.y_dtype = y_dtype;
    const int smem = gemv_smem_for(member, n);
    // Upper bound on work items: every pair its own tile of every row tile.
    const int64_t max_items = pairs * (out_features / 16);
    int64_t blocks = (max_items + kWarps - 1) / kWarps;
    if (blocks > num_sms) blocks = num_sms;
    if (blocks < 1) blocks = 1;
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
