// iqk_gemv_static: the fused dequant + GEMV with its scratch in a static
// device array instead of a caller-provided workspace.
//
// Some callers cannot allocate device memory at the point where they launch:
// a host runtime that hands out only its own pre-planned buffers (an
// inference server whose memory plan is fixed before the first request),
// code running inside a custom allocator's hooks (where asking the
// allocator again would re-enter it), or a foreign-language binding that
// has no device allocator of its own. This entry point needs nothing from
// them beyond x, sel, tok and y: its scratch is the file-scope array below,
// resolved once per device with cudaGetSymbolAddress.
//
// Nothing here calls cudaMalloc, cudaFree or any allocating library. The
// kernels are the same ones iqk_gemv launches (iqk_gemv.cu); only where the
// scratch lives differs.
#include <atomic>
#include <mutex>

#include "iqk_common.cuh"
#include "iqk_gemv.cuh"

namespace {

using namespace iqk;

// Largest scratch one call may use: the iqk_gemv workspace of its geometry
// must fit. 1 MiB covers 64 activation rows with 512 pairs at
// in_features 4096 (or 128 rows at 2048) -- a decode step of up to 8 tokens
// with top-6 routing, for the gate/up seam and the down seam alike.
constexpr size_t kStaticScratchBytes = size_t(1) << 20;
constexpr int kMaxDevices = 64;

// No byte of it needs to start at zero: the preparation kernel writes every
// field the run kernel reads (error word, tile count, order, tiles, scales,
// activation planes) before the run kernel starts.
__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

// The array's address belongs to one CUDA context: every context that loads
// this library's device code gets its own copy. The cache therefore keeps,
// per device ordinal, the context the address was resolved in, and resolves
// again when a different context is current (a non-primary driver context,
// or the primary context re-created after cudaDeviceReset).
struct ScratchEntry {
    void *ctx = nullptr;
    void *ptr = nullptr;
};
ScratchEntry g_scratch[kMaxDevices];
std::mutex g_scratch_mutex;

// The current driver context, through the runtime's driver entry point (the
// library does not link libcuda). nullptr when it cannot be queried.
void *current_context() {
    using GetCtxFn = int (*)(void **);
    static std::atomic<GetCtxFn> fn{nullptr};
    GetCtxFn f = fn.load(std::memory_order_acquire);
    if (!f) {
        void *sym = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &sym, cudaEnableDefault, &q) !=
                cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !sym)
            return nullptr;
        f = reinterpret_cast<GetCtxFn>(sym);
        fn.store(f, std::memory_order_release);
    }
    void *ctx = nullptr;
    return f(&ctx) == 0 ? ctx : nullptr;
}

// Address of the current context's copy of g_static_scratch. The first call
// in a context resolves it with cudaGetSymbolAddress, which may load the
// library's device code there; later calls in that context reuse it.
cudaError_t scratch_for_current_device(void **out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    // No context may be current yet (nothing else has touched the device in
    // this thread): then resolve, which makes the primary context current,
    // and record the context that is current afterwards.
    void *ctx = current_context();
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    ScratchEntry &e = g_scratch[dev];
    if (!e.ptr || !ctx || e.ctx != ctx) {
        void *p = nullptr;
        err = cudaGetSymbolAddress(&p, g_static_scratch);
        if (err != cudaSuccess) return err;
        if (!p) return cudaErrorInvalidSymbol;
        e.ptr = p;
        e.ctx = current_context();
    }
    *out = e.ptr;
    return cudaSuccess;
}

}  // namespace

extern "C" {

size_t iqk_gemv_static_max_bytes(void) { return kStaticScratchBytes; }

int iqk_gemv_static(int member, const void *x, int x_dtype, int64_t x_rows,
                    const void *const *streams, int64_t num_experts, int64_t out_features,
                    int64_t in_features, const int32_t *sel, const int32_t *tok, int64_t pairs,
                    void *y, int y_dtype, iqk_stream_t stream) {
    if (member != IQK_IQ2_KS && member != IQK_IQ2_K && member != IQK_IQ1_S_R4)
        return IQK_ERR_MEMBER;
    if (in_features != 2048 && in_features != 4096) return IQK_ERR_WIDTH;
    if (x_rows < 0 || pairs < 0 || x_rows > (1 << 24) || pairs > (1 << 24))
        return IQK_ERR_GEOMETRY;
    // Checked before anything touches the device, so an oversized call fails
    // the same way on every device and never resolves the scratch.
    if (gemv_layout(member, in_features, x_rows, pairs).total > kStaticScratchBytes)
        return IQK_ERR_WORKSPACE;
    if (pairs == 0) return iqk_gemv(member, x, x_dtype, x_rows, streams, num_experts,
                                    out_features, in_features, sel, tok, pairs, y, y_dtype,
                                    nullptr, 0, stream);
    void *scratch = nullptr;
    if (scratch_for_current_device(&scratch) != cudaSuccess) {
        cudaGetLastError();
        return IQK_ERR_CUDA;
    }
    return iqk_gemv(member, x, x_dtype, x_rows, streams, num_experts, out_features,
                    in_features, sel, tok, pairs, y, y_dtype, scratch, kStaticScratchBytes,
                    stream);
}

int iqk_gemv_static_read_error(int64_t in_features, int64_t x_rows, int64_t pairs,
                               int32_t *flags, iqk_stream_t stream) {
    if (!flags) return IQK_ERR_ARGUMENT;
    if (in_features != 2048 && in_features != 4096) return IQK_ERR_WIDTH;
    if (x_rows < 0 || pairs < 0 || x_rows > (1 << 24) || pairs > (1 << 24))
        return IQK_ERR_GEOMETRY;
    if (gemv_layout(IQK_IQ2_KS, in_features, x_rows, pairs).total > kStaticScratchBytes)
        return IQK_ERR_WORKSPACE;
    void *scratch = nullptr;
    if (scratch_for_current_device(&scratch) != cudaSuccess) {
        cudaGetLastError();
        return IQK_ERR_CUDA;
    }
    return iqk_read_error(scratch, in_features, x_rows, pairs, flags, stream);
}

}  // extern "C"
