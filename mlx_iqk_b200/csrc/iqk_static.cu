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

std::atomic<void *> g_scratch_ptr[kMaxDevices];
std::mutex g_scratch_mutex;

// Address of this device's copy of g_static_scratch. The first call on a
// device resolves it with cudaGetSymbolAddress, which may load the library's
// device code onto that device; later calls read the cached pointer.
cudaError_t scratch_for_current_device(void **out) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    void *p = g_scratch_ptr[dev].load(std::memory_order_acquire);
    if (!p) {
        std::lock_guard<std::mutex> lock(g_scratch_mutex);
        p = g_scratch_ptr[dev].load(std::memory_order_relaxed);
        if (!p) {
            err = cudaGetSymbolAddress(&p, g_static_scratch);
            if (err != cudaSuccess) return err;
            if (!p) return cudaErrorInvalidSymbol;
            g_scratch_ptr[dev].store(p, std::memory_order_release);
        }
    }
    *out = p;
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

}  // extern "C"
