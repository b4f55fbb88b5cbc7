// extern "C" entry points of libiqk_b200.so (declared in include/iqk_b200.h).
//
// Every entry point validates its geometry and pointers on the host before
// any launch (the reference fails closed the same way before compiling:
// src/mlx_iqk/kernels.py:100-128, src/mlx_iqk/nn.py:110-126) and returns a
// status instead of raising.
#include <atomic>
#include <cstdio>

#include "iqk_common.cuh"
#include "iqk_gemv.cuh"
#include "iqk_dense.cuh"
#include "iqk_grouped.cuh"

namespace {

using namespace iqk;

bool member_ok(int m) { return m == IQK_IQ2_KS || m == IQK_IQ2_K || m == IQK_IQ1_S_R4; }
bool dtype_ok(int d) { return d == IQK_F32 || d == IQK_F16 || d == IQK_BF16; }
bool width_ok(int64_t n) { return n == 2048 || n == 4096; }
bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// SM count of the current device, queried once per device.
int num_sms_current() {
    static std::atomic<int> cached[64];
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 148;
    if (dev >= 0 && dev < 64 && (sms = cached[dev].load()) > 0) return sms;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
        sms = 148;
    if (dev >= 0 && dev < 64) cached[dev].store(sms);
    return sms;
}

// Stream pointers: present, and 16-byte aligned (the kernels move them with
// 16-byte copies; the caller's allocator gives 256).
int check_streams(int member, const void *const *streams) {
    if (!streams) return IQK_ERR_ARGUMENT;
    const RowBytes rb = row_bytes(member, 2048);
    for (int i = 0; i < rb.count; ++i) {
        if (!streams[i]) return IQK_ERR_ARGUMENT;
        if (!aligned(streams[i], 16)) return IQK_ERR_ALIGNMENT;
    }
    return IQK_OK;
}

bool dense_member_ok(int m) {
    return m == IQK_IQ4_KS || m == IQK_IQ4_K || m == IQK_IQ5_K || m == IQK_IQ6_K;
}
bool dense_width_ok(int64_t n) { return n == 1024 || n == 2048 || n == 4096 || n == 8192; }

// Dense streams: present and 16-byte aligned (the GEMV stages every stream's
// rows with 16-byte asynchronous copies; rows of every width are whole
// 16-byte multiples, so aligned bases keep every copy aligned).
int check_dense_streams(int member, const void *const *streams) {
    if (!streams) return IQK_ERR_ARGUMENT;
    const int count = member == IQK_IQ4_KS ? 3 : member == IQK_IQ5_K ? 6 : 5;
    for (int i = 0; i < count; ++i) {
        if (!streams[i]) return IQK_ERR_ARGUMENT;
        if (!aligned(streams[i], 16)) return IQK_ERR_ALIGNMENT;
    }
    return IQK_OK;
}

int cuda_status(cudaError_t err) {
    if (err == cudaSuccess) return IQK_OK;
    cudaGetLastError();  // clear a sticky launch error for the caller
    return IQK_ERR_CUDA;
}

}  // namespace

extern "C" {

const char *iqk_status_string(int status) {
    switch (status) {
        case IQK_OK: return "ok";
        case IQK_ERR_MEMBER: return "member is not one of iq2_ks, iq2_k, iq1_s_r4";
        case IQK_ERR_WIDTH: return "in_features is not a sized width (2048 or 4096)";
        case IQK_ERR_GEOMETRY: return "geometry rejected (out_features, experts, rows or pairs)";
        case IQK_ERR_ARGUMENT: return "invalid argument (null pointer, dtype or count)";
        case IQK_ERR_ALIGNMENT: return "pointer is not 16-byte aligned";
        case IQK_ERR_WORKSPACE: return "workspace missing or too small";
        case IQK_ERR_CUDA: return "CUDA runtime error";
        case IQK_ERR_DEVICE: return "current device is not compute capability 10.0";
        default: return "unknown status";
    }
}

int iqk_abi_version(void) { return 1; }

int iqk_dense_dequant(int member, const void *const *streams, int64_t out_features,
                      int64_t in_features, int64_t row_start, int64_t rows, int out_dtype,
                      void *dst, iqk_stream_t stream) {
    if (!dense_member_ok(member)) return IQK_ERR_MEMBER;
    if (!dense_width_ok(in_features)) return IQK_ERR_WIDTH;
    if (out_features <= 0 || out_features > ((int64_t)1 << 31)) return IQK_ERR_GEOMETRY;
    if (row_start < 0 || rows < 0 || row_start + rows > out_features) return IQK_ERR_GEOMETRY;
    if (!dtype_ok(out_dtype)) return IQK_ERR_ARGUMENT;
    if (rows == 0) return IQK_OK;
    if (!dst) return IQK_ERR_ARGUMENT;
    if (!aligned(dst, 16)) return IQK_ERR_ALIGNMENT;
    const int st = check_dense_streams(member, streams);
    if (st != IQK_OK) return st;
    return cuda_status(launch_dense_dequant(member, streams, (int)in_features, row_start, rows,
                                            dst, out_dtype, reinterpret_cast<cudaStream_t>(stream),
                                            num_sms_current()));
}

int iqk_dense_gemv(int member, const void *x, int64_t tokens, const void *const *streams,
                   int64_t out_features, int64_t in_features, void *y, int y_dtype,
                   iqk_stream_t stream) {
    if (!dense_member_ok(member)) return IQK_ERR_MEMBER;
    if (!dense_width_ok(in_features)) return IQK_ERR_WIDTH;
    if (out_features <= 0 || out_features % 16 || out_features > ((int64_t)1 << 30))
        return IQK_ERR_GEOMETRY;
    if (tokens < 0 || tokens > (1 << 24)) return IQK_ERR_GEOMETRY;
    if (y_dtype != IQK_F16 && y_dtype != IQK_F32) return IQK_ERR_ARGUMENT;
    if (tokens == 0) return IQK_OK;
    if (!x || !y) return IQK_ERR_ARGUMENT;
    if (!aligned(x, 16) || !aligned(y, 4)) return IQK_ERR_ALIGNMENT;  // x: 8-byte fragment loads
    const int st = check_dense_streams(member, streams);
    if (st != IQK_OK) return st;
    return cuda_status(launch_dense_gemv(member, streams, (int)in_features, (int)out_features, x,
                                         (int)tokens, y, y_dtype,
                                         reinterpret_cast<cudaStream_t>(stream)));
}

int iqk_check_bounded_wait(int64_t limit_ns, int32_t *flags, iqk_stream_t stream) {
    if (limit_ns < 0 || limit_ns > 2000000000LL) return IQK_ERR_ARGUMENT;
    if (!flags) return IQK_ERR_ARGUMENT;
    if (!aligned(flags, 4)) return IQK_ERR_ALIGNMENT;
    return cuda_status(launch_bounded_wait_check(limit_ns, flags,
                                                 reinterpret_cast<cudaStream_t>(stream)));
}

int iqk_check_device(void) {
    int dev = 0, major = 0, minor = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return cuda_status(cudaErrorNoDevice);
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
        return IQK_ERR_CUDA;
    return (major == 10 && minor == 0) ? IQK_OK : IQK_ERR_DEVICE;
}

int iqk_dequant(int member, const void *const *streams, int64_t num_experts,
                int64_t out_features, int64_t in_features, int64_t row_start, int64_t rows,
                int out_dtype, void *dst, iqk_stream_t stream) {
    if (!member_ok(member)) return IQK_ERR_MEMBER;
    if (!width_ok(in_features)) return IQK_ERR_WIDTH;
    if (num_experts <= 0 || out_features <= 0) return IQK_ERR_GEOMETRY;
    if (member == IQK_IQ1_S_R4 && out_features % 4) return IQK_ERR_GEOMETRY;
    if (row_start < 0 || rows < 0 || row_start + rows > out_features) return IQK_ERR_GEOMETRY;
    if (!dtype_ok(out_dtype) || !dst) return IQK_ERR_ARGUMENT;
    if (!aligned(dst, 16)) return IQK_ERR_ALIGNMENT;
    const int st = check_streams(member, streams);
    if (st != IQK_OK) return st;
    if (rows == 0) return IQK_OK;
    return cuda_status(launch_dequant(member, streams, num_experts, out_features,
                                      (int)in_features, row_start, rows, out_dtype, dst,
                                      reinterpret_cast<cudaStream_t>(stream),
                                      num_sms_current()));
}

int iqk_dequant_floor(int member, const void *const *streams, int64_t num_experts,
                      int64_t out_features, int64_t in_features, int64_t row_start,
                      int64_t rows, int out_dtype, void *dst, iqk_stream_t stream) {
    if (!member_ok(member)) return IQK_ERR_MEMBER;
    if (!width_ok(in_features)) return IQK_ERR_WIDTH;
    if (num_experts <= 0 || out_features <= 0) return IQK_ERR_GEOMETRY;
    if (member == IQK_IQ1_S_R4 && out_features % 4) return IQK_ERR_GEOMETRY;
    if (row_start < 0 || rows < 0 || row_start + rows > out_features) return IQK_ERR_GEOMETRY;
    if (!dtype_ok(out_dtype) || !dst) return IQK_ERR_ARGUMENT;
    if (!aligned(dst, 16)) return IQK_ERR_ALIGNMENT;
    const int st = check_streams(member, streams);
    if (st != IQK_OK) return st;
    if (rows == 0) return IQK_OK;
    return cuda_status(launch_dequant(member, streams, num_experts, out_features,
                                      (int)in_features, row_start, rows, out_dtype, dst,
                                      reinterpret_cast<cudaStream_t>(stream),
                                      num_sms_current(), true));
}

int iqk_pack(int member, const void *wire, int64_t rows, int64_t in_features,
             void *const *streams, iqk_stream_t stream) {
    if (!member_ok(member)) return IQK_ERR_MEMBER;
    if (in_features <= 0 || in_features % 256 || in_features > (1 << 20)) return IQK_ERR_WIDTH;
    if (rows < 0 || rows > ((int64_t)1 << 31)) return IQK_ERR_GEOMETRY;
    if (member == IQK_IQ1_S_R4 && rows % 4) return IQK_ERR_GEOMETRY;
    if (rows == 0) return IQK_OK;
    if (!wire || !streams) return IQK_ERR_ARGUMENT;
    if (!aligned(wire, 16)) return IQK_ERR_ALIGNMENT;
    const RowBytes rb = row_bytes(member, in_features);
    for (int i = 0; i < rb.count; ++i) {
        if (!streams[i]) return IQK_ERR_ARGUMENT;
        if (!aligned(streams[i], 16)) return IQK_ERR_ALIGNMENT;
    }
    return cuda_status(launch_pack(member, wire, rows, (int)in_features, streams,
                                   reinterpret_cast<cudaStream_t>(stream), num_sms_current()));
}

size_t iqk_gemv_workspace_bytes(int member, int64_t in_features, int64_t x_rows,
                                int64_t pairs) {
    if (!member_ok(member) || !width_ok(in_features) || x_rows < 0 || pairs < 0) return 0;
    return gemv_layout(member, in_features, x_rows, pairs).total;
}

size_t iqk_gemv_workspace_min_bytes(int member, int64_t in_features, int64_t x_rows,
                                    int64_t pairs) {
    if (!member_ok(member) || !width_ok(in_features) || x_rows < 0 || pairs < 0) return 0;
    return gemv_layout(member, in_features, x_rows, pairs).total;
}

// The GEMV addresses weight rows (expert * out_features + row) with 32-bit
// tensor-map coordinates and counts its work items (pair x 64-row block) in
// 32 bits.
static bool gemv_rows_ok(int64_t num_experts, int64_t out_features, int64_t pairs) {
    return num_experts * out_features <= (int64_t)1 << 30 &&
           pairs * ((out_features + 63) / 64) < (int64_t)1 << 31;
}

static int check_prepare(int64_t in_features, int64_t num_experts, int64_t x_rows,
                         int64_t pairs, const int32_t *tok, int x_dtype) {
    if (!width_ok(in_features)) return IQK_ERR_WIDTH;
    if (num_experts <= 0 || num_experts > 4096) return IQK_ERR_GEOMETRY;
    if (pairs < 0 || x_rows < 0 || pairs > (1 << 24) || x_rows > (1 << 24))
        return IQK_ERR_GEOMETRY;
    if (!tok && x_rows > 0 && pairs % x_rows) return IQK_ERR_GEOMETRY;
    if (!tok && x_rows == 0 && pairs > 0) return IQK_ERR_GEOMETRY;
    if (!dtype_ok(x_dtype)) return IQK_ERR_ARGUMENT;
    return IQK_OK;
}

int iqk_gemv_prepare(const void *x, int x_dtype, int64_t x_rows, int64_t in_features,
                     int64_t num_experts, const int32_t *sel, const int32_t *tok, int64_t pairs,
                     void *workspace, size_t workspace_bytes, iqk_stream_t stream) {
    int st = check_prepare(in_features, num_experts, x_rows, pairs, tok, x_dtype);
    if (st != IQK_OK) return st;
    if (pairs == 0) return IQK_OK;
    if (!x || !sel || !workspace) return IQK_ERR_ARGUMENT;
    if (!aligned(x, 16) || !aligned(workspace, 256)) return IQK_ERR_ALIGNMENT;
    if (workspace_bytes < gemv_layout(0, in_features, x_rows, pairs).total)
        return IQK_ERR_WORKSPACE;
    return cuda_status(launch_gemv_prepare(x, x_dtype, x_rows, (int)in_features, num_experts,
                                           sel, tok, pairs, workspace,
                                           reinterpret_cast<cudaStream_t>(stream)));
}

int iqk_gemv_run(int member, const void *const *streams, int64_t num_experts,
                 int64_t out_features, int64_t in_features, int64_t x_rows, int64_t pairs,
                 void *y, int y_dtype, const void *workspace, size_t workspace_bytes,
                 iqk_stream_t stream) {
    if (!member_ok(member)) return IQK_ERR_MEMBER;
    if (!width_ok(in_features)) return IQK_ERR_WIDTH;
    if (num_experts <= 0 || num_experts > 4096) return IQK_ERR_GEOMETRY;
    if (out_features <= 0 || out_features % 16) return IQK_ERR_GEOMETRY;
    if (!gemv_rows_ok(num_experts, out_features, pairs)) return IQK_ERR_GEOMETRY;
    if (pairs < 0 || x_rows < 0 || pairs > (1 << 24) || x_rows > (1 << 24))
        return IQK_ERR_GEOMETRY;
    if (!dtype_ok(y_dtype)) return IQK_ERR_ARGUMENT;
    if (pairs == 0) return IQK_OK;
    if (!y || !workspace) return IQK_ERR_ARGUMENT;
    if (!aligned(y, 4) || !aligned(workspace, 256)) return IQK_ERR_ALIGNMENT;
    const int st = check_streams(member, streams);
    if (st != IQK_OK) return st;
    if (workspace_bytes < gemv_layout(member, in_features, x_rows, pairs).total)
        return IQK_ERR_WORKSPACE;
    return cuda_status(launch_gemv_run(member, streams, num_experts, out_features, (int)in_features, x_rows,
                                       pairs, y, y_dtype, workspace,
                                       reinterpret_cast<cudaStream_t>(stream),
                                       num_sms_current()));
}

int iqk_gemv_floor_run(int member, const void *const *streams, int64_t num_experts,
                       int64_t out_features, int64_t in_features, int64_t x_rows, int64_t pairs,
                       void *y, int y_dtype, const void *workspace, size_t workspace_bytes,
                       iqk_stream_t stream) {
    if (!member_ok(member)) return IQK_ERR_MEMBER;
    if (!width_ok(in_features)) return IQK_ERR_WIDTH;
    if (num_experts <= 0 || num_experts > 4096) return IQK_ERR_GEOMETRY;
    if (out_features <= 0 || out_features % 16) return IQK_ERR_GEOMETRY;
    if (!gemv_rows_ok(num_experts, out_features, pairs)) return IQK_ERR_GEOMETRY;
    if (pairs < 0 || x_rows < 0 || pairs > (1 << 24) || x_rows > (1 << 24))
        return IQK_ERR_GEOMETRY;
    if (!dtype_ok(y_dtype)) return IQK_ERR_ARGUMENT;
    if (pairs == 0) return IQK_OK;
    if (!y || !workspace) return IQK_ERR_ARGUMENT;
    if (!aligned(y, 4) || !aligned(workspace, 256)) return IQK_ERR_ALIGNMENT;
    const int st = check_streams(member, streams);
    if (st != IQK_OK) return st;
    if (workspace_bytes < gemv_layout(member, in_features, x_rows, pairs).total)
        return IQK_ERR_WORKSPACE;
    return cuda_status(launch_gemv_run(member, streams, num_experts, out_features,
                                       (int)in_features, x_rows, pairs, y, y_dtype, workspace,
                                       reinterpret_cast<cudaStream_t>(stream),
                                       num_sms_current(), true));
}

int iqk_gemv_glu_run(int member, const void *const *gate_streams,
                     const void *const *up_streams, int64_t num_experts, int64_t out_features,
                     int64_t in_features, int64_t x_rows, int64_t pairs, const float *weight,
                     float *h, const void *workspace, size_t workspace_bytes,
                     iqk_stream_t stream) {
    if (!member_ok(member)) return IQK_ERR_MEMBER;
    if (!width_ok(in_features)) return IQK_ERR_WIDTH;
    if (num_experts <= 0 || num_experts > 4096) return IQK_ERR_GEOMETRY;
    if (out_features <= 0 || out_features % 32) return IQK_ERR_GEOMETRY;
    if (!gemv_rows_ok(num_experts, out_features, pairs)) return IQK_ERR_GEOMETRY;
    if (pairs < 0 || x_rows < 0 || pairs > (1 << 24) || x_rows > (1 << 24))
        return IQK_ERR_GEOMETRY;
    if (pairs == 0) return IQK_OK;
    if (!h || !workspace) return IQK_ERR_ARGUMENT;
    if (!aligned(h, 4) || !aligned(workspace, 256) || (weight && !aligned(weight, 4)))
        return IQK_ERR_ALIGNMENT;
    int st = check_streams(member, gate_streams);
    if (st != IQK_OK) return st;
    st = check_streams(member, up_streams);
    if (st != IQK_OK) return st;
    if (workspace_bytes < gemv_layout(member, in_features, x_rows, pairs).total)
        return IQK_ERR_WORKSPACE;
    return cuda_status(launch_gemv_run(member, gate_streams, num_experts, out_features,
                                       (int)in_features, x_rows, pairs, h, IQK_F32, workspace,
                                       reinterpret_cast<cudaStream_t>(stream), num_sms_current(),
                                       false, up_streams, weight));
}

int iqk_swiglu_rows(const float *gate, const float *up, const float *weight, int64_t rows,
                    int64_t cols, float *h, iqk_stream_t stream) {
    if (rows < 0 || rows > ((int64_t)1 << 31) - 1) return IQK_ERR_GEOMETRY;
    if (cols <= 0 || cols % 4 || cols > (1 << 20)) return IQK_ERR_GEOMETRY;
    if (rows == 0) return IQK_OK;
    if (!gate || !up || !h) return IQK_ERR_ARGUMENT;
    if (!aligned(gate, 16) || !aligned(up, 16) || !aligned(h, 16) || (weight && !aligned(weight, 4)))
        return IQK_ERR_ALIGNMENT;
    return cuda_status(launch_rows_swiglu(gate, up, weight, rows, (int)cols, h,
                                          reinterpret_cast<cudaStream_t>(stream)));
}

int iqk_gemv(int member, const void *x, int x_dtype, int64_t x_rows,
             const void *const *streams, int64_t num_experts, int64_t out_features,
             int64_t in_features, const int32_t *sel, const int32_t *tok, int64_t pairs,
             void *y, int y_dtype, void *workspace, size_t workspace_bytes,
             iqk_stream_t stream) {
    if (!member_ok(member)) return IQK_ERR_MEMBER;
    int st = check_prepare(in_features, num_experts, x_rows, pairs, tok, x_dtype);
    if (st != IQK_OK) return st;
    if (out_features <= 0 || out_features % 16) return IQK_ERR_GEOMETRY;
    if (!gemv_rows_ok(num_experts, out_features, pairs)) return IQK_ERR_GEOMETRY;
    if (!dtype_ok(y_dtype)) return IQK_ERR_ARGUMENT;
    if (pairs == 0) return IQK_OK;
    if (!y || !streams) return IQK_ERR_ARGUMENT;
    st = check_streams(member, streams);
    if (st != IQK_OK) return st;
    st = iqk_gemv_prepare(x, x_dtype, x_rows, in_features, num_experts, sel, tok, pairs,
                          workspace, workspace_bytes, stream);
    if (st != IQK_OK) return st;
    return iqk_gemv_run(member, streams, num_experts, out_features, in_features, x_rows, pairs,
                        y, y_dtype, workspace, workspace_bytes, stream);
}

size_t iqk_grouped_workspace_bytes(int64_t in_features, int64_t num_experts, int64_t pairs) {
    if (!width_ok(in_features) || num_experts <= 0 || pairs < 0) return 0;
    return grouped_layout(in_features, num_experts, pairs).total;
}

int iqk_grouped_prepare(const void *x, int x_dtype, int64_t x_rows, int64_t in_features,
                        int64_t num_experts, const int32_t *sel, const int32_t *tok,
                        int64_t pairs, void *workspace, size_t workspace_bytes,
                        iqk_stream_t stream) {
    int st = check_prepare(in_features, num_experts, x_rows, pairs, tok, x_dtype);
    if (st != IQK_OK) return st;
    if (pairs == 0) return IQK_OK;
    if (!x || !sel || !workspace) return IQK_ERR_ARGUMENT;
    if (!aligned(x, 16) || !aligned(workspace, 256)) return IQK_ERR_ALIGNMENT;
    if (workspace_bytes < grouped_layout(in_features, num_experts, pairs).total)
        return IQK_ERR_WORKSPACE;
    return cuda_status(launch_grouped_prepare(x, x_dtype, x_rows, (int)in_features, num_experts,
                                              sel, tok, pairs, workspace,
                                              reinterpret_cast<cudaStream_t>(stream)));
}

int iqk_grouped_prepare_shard(const void *x, int x_dtype, int64_t x_rows, int64_t in_features,
                              int64_t num_experts, const int32_t *sel, const int32_t *tok,
                              int64_t pairs, void *workspace, size_t workspace_bytes,
                              iqk_stream_t stream) {
    int st = check_prepare(in_features, num_experts, x_rows, pairs, tok, x_dtype);
    if (st != IQK_OK) return st;
    if (pairs == 0) return IQK_OK;
    if (!x || !sel || !workspace) return IQK_ERR_ARGUMENT;
    if (!aligned(x, 16) || !aligned(workspace, 256)) return IQK_ERR_ALIGNMENT;
    if (workspace_bytes < grouped_layout(in_features, num_experts, pairs).total)
        return IQK_ERR_WORKSPACE;
    return cuda_status(launch_grouped_prepare(x, x_dtype, x_rows, (int)in_features, num_experts,
                                              sel, tok, pairs, workspace,
                                              reinterpret_cast<cudaStream_t>(stream), true));
}

int iqk_pairs_swiglu(const float *gate, const float *up, const float *weight, int64_t inter,
                     int64_t in_features, int64_t num_experts, int64_t pairs,
                     const void *workspace, size_t workspace_bytes, void *h,
                     iqk_stream_t stream) {
    if (!width_ok(in_features)) return IQK_ERR_WIDTH;
    if (num_experts <= 0 || num_experts > 4096) return IQK_ERR_GEOMETRY;
    if (inter <= 0 || inter % 16 || inter > (1 << 20)) return IQK_ERR_GEOMETRY;
    if (pairs < 0 || pairs > (1 << 24)) return IQK_ERR_GEOMETRY;
    if (pairs == 0) return IQK_OK;
    if (!gate || !up || !weight || !workspace || !h) return IQK_ERR_ARGUMENT;
    if (!aligned(gate, 16) || !aligned(up, 16) || !aligned(h, 16) || !aligned(weight, 4) ||
        !aligned(workspace, 256))
        return IQK_ERR_ALIGNMENT;
    if (workspace_bytes < grouped_layout(in_features, num_experts, pairs).total)
        return IQK_ERR_WORKSPACE;
    return cuda_status(launch_pairs_swiglu(gate, up, weight, (int)inter, (int)in_features,
                                           num_experts, pairs, workspace, h,
                                           reinterpret_cast<cudaStream_t>(stream)));
}

int iqk_pairs_combine(const float *y, const int32_t *sel, int64_t rows, int top_k,
                      int64_t num_experts, int64_t hidden, void *out, int out_dtype,
                      iqk_stream_t stream) {
    if (rows < 0 || rows > ((int64_t)1 << 31) - 1) return IQK_ERR_GEOMETRY;
    if (top_k <= 0 || top_k > 64 || num_experts <= 0) return IQK_ERR_GEOMETRY;
    if (hidden <= 0 || hidden % 4 || hidden > (1 << 20)) return IQK_ERR_GEOMETRY;
    if (out_dtype != IQK_F32 && out_dtype != IQK_BF16) return IQK_ERR_ARGUMENT;
    if (rows == 0) return IQK_OK;
    if (!y || !sel || !out) return IQK_ERR_ARGUMENT;
    if (!aligned(y, 16) || !aligned(sel, 4) || !aligned(out, 16)) return IQK_ERR_ALIGNMENT;
    return cuda_status(launch_pairs_combine(y, sel, rows, top_k, num_experts, (int)hidden, out,
                                            out_dtype, reinterpret_cast<cudaStream_t>(stream)));
}

int iqk_grouped_run(int member, const void *const *streams, int64_t num_experts,
                    int64_t out_features, int64_t in_features, int64_t pairs, void *y,
                    int y_dtype, const void *workspace, size_t workspace_bytes,
                    iqk_stream_t stream) {
    if (!member_ok(member)) return IQK_ERR_MEMBER;
    if (member == IQK_IQ1_S_R4 && out_features % 4) return IQK_ERR_GEOMETRY;
    if (!width_ok(in_features)) return IQK_ERR_WIDTH;
    if (num_experts <= 0 || num_experts > 4096) return IQK_ERR_GEOMETRY;
    if (out_features <= 0 || out_features % 16) return IQK_ERR_GEOMETRY;
    if (num_experts * out_features > (int64_t)1 << 30) return IQK_ERR_GEOMETRY;
    if (pairs < 0 || pairs > (1 << 24)) return IQK_ERR_GEOMETRY;
    if (!dtype_ok(y_dtype)) return IQK_ERR_ARGUMENT;
    if (pairs == 0) return IQK_OK;
    if (!y || !workspace) return IQK_ERR_ARGUMENT;
    if (!aligned(y, 4) || !aligned(workspace, 256)) return IQK_ERR_ALIGNMENT;
    const int st = check_streams(member, streams);
    if (st != IQK_OK) return st;
    if (workspace_bytes < grouped_layout(in_features, num_experts, pairs).total)
        return IQK_ERR_WORKSPACE;
    return cuda_status(launch_grouped_run(member, streams, num_experts, out_features,
                                          (int)in_features, pairs, y, y_dtype, workspace,
                                          reinterpret_cast<cudaStream_t>(stream),
                                          num_sms_current()));
}

int iqk_grouped_run_range(int member, const void *const *streams, int64_t num_experts,
                          int64_t out_features, int64_t in_features, int64_t pairs,
                          int64_t row_start, int64_t rows, void *y, int y_dtype,
                          const void *workspace, size_t workspace_bytes, iqk_stream_t stream) {
    if (!member_ok(member)) return IQK_ERR_MEMBER;
    if (member == IQK_IQ1_S_R4 && out_features % 4) return IQK_ERR_GEOMETRY;
    if (!width_ok(in_features)) return IQK_ERR_WIDTH;
    if (num_experts <= 0 || num_experts > 4096) return IQK_ERR_GEOMETRY;
    if (out_features <= 0 || out_features % 16) return IQK_ERR_GEOMETRY;
    if (num_experts * out_features > (int64_t)1 << 30) return IQK_ERR_GEOMETRY;
    if (row_start < 0 || rows <= 0 || row_start + rows > out_features) return IQK_ERR_GEOMETRY;
    if (pairs < 0 || pairs > (1 << 24)) return IQK_ERR_GEOMETRY;
    if (!dtype_ok(y_dtype)) return IQK_ERR_ARGUMENT;
    if (pairs == 0) return IQK_OK;
    if (!y || !workspace) return IQK_ERR_ARGUMENT;
    if (!aligned(y, 4) || !aligned(workspace, 256)) return IQK_ERR_ALIGNMENT;
    const int st = check_streams(member, streams);
    if (st != IQK_OK) return st;
    if (workspace_bytes < grouped_layout(in_features, num_experts, pairs).total)
        return IQK_ERR_WORKSPACE;
    return cuda_status(launch_grouped_run(member, streams, num_experts, out_features,
                                          (int)in_features, pairs, y, y_dtype, workspace,
                                          reinterpret_cast<cudaStream_t>(stream),
                                          num_sms_current(), row_start, rows));
}

int iqk_grouped_gemm(int member, const void *x, int x_dtype, int64_t x_rows,
                     const void *const *streams, int64_t num_experts, int64_t out_features,
                     int64_t in_features, const int32_t *sel, const int32_t *tok, int64_t pairs,
                     void *y, int y_dtype, void *workspace, size_t workspace_bytes,
                     iqk_stream_t stream) {
    if (!member_ok(member)) return IQK_ERR_MEMBER;
    if (member == IQK_IQ1_S_R4 && out_features % 4) return IQK_ERR_GEOMETRY;
    int st = check_prepare(in_features, num_experts, x_rows, pairs, tok, x_dtype);
    if (st != IQK_OK) return st;
    if (out_features <= 0 || out_features % 16) return IQK_ERR_GEOMETRY;
    if (!dtype_ok(y_dtype)) return IQK_ERR_ARGUMENT;
    if (pairs == 0) return IQK_OK;
    if (!y || !streams) return IQK_ERR_ARGUMENT;
    st = check_streams(member, streams);
    if (st != IQK_OK) return st;
    st = iqk_grouped_prepare(x, x_dtype, x_rows, in_features, num_experts, sel, tok, pairs,
                             workspace, workspace_bytes, stream);
    if (st != IQK_OK) return st;
    return iqk_grouped_run(member, streams, num_experts, out_features, in_features, pairs, y,
                           y_dtype, workspace, workspace_bytes, stream);
}

int iqk_grouped_read_error(const void *workspace, int32_t *flags, iqk_stream_t stream) {
    if (!workspace || !flags) return IQK_ERR_ARGUMENT;
    *flags = 0;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int32_t hdr0 = 0;
    cudaError_t err = cudaMemcpyAsync(&hdr0, workspace, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err == cudaSuccess) *flags = hdr0;
    return cuda_status(err);
}

int iqk_read_error(const void *workspace, int64_t in_features, int64_t x_rows, int64_t pairs,
                   int32_t *flags, iqk_stream_t stream) {
    if (!workspace || !flags || !width_ok(in_features) || x_rows < 0 || pairs < 0)
        return IQK_ERR_ARGUMENT;
    *flags = 0;
    if (pairs == 0) return IQK_OK;
    const GemvLayout L = gemv_layout(0, in_features, x_rows, pairs);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int32_t hdr0 = 0;
    int32_t *scales = new int32_t[x_rows > 0 ? x_rows : 1];
    const char *w = static_cast<const char *>(workspace);
    cudaError_t err = cudaMemcpyAsync(&hdr0, w + L.hdr, sizeof(int32_t),
                                      cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess && x_rows > 0)
        err = cudaMemcpyAsync(scales, w + L.xscale, sizeof(int32_t) * x_rows,
                              cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err == cudaSuccess) {
        int32_t f = hdr0;
        for (int64_t r = 0; r < x_rows; ++r)
            if (scales[r] == kScaleNonFinite) f |= IQK_DEVERR_NONFINITE;
        *flags = f;
    }
    delete[] scales;
    return cuda_status(err);
}

}  // extern "C"
