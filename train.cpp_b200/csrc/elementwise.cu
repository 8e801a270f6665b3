// elementwise.cu -- the graph ops of mul_mat's composed backward (and the injected-gradient loss)
// for sm_100a: cont, in-place acc, repeat_back, repeat, add/sub/mul/div with broadcast, sum, fill.
//
// Each kernel keeps the reference's per-element arithmetic (one fp32 add/mul/div per element, and
// for repeat_back the reference's summation order), so results are bit-exact with
// src/backends/cpu/trc_cpu_ops.cpp of train.cpp. They are HBM-bound; contiguous cases take a
// vectorised fast path and the transposed copy of the dW gradient goes through a shared-memory
// tile so that both its reads and its writes are coalesced.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "trc_internal.h"

namespace trc {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float ldf(const char* base, int64_t off) {
    return *reinterpret_cast<const float*>(base + off);
}
__device__ __forceinline__ void stf(char* base, int64_t off, float v) { *reinterpret_cast<float*>(base + off) = v; }

// linear index (ne[0] fastest) -> 4-D index
__device__ __forceinline__ void unravel(int64_t i, const int64_t (&ne)[4], int64_t (&idx)[4]) {
    idx[0] = i % ne[0];
    i /= ne[0];
    idx[1] = i % ne[1];
    i /= ne[1];
    idx[2] = i % ne[2];
    idx[3] = i / ne[2];
}

__device__ __forceinline__ int64_t offset_of(const View4& v, const int64_t (&idx)[4]) {
    return idx[0] * v.nb[0] + idx[1] * v.nb[1] + idx[2] * v.nb[2] + idx[3] * v.nb[3];
}

unsigned grid_for(int64_t n, int per_thread = 1) {
    const int64_t want = (n + static_cast<int64_t>(kThreads) * per_thread - 1) / (static_cast<int64_t>(kThreads) * per_thread);
    const int64_t cap  = static_cast<int64_t>(std::max(1, sm_count_current())) * 16;
    return static_cast<unsigned>(std::max<int64_t>(1, std::min(want, cap)));
}

// ------------------------------------------------------------------ cont (compute_dup)
__global__ void cont_generic_kernel(View4 src, View4 dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        int64_t idx[4];
        unravel(i, dst.ne, idx);
        stf(dst.data, offset_of(dst, idx), ldf(src.data, offset_of(src, idx)));
    }
}

// dst contiguous, src with nb[1] == 4 (a transposed plane): 32x32 tiles through shared memory.
__global__ void cont_transpose_kernel(View4 src, View4 dst) {
    __shared__ float tile[32][33];
    const int64_t ne0 = dst.ne[0], ne1 = dst.ne[1];
    const int64_t t0 = (int64_t) blockIdx.x * 32, t1 = (int64_t) blockIdx.y * 32;
    const int64_t plane = blockIdx.z;
    const int64_t p2 = plane % dst.ne[2], p3 = plane / dst.ne[2];
    const char* s = src.data + p2 * src.nb[2] + p3 * src.nb[3];
    char*       d = dst.data + p2 * dst.nb[2] + p3 * dst.nb[3];
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
    // read: consecutive threads walk i1 (unit stride in src)
    for (int r = ty; r < 32; r += 8) {
        const int64_t i0 = t0 + r, i1 = t1 + tx;
        if (i0 < ne0 && i1 < ne1) tile[r][tx] = ldf(s, i0 * src.nb[0] + i1 * src.nb[1]);
    }
    __syncthreads();
    // write: consecutive threads walk i0 (unit stride in dst)
    for (int r = ty; r < 32; r += 8) {
        const int64_t i0 = t0 + tx, i1 = t1 + r;
        if (i0 < ne0 && i1 < ne1) stf(d, i0 * dst.nb[0] + i1 * dst.nb[1], tile[tx][r]);
    }
}

// ------------------------------------------------------------------ acc (inplace)
__global__ void acc_kernel(char* dst, View4 b, int64_t nb1, int64_t nb2, int64_t nb3, int64_t offset, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        int64_t idx[4];
        unravel(i, b.ne, idx);
        const int64_t od = offset + idx[0] * 4 + idx[1] * nb1 + idx[2] * nb2 + idx[3] * nb3;
        stf(dst, od, __fadd_rn(ldf(dst, od), ldf(b.data, offset_of(b, idx))));
    }
}

// contiguous destination region and contiguous b: float4 fast path (the common grad_acc case).
__global__ void acc_contig_kernel(float* dst, const float* b, int64_t n) {
    const int64_t n4 = n / 4;
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n4; i += (int64_t) gridDim.x * blockDim.x) {
        float4       x = reinterpret_cast<const float4*>(dst)[i];
        const float4 y = reinterpret_cast<const float4*>(b)[i];
        x.x = __fadd_rn(x.x, y.x);
        x.y = __fadd_rn(x.y, y.y);
        x.z = __fadd_rn(x.z, y.z);
        x.w = __fadd_rn(x.w, y.w);
        reinterpret_cast<float4*>(dst)[i] = x;
    }
    if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
        const int64_t i = n4 * 4 + threadIdx.x;
        dst[i] = __fadd_rn(dst[i], b[i]);
    }
}

// ------------------------------------------------------------------ repeat_back
// One thread per destination element; the repeated source elements are added in increasing
// linear source index (t3, t2, t1, t0 nested), the order of the reference's scatter loop.
__global__ void repeat_back_kernel(View4 src, View4 dst, int64_t n) {
    const int64_t r0 = src.ne[0] / dst.ne[0], r1 = src.ne[1] / dst.ne[1];
    const int64_t r2 = src.ne[2] / dst.ne[2], r3 = src.ne[3] / dst.ne[3];
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        int64_t j[4];
        unravel(i, dst.ne, j);
        float acc = 0.0f;
        for (int64_t t3 = 0; t3 < r3; ++t3)
            for (int64_t t2 = 0; t2 < r2; ++t2)
                for (int64_t t1 = 0; t1 < r1; ++t1)
                    for (int64_t t0 = 0; t0 < r0; ++t0) {
                        const int64_t off = (j[0] + t0 * dst.ne[0]) * src.nb[0] + (j[1] + t1 * dst.ne[1]) * src.nb[1] +
                                            (j[2] + t2 * dst.ne[2]) * src.nb[2] + (j[3] + t3 * dst.ne[3]) * src.nb[3];
                        acc = __fadd_rn(acc, ldf(src.data, off));
                    }
        stf(dst.data, offset_of(dst, j), acc);
    }
}

// ------------------------------------------------------------------ repeat
__global__ void repeat_kernel(View4 src, View4 dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        int64_t idx[4];
        unravel(i, dst.ne, idx);
        int64_t os = 0;
#pragma unroll
        for (int d = 0; d < 4; ++d) os += (src.ne[d] == 1 ? 0 : idx[d] % src.ne[d]) * src.nb[d];
        stf(dst.data, offset_of(dst, idx), ldf(src.data, os));
    }
}

// ------------------------------------------------------------------ binary
__device__ __forceinline__ float bin_apply(int op, float x, float y) {
    switch (op) {
        case TRC_CUDA_BIN_ADD: return __fadd_rn(x, y);
        case TRC_CUDA_BIN_SUB: return __fsub_rn(x, y);
        case TRC_CUDA_BIN_MUL: return __fmul_rn(x, y);
        default: return __fdiv_rn(x, y);
    }
}

__global__ void binary_kernel(int op, View4 a, View4 b, View4 dst, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        int64_t idx[4];
        unravel(i, dst.ne, idx);
        int64_t ob = 0;
#pragma unroll
        for (int d = 0; d < 4; ++d) ob += (b.ne[d] == 1 ? 0 : idx[d] % b.ne[d]) * b.nb[d];
        stf(dst.data, offset_of(dst, idx), bin_apply(op, ldf(a.data, offset_of(a, idx)), ldf(b.data, ob)));
    }
}

__global__ void binary_contig_kernel(int op, const float* a, const float* b, float* dst, int64_t n) {
    const int64_t n4 = n / 4;
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n4; i += (int64_t) gridDim.x * blockDim.x) {
        const float4 x = reinterpret_cast<const float4*>(a)[i];
        const float4 y = reinterpret_cast<const float4*>(b)[i];
        float4       z;
        z.x = bin_apply(op, x.x, y.x);
        z.y = bin_apply(op, x.y, y.y);
        z.z = bin_apply(op, x.z, y.z);
        z.w = bin_apply(op, x.w, y.w);
        reinterpret_cast<float4*>(dst)[i] = z;
    }
    if (blockIdx.x == 0 && threadIdx.x < (n & 3)) {
        const int64_t i = n4 * 4 + threadIdx.x;
        dst[i] = bin_apply(op, a[i], b[i]);
    }
}

// a (any shape/strides) op scalar b[0] into contiguous dst: the injected-gradient pattern
// mul(repeat(1.0), G) and scalar broadcasts.
// ------------------------------------------------------------------ sum (two passes, double)
constexpr int kSumThreads  = 512;
constexpr int kSumMaxParts = 1024;

__device__ __forceinline__ double block_reduce_double(double v, double* sh) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xFFFFFFFFu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    v = 0.0;
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        v = lane < nw ? sh[lane] : 0.0;
        for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xFFFFFFFFu, v, o);
    }
    return v;
}

// Pass 1: block p sums elements [p*chunk, min((p+1)*chunk, n)) in double.
__global__ void sum_partial_kernel(View4 src, int64_t n, int64_t chunk, bool contig, double* partials) {
    __shared__ double sh[32];
    const int64_t lo = blockIdx.x * chunk, hi = min(n, lo + chunk);
    double v = 0.0;
    if (contig) {
        const float* p = reinterpret_cast<const float*>(src.data);
        for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) v += static_cast<double>(p[i]);
    } else {
        for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
            int64_t idx[4];
            unravel(i, src.ne, idx);
            v += static_cast<double>(ldf(src.data, offset_of(src, idx)));
        }
    }
    v = block_reduce_double(v, sh);
    if (threadIdx.x == 0) partials[blockIdx.x] = v;
}

__global__ void sum_final_kernel(const double* partials, int n_parts, float* dst) {
    __shared__ double sh[32];
    double v = 0.0;
    for (int i = threadIdx.x; i < n_parts; i += blockDim.x) v += partials[i];
    v = block_reduce_double(v, sh);
    if (threadIdx.x == 0) *dst = static_cast<float>(v);
}

int sum_parts_for(int64_t n) {
    const int64_t per = 16384;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(kSumMaxParts, (n + per - 1) / per)));
}

// ------------------------------------------------------------------ fill
__global__ void fill_kernel(float* dst, int64_t n, float value) {
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x)
        dst[i] = value;
}

bool same_shape(const trc_cuda_view& a, const trc_cuda_view& b) {
    return a.ne[0] == b.ne[0] && a.ne[1] == b.ne[1] && a.ne[2] == b.ne[2] && a.ne[3] == b.ne[3];
}

bool aligned16(const void* p) { return (reinterpret_cast<uint64_t>(p) & 15u) == 0; }

}  // namespace

}  // namespace trc

using namespace trc;

extern "C" int trc_cuda_cont(const trc_cuda_view* src, const trc_cuda_view* dst, void* stream) {
    if (!view_ok(src) || !view_ok(dst) || !same_shape(*src, *dst)) return TRC_CUDA_EINVAL;
    const int64_t n = nelements(*dst);
    if (n == 0) return TRC_CUDA_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (view_contiguous(*src) && view_contiguous(*dst)) {
        const cudaError_t e = cudaMemcpyAsync(dst->data, src->data, static_cast<size_t>(n) * 4,
                                              cudaMemcpyDeviceToDevice, s);
        return e == cudaSuccess ? TRC_CUDA_OK : cuda_fail(e);
    }
    const View4 vs = to_view4(*src), vd = to_view4(*dst);
    const int64_t planes = dst->ne[2] * dst->ne[3];
    if (src->nb[1] == 4 && dst->nb[0] == 4 && planes < 65536) {
        const dim3 grid(static_cast<unsigned>((dst->ne[0] + 31) / 32), static_cast<unsigned>((dst->ne[1] + 31) / 32),
                        static_cast<unsigned>(planes));
        if (grid.y < 65536) {
            cont_transpose_kernel<<<grid, 256, 0, s>>>(vs, vd);
            note_launch();
            return check_launch();
        }
    }
    cont_generic_kernel<<<grid_for(n), kThreads, 0, s>>>(vs, vd, n);
    note_launch();
    return check_launch();
}

extern "C" int trc_cuda_acc(void* dst, int64_t dst_bytes, const trc_cuda_view* b, int64_t nb1, int64_t nb2,
                            int64_t nb3, int64_t offset, void* stream) {
    if (dst == nullptr || !view_ok(b) || offset < 0 || nb1 < 0 || nb2 < 0 || nb3 < 0) return TRC_CUDA_EINVAL;
    const int64_t n = nelements(*b);
    if (n == 0) return TRC_CUDA_OK;
    // the constructor's bounds rule (src/core/trc_tensor.cpp:333-340)
    int64_t last = (b->ne[0] - 1) * 4;
    last += b->ne[1] > 1 ? (b->ne[1] - 1) * nb1 : 0;
    last += b->ne[2] > 1 ? (b->ne[2] - 1) * nb2 : 0;
    last += b->ne[3] > 1 ? (b->ne[3] - 1) * nb3 : 0;
    if (offset + last + 4 > dst_bytes) return TRC_CUDA_EINVAL;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool dense = view_contiguous(*b) && (b->ne[1] == 1 || nb1 == b->ne[0] * 4) &&
                       (b->ne[2] == 1 || nb2 == b->ne[0] * b->ne[1] * 4) &&
                       (b->ne[3] == 1 || nb3 == b->ne[0] * b->ne[1] * b->ne[2] * 4);
    char* base = static_cast<char*>(dst);
    if (dense && aligned16(base + offset) && aligned16(b->data)) {
        acc_contig_kernel<<<grid_for(n, 4), kThreads, 0, s>>>(reinterpret_cast<float*>(base + offset),
                                                              static_cast<const float*>(b->data), n);
    } else {
        acc_kernel<<<grid_for(n), kThreads, 0, s>>>(base, to_view4(*b), nb1, nb2, nb3, offset, n);
    }
    note_launch();
    return check_launch();
}

extern "C" int trc_cuda_repeat_back(const trc_cuda_view* src, const trc_cuda_view* dst, void* stream) {
    if (!view_ok(src) || !view_ok(dst)) return TRC_CUDA_EINVAL;
    for (int d = 0; d < 4; ++d) {
        if (dst->ne[d] <= 0 || src->ne[d] % dst->ne[d] != 0) return TRC_CUDA_EINVAL;
    }
    const int64_t n = nelements(*dst);
    if (n == 0) return TRC_CUDA_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    repeat_back_kernel<<<grid_for(n), kThreads, 0, s>>>(to_view4(*src), to_view4(*dst), n);
    note_launch();
    return check_launch();
}

extern "C" int trc_cuda_repeat(const trc_cuda_view* src, const trc_cuda_view* dst, void* stream) {
    if (!view_ok(src) || !view_ok(dst)) return TRC_CUDA_EINVAL;
    for (int d = 0; d < 4; ++d) {
        if (src->ne[d] != 1 && (src->ne[d] == 0 || dst->ne[d] % src->ne[d] != 0)) return TRC_CUDA_EINVAL;
    }
    const int64_t n = nelements(*dst);
    if (n == 0) return TRC_CUDA_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    repeat_kernel<<<grid_for(n), kThreads, 0, s>>>(to_view4(*src), to_view4(*dst), n);
    note_launch();
    return check_launch();
}

extern "C" int trc_cuda_binary(int op, const trc_cuda_view* a, const trc_cuda_view* b, const trc_cuda_view* dst,
                               void* stream) {
    if (op < TRC_CUDA_BIN_ADD || op > TRC_CUDA_BIN_DIV) return TRC_CUDA_EINVAL;
    if (!view_ok(a) || !view_ok(b) || !view_ok(dst) || !same_shape(*a, *dst)) return TRC_CUDA_EINVAL;
    for (int d = 0; d < 4; ++d) {
        if (b->ne[d] != 1 && b->ne[d] != a->ne[d]) return TRC_CUDA_EINVAL;  // ggml_can_repeat(b, a)
    }
    const int64_t n = nelements(*dst);
    if (n == 0) return TRC_CUDA_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (same_shape(*a, *b) && view_contiguous(*a) && view_contiguous(*b) && view_contiguous(*dst) &&
        aligned16(a->data) && aligned16(b->data) && aligned16(dst->data)) {
        binary_contig_kernel<<<grid_for(n, 4), kThreads, 0, s>>>(op, static_cast<const float*>(a->data),
                                                                 static_cast<const float*>(b->data),
                                                                 static_cast<float*>(dst->data), n);
    } else {
        binary_kernel<<<grid_for(n), kThreads, 0, s>>>(op, to_view4(*a), to_view4(*b), to_view4(*dst), n);
    }
    note_launch();
    return check_launch();
}

extern "C" size_t trc_cuda_sum_workspace_bytes(int64_t n) {
    return static_cast<size_t>(sum_parts_for(n < 0 ? 0 : n)) * sizeof(double);
}

extern "C" int trc_cuda_sum(const trc_cuda_view* src, float* dst, void* workspace, size_t workspace_bytes,
                            void* stream) {
    if (!view_ok(src) || dst == nullptr) return TRC_CUDA_EINVAL;
    const int64_t n     = nelements(*src);
    const int     parts = sum_parts_for(n);
    if (workspace == nullptr || workspace_bytes < static_cast<size_t>(parts) * sizeof(double) ||
        (reinterpret_cast<uint64_t>(workspace) & 7u) != 0)
        return TRC_CUDA_EINVAL;
    cudaStream_t s     = static_cast<cudaStream_t>(stream);
    const int64_t chunk = n == 0 ? 1 : (n + parts - 1) / parts;
    double* partials    = static_cast<double*>(workspace);
    sum_partial_kernel<<<parts, kSumThreads, 0, s>>>(to_view4(*src), n, chunk, view_contiguous(*src), partials);
    note_launch();
    int st = check_launch();
    if (st != TRC_CUDA_OK) return st;
    sum_final_kernel<<<1, kSumThreads, 0, s>>>(partials, parts, dst);
    note_launch();
    return check_launch();
}

extern "C" int trc_cuda_fill(float* dst, int64_t n, float value, void* stream) {
    if (n < 0 || (n > 0 && dst == nullptr)) return TRC_CUDA_EINVAL;
    if (n == 0) return TRC_CUDA_OK;
    fill_kernel<<<grid_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(dst, n, value);
    note_launch();
    return check_launch();
}
