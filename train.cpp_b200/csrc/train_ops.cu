// train_ops.cu -- the graph ops a Linear training step needs on the device besides mul_mat and its
// backward: element-wise unaries of a loss (sqr, sqrt, abs, neg, sgn, step, scale), row sums and
// means, and the optimizer graph train.cpp builds for a device-resident model (opt_step_adamw,
// opt_step_sgd, and the grad-norm clip pair sum_sqr_acc / clip_scale_inplace).
//
// Every element-wise result is bit-exact with train.cpp's CPU backend
// (src/backends/cpu/trc_cpu_ops.cpp): each fp32 operation is one explicitly rounded op in the
// reference's order (no contraction into fused multiply-adds, which the reference's x86 build
// does not do either). Row sums keep the reference's sequential double accumulation per row.
// sum_sqr_acc adds Σ x² over a whole tensor in double like the reference, but in a parallel order;
// after the final conversion to float it matches the sequential sum except when the two double
// sums round to different floats.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "trc_internal.h"
#include "trc_ptx.cuh"

namespace trc {

namespace {

constexpr int kThreads = 256;

unsigned grid_for(int64_t n) {
    const int64_t want = (n + kThreads - 1) / kThreads;
    const int64_t cap  = static_cast<int64_t>(std::max(1, sm_count_current())) * 16;
    return static_cast<unsigned>(std::max<int64_t>(1, std::min(want, cap)));
}

__device__ __forceinline__ int64_t view_offset(const View4& v, int64_t i) {
    const int64_t i0 = i % v.ne[0];
    i /= v.ne[0];
    const int64_t i1 = i % v.ne[1];
    i /= v.ne[1];
    const int64_t i2 = i % v.ne[2];
    const int64_t i3 = i / v.ne[2];
    return i0 * v.nb[0] + i1 * v.nb[1] + i2 * v.nb[2] + i3 * v.nb[3];
}

// ------------------------------------------------------------------ unary (compute_unary, compute_scale)
// fn_sqr / fn_sqrt / fn_abs / fn_neg / fn_sgn / fn_step (trc_cpu_ops.cpp:84-94) and compute_scale
// (:139-149), over any strides, element i of src to element i of dst in ggml linear order.
__device__ __forceinline__ float unary_value(int op, float x, float s) {
    switch (op) {
        case TRC_CUDA_UNARY_SQR: return __fmul_rn(x, x);
        case TRC_CUDA_UNARY_SQRT: return __fsqrt_rn(x);
        case TRC_CUDA_UNARY_ABS: return fabsf(x);
        case TRC_CUDA_UNARY_NEG: return -x;
        case TRC_CUDA_UNARY_SGN: return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f);
        case TRC_CUDA_UNARY_STEP: return x > 0.0f ? 1.0f : 0.0f;
        default: return __fmul_rn(x, s);  // TRC_CUDA_UNARY_SCALE
    }
}

__global__ void unary_kernel(int op, View4 src, View4 dst, float s, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        const float x = *reinterpret_cast<const float*>(src.data + view_offset(src, i));
        *reinterpret_cast<float*>(dst.data + view_offset(dst, i)) = unary_value(op, x, s);
    }
}

__global__ void unary_contig_kernel(int op, const float* src, float* dst, float s, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x)
        dst[i] = unary_value(op, src[i], s);
}

// ------------------------------------------------------------------ sum_rows / mean (compute_sum_rows_or_mean)
// One thread per row: the reference's sequential double sum over i0 (row_sum_f32,
// trc_cpu_ops.cpp:284-300), then (float) sum or (float) (sum / ne0) (:317-333).
__global__ void sum_rows_kernel(View4 src, View4 dst, int take_mean, int64_t rows) {
    for (int64_t r = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; r < rows; r += (int64_t) gridDim.x * blockDim.x) {
        const int64_t i1 = r % src.ne[1], i2 = (r / src.ne[1]) % src.ne[2], i3 = r / (src.ne[1] * src.ne[2]);
        const char* row = src.data + i1 * src.nb[1] + i2 * src.nb[2] + i3 * src.nb[3];
        double sum = 0.0;
        for (int64_t i0 = 0; i0 < src.ne[0]; ++i0)
            sum = __dadd_rn(sum, static_cast<double>(*reinterpret_cast<const float*>(row + i0 * src.nb[0])));
        const float v = take_mean ? __double2float_rn(__ddiv_rn(sum, static_cast<double>(src.ne[0])))
                                  : __double2float_rn(sum);
        *reinterpret_cast<float*>(dst.data + i1 * dst.nb[1] + i2 * dst.nb[2] + i3 * dst.nb[3]) = v;
    }
}

// ------------------------------------------------------------------ optimizer steps
// compute_opt_step_adamw (trc_cpu_ops.cpp:1506-1538): per element
//   m += (g - m) * (1 - beta1);  v = v * beta2 + g * g * (1 - beta2);
//   p = p * decay - step_sz * (m / (sqrt(v) / bc2_sqrt + eps))
struct AdamwArgs {
    float step_sz, bc2_sqrt, decay, beta1, beta2, eps;
};

__global__ void adamw_kernel(float* p, const float* g, float* m, float* v, int64_t n, AdamwArgs a) {
    const float one_b1 = __fsub_rn(1.0f, a.beta1), one_b2 = __fsub_rn(1.0f, a.beta2);
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        const float gi = g[i];
        const float mi = __fadd_rn(m[i], __fmul_rn(__fsub_rn(gi, m[i]), one_b1));
        const float vi = __fadd_rn(__fmul_rn(v[i], a.beta2), __fmul_rn(__fmul_rn(gi, gi), one_b2));
        m[i] = mi;
        v[i] = vi;
        const float pv    = __fmul_rn(p[i], a.decay);
        const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(vi), a.bc2_sqrt), a.eps);
        p[i] = __fsub_rn(pv, __fmul_rn(a.step_sz, __fdiv_rn(mi, denom)));
    }
}

// compute_opt_step_sgd (trc_cpu_ops.cpp:1540-1573): d = g + wd * p; with momentum, mom = d on the
// first step, else momentum * mom + (1 - dampening) * d, and d = nesterov ? d + momentum * mom : mom;
// p -= lr * d.
struct SgdArgs {
    float lr, momentum, dampening, weight_decay, nesterov, is_first;
};

__global__ void sgd_kernel(float* p, const float* g, float* mom, int64_t n, SgdArgs a) {
    const float one_damp = __fsub_rn(1.0f, a.dampening);
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        float d = __fadd_rn(g[i], __fmul_rn(a.weight_decay, p[i]));
        if (a.momentum != 0.0f) {
            float mi;
            if (a.is_first != 0.0f) mi = d;
            else mi = __fadd_rn(__fmul_rn(a.momentum, mom[i]), __fmul_rn(one_damp, d));
            mom[i] = mi;
            d = a.nesterov != 0.0f ? __fadd_rn(d, __fmul_rn(a.momentum, mi)) : mi;
        }
        p[i] = __fsub_rn(p[i], __fmul_rn(a.lr, d));
    }
}

// ------------------------------------------------------------------ grad-norm clip
// compute_sum_sqr_acc (trc_cpu_ops.cpp:1578-1591): acc[0] += (float) Σ (double) x * (double) x.
// Each square is exact in double; the partial sums go to the caller's workspace.
__device__ double block_sum_double(double v) {
    __shared__ double sh[32];
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = v;
    __syncthreads();
    v = threadIdx.x < (blockDim.x >> 5) ? sh[threadIdx.x] : 0.0;
    if (threadIdx.x < 32)
        for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    return v;
}

__global__ void sum_sqr_partial_kernel(const float* a, int64_t n, int64_t chunk, double* partials) {
    const int64_t lo = blockIdx.x * chunk, hi = min(n, lo + chunk);
    double s = 0.0;
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const double x = static_cast<double>(a[i]);
        s = __dadd_rn(s, __dmul_rn(x, x));
    }
    s = block_sum_double(s);
    if (threadIdx.x == 0) partials[blockIdx.x] = s;
}

__global__ void sum_sqr_final_kernel(const double* partials, int n_parts, float* acc) {
    double s = 0.0;
    for (int i = threadIdx.x; i < n_parts; i += blockDim.x) s = __dadd_rn(s, partials[i]);
    s = block_sum_double(s);
    if (threadIdx.x == 0) acc[0] = __fadd_rn(acc[0], __double2float_rn(s));
}

// compute_clip_scale_inplace (trc_cpu_ops.cpp:1594-1611): a *= min(1, max_norm / (sqrt(norm) + eps)).
__global__ void clip_scale_kernel(float* a, int64_t n, const float* norm, float max_norm, float eps) {
    float scale = __fdiv_rn(max_norm, __fadd_rn(__fsqrt_rn(norm[0]), eps));
    if (scale > 1.0f) scale = 1.0f;
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x)
        a[i] = __fmul_rn(a[i], scale);
}

constexpr int kSqrMaxParts = 4096;

int sqr_parts_for(int64_t n) {
    const int64_t per = 16384;
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(kSqrMaxParts, (n + per - 1) / per)));
}

bool contiguous(const trc_cuda_view& v) {
    int64_t expect = 4;
    for (int i = 0; i < 4; ++i) {
        if (v.ne[i] > 1 && v.nb[i] != expect) return false;
        expect *= v.ne[i];
    }
    return true;
}

}  // namespace

}  // namespace trc

using namespace trc;

extern "C" {

int trc_cuda_unary(int op, const trc_cuda_view* src, const trc_cuda_view* dst, float param, void* stream) {
    if (op < TRC_CUDA_UNARY_SQR || op > TRC_CUDA_UNARY_SCALE) return TRC_CUDA_EUNSUPPORTED;
    if (!view_ok(src) || !view_ok(dst)) return TRC_CUDA_EINVAL;
    for (int i = 0; i < 4; ++i)
        if (src->ne[i] != dst->ne[i]) return TRC_CUDA_EINVAL;
    const int64_t n = nelements(*dst);
    if (n == 0) return TRC_CUDA_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (contiguous(*src) && contiguous(*dst))
        unary_contig_kernel<<<grid_for(n), kThreads, 0, s>>>(op, static_cast<const float*>(src->data),
                                                              static_cast<float*>(dst->data), param, n);
    else
        unary_kernel<<<grid_for(n), kThreads, 0, s>>>(op, to_view4(*src), to_view4(*dst), param, n);
    note_launch();
    return check_launch();
}

int trc_cuda_sum_rows(const trc_cuda_view* src, const trc_cuda_view* dst, int take_mean, void* stream) {
    if (!view_ok(src) || !view_ok(dst)) return TRC_CUDA_EINVAL;
    if (dst->ne[0] != 1 || dst->ne[1] != src->ne[1] || dst->ne[2] != src->ne[2] || dst->ne[3] != src->ne[3])
        return TRC_CUDA_EINVAL;
    const int64_t rows = src->ne[1] * src->ne[2] * src->ne[3];
    if (rows == 0) return TRC_CUDA_OK;
    if (take_mean && src->ne[0] == 0) return TRC_CUDA_EINVAL;
    sum_rows_kernel<<<grid_for(rows), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        to_view4(*src), to_view4(*dst), take_mean ? 1 : 0, rows);
    note_launch();
    return check_launch();
}

int trc_cuda_opt_step_adamw(float* param, const float* grad, float* m, float* v, int64_t n, const float* params6,
                            void* stream) {
    if (n < 0 || params6 == nullptr) return TRC_CUDA_EINVAL;
    if (n == 0) return TRC_CUDA_OK;
    if (param == nullptr || grad == nullptr || m == nullptr || v == nullptr) return TRC_CUDA_EINVAL;
    const AdamwArgs a{params6[0], params6[1], params6[2], params6[3], params6[4], params6[5]};
    adamw_kernel<<<grid_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(param, grad, m, v, n, a);
    note_launch();
    return check_launch();
}

int trc_cuda_opt_step_sgd(float* param, const float* grad, float* momentum, int64_t n, const float* params6,
                          void* stream) {
    if (n < 0 || params6 == nullptr) return TRC_CUDA_EINVAL;
    if (n == 0) return TRC_CUDA_OK;
    if (param == nullptr || grad == nullptr || (momentum == nullptr && params6[1] != 0.0f)) return TRC_CUDA_EINVAL;
    const SgdArgs a{params6[0], params6[1], params6[2], params6[3], params6[4], params6[5]};
    sgd_kernel<<<grid_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(param, grad, momentum, n, a);
    note_launch();
    return check_launch();
}

size_t trc_cuda_sum_sqr_workspace_bytes(int64_t n) {
    return static_cast<size_t>(sqr_parts_for(std::max<int64_t>(n, 1))) * sizeof(double);
}

int trc_cuda_sum_sqr_acc(float* acc, const float* a, int64_t n, void* workspace, size_t workspace_bytes,
                         void* stream) {
    if (acc == nullptr || n < 0 || (n > 0 && a == nullptr)) return TRC_CUDA_EINVAL;
    if (n == 0) return TRC_CUDA_OK;  // acc += 0.0f leaves every value unchanged
    const int parts = sqr_parts_for(n);
    if (workspace == nullptr || workspace_bytes < static_cast<size_t>(parts) * sizeof(double)) return TRC_CUDA_EINVAL;
    const int64_t chunk = (n + parts - 1) / parts;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    double* partials = static_cast<double*>(workspace);
    sum_sqr_partial_kernel<<<parts, kThreads, 0, s>>>(a, n, chunk, partials);
    sum_sqr_final_kernel<<<1, kThreads, 0, s>>>(partials, parts, acc);
    note_launch(2);
    return check_launch();
}

int trc_cuda_clip_scale_inplace(float* a, int64_t n, const float* norm, float max_norm, float eps, void* stream) {
    if (n < 0 || norm == nullptr || (n > 0 && a == nullptr)) return TRC_CUDA_EINVAL;
    if (n == 0) return TRC_CUDA_OK;
    clip_scale_kernel<<<grid_for(n), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(a, n, norm, max_norm, eps);
    note_launch();
    return check_launch();
}

}  // extern "C"

// ------------------------------------------------------------------ measurement support
namespace trc {
namespace {

// The dequant kernel's traffic shape without its arithmetic: every warp reads 512 contiguous bytes
// and writes `ratio` x 512 contiguous bytes with 16-byte streaming stores.
template <int R>
__global__ void stream_probe_kernel(const uint4* in, uint4* out, int64_t n_in16) {
    const int lane = threadIdx.x & 31;
    const int64_t wstep = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    for (int64_t w = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) >> 5; (w + 1) * 32 <= n_in16;
         w += wstep) {
        uint4 v = __ldcs(in + w * 32 + lane);
#pragma unroll
        for (int j = 0; j < R; ++j) {
            v.x += 1u;
            __stcs(out + (w * 32) * R + j * 32 + lane, v);
        }
    }
}

// The same traffic and output layout with the writes staged in shared memory and written by bulk
// copies, the dequant kernel's store path: each CTA reads 256 x 16 bytes, places its R copies in one
// of two shared buffers and stores the buffer with one cp.async.bulk while it fills the other.
template <int R>
__global__ void __launch_bounds__(256) stream_probe_bulk_kernel(const uint4* in, uint4* out, int64_t n_in16) {
    extern __shared__ __align__(128) uint4 sbuf[];  // 2 x R x 256
    const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
    const int64_t chunks = n_in16 / 256;
    int b = 0;
    for (int64_t c = blockIdx.x; c < chunks; c += gridDim.x, b ^= 1) {
        uint4* buf = sbuf + b * R * 256;
        uint4 v = __ldcs(in + c * 256 + threadIdx.x);
#pragma unroll
        for (int j = 0; j < R; ++j) {
            v.x += 1u;
            buf[wp * 32 * R + j * 32 + lane] = v;
        }
        fence_proxy_async_smem();
        __syncthreads();
        if (threadIdx.x == 0) {
            bulk_store(out + c * 256 * R, smem_u32(buf), static_cast<uint32_t>(R * 256 * 16));
            bulk_commit_group();
            bulk_wait_group_read<1>();  // the other buffer's copy has been read: it may be refilled
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) bulk_wait_group_all();
}

template <int R>
int launch_probe_bulk(const uint4* in, uint4* out, int64_t n_in16, cudaStream_t s) {
    const int smem = 2 * R * 256 * 16;
    static bool configured[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TRC_CUDA_ECUDA;
    if (!configured[dev]) {
        const cudaError_t e =
            cudaFuncSetAttribute(stream_probe_bulk_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_fail(e);
        configured[dev] = true;
    }
    const int sms = std::max(1, sm_count_current());
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(n_in16 / 256, int64_t(sms) * 3));
    stream_probe_bulk_kernel<R><<<grid, 256, smem, s>>>(in, out, n_in16);
    note_launch();
    return check_launch();
}

}  // namespace
}  // namespace trc

extern "C" int trc_cuda_stream_probe_bulk(const void* in, void* out, int64_t n_in16, int ratio, void* stream) {
    using namespace trc;
    if (in == nullptr || out == nullptr || n_in16 <= 0 || (n_in16 % 256) != 0 || ratio < 1 || ratio > 8)
        return TRC_CUDA_EINVAL;
    if ((reinterpret_cast<uint64_t>(in) & 15u) != 0 || (reinterpret_cast<uint64_t>(out) & 15u) != 0) return TRC_CUDA_EINVAL;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint4* pi = static_cast<const uint4*>(in);
    uint4* po = static_cast<uint4*>(out);
    switch (ratio) {
        case 1: return launch_probe_bulk<1>(pi, po, n_in16, s);
        case 2: return launch_probe_bulk<2>(pi, po, n_in16, s);
        case 3: return launch_probe_bulk<3>(pi, po, n_in16, s);
        case 4: return launch_probe_bulk<4>(pi, po, n_in16, s);
        case 5: return launch_probe_bulk<5>(pi, po, n_in16, s);
        case 6: return launch_probe_bulk<6>(pi, po, n_in16, s);
        case 7: return launch_probe_bulk<7>(pi, po, n_in16, s);
        default: return launch_probe_bulk<8>(pi, po, n_in16, s);
    }
}

extern "C" int trc_cuda_stream_probe(const void* in, void* out, int64_t n_in16, int ratio, void* stream) {
    using namespace trc;
    if (in == nullptr || out == nullptr || n_in16 <= 0 || (n_in16 % 32) != 0 || ratio < 1 || ratio > 8)
        return TRC_CUDA_EINVAL;
    if ((reinterpret_cast<uint64_t>(in) & 15u) != 0 || (reinterpret_cast<uint64_t>(out) & 15u) != 0) return TRC_CUDA_EINVAL;
    const int sms = std::max(1, sm_count_current());
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(n_in16 / 32 * 32 / 256 + 1, int64_t(sms) * 16));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const uint4* pi = static_cast<const uint4*>(in);
    uint4* po = static_cast<uint4*>(out);
    switch (ratio) {
        case 1: stream_probe_kernel<1><<<grid, 256, 0, s>>>(pi, po, n_in16); break;
        case 2: stream_probe_kernel<2><<<grid, 256, 0, s>>>(pi, po, n_in16); break;
        case 3: stream_probe_kernel<3><<<grid, 256, 0, s>>>(pi, po, n_in16); break;
        case 4: stream_probe_kernel<4><<<grid, 256, 0, s>>>(pi, po, n_in16); break;
        case 5: stream_probe_kernel<5><<<grid, 256, 0, s>>>(pi, po, n_in16); break;
        case 6: stream_probe_kernel<6><<<grid, 256, 0, s>>>(pi, po, n_in16); break;
        case 7: stream_probe_kernel<7><<<grid, 256, 0, s>>>(pi, po, n_in16); break;
        default: stream_probe_kernel<8><<<grid, 256, 0, s>>>(pi, po, n_in16); break;
    }
    note_launch();
    return check_launch();
}
