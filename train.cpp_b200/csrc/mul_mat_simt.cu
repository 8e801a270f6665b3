// mul_mat_simt.cu -- fp32 SIMT mul_mat for views the TMA-fed tensor-core kernel cannot address
// (byte strides that are not multiples of 16, e.g. K = 5 or 33 rows of the conformance tests, or
// an operand contiguous along neither K nor M/N).
//
// Every output element is a separately rounded multiply-then-add chain over k = 0..K-1 in
// ascending order starting from +0.0f -- the exact arithmetic of compute_mul_mat
// (src/backends/cpu/trc_cpu_ops.cpp:182-216 of train.cpp) -- so this kernel is bit-identical to
// the reference for any shape and stride, including ne[2]/ne[3] modulo broadcasting of a.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "trc_internal.h"

namespace trc {

namespace {

constexpr int kTM = 64, kTN = 64, kTK = 16;

// d has d.ne[2] x d.ne[3] planes; output plane (q2, q3) receives, in order r3 = 0.., r2 = 0..,
// the rounded product of source plane (q2 + r2 d.ne2, q3 + r3 d.ne3) added onto a running total
// that starts at 0 -- mul_mat followed by repeat_back, with the reference's rounding and order.
__global__ void __launch_bounds__(256) mm_simt_kernel(View4 a, View4 b, View4 d, int accumulate, int64_t plane0) {
    __shared__ float As[kTK][kTM + 1];
    __shared__ float Bs[kTK][kTN + 1];
    const int64_t K = a.ne[0], M = a.ne[1], N = b.ne[1];
    const int64_t plane = plane0 + blockIdx.z;
    const int64_t q2 = plane % d.ne[2], q3 = plane / d.ne[2];
    const int64_t red2 = b.ne[2] / d.ne[2], red3 = b.ne[3] / d.ne[3];
    char*       pd = d.data + q2 * d.nb[2] + q3 * d.nb[3];
    const int64_t i0 = (int64_t) blockIdx.x * kTM, j0 = (int64_t) blockIdx.y * kTN;
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;

    float total[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) total[r][c] = 0.0f;
    for (int64_t rr = 0; rr < red2 * red3; ++rr) {
        const int64_t p2 = q2 + d.ne[2] * (rr % red2), p3 = q3 + d.ne[3] * (rr / red2);
        const char* pa = a.data + (p2 % a.ne[2]) * a.nb[2] + (p3 % a.ne[3]) * a.nb[3];
        const char* pb = b.data + p2 * b.nb[2] + p3 * b.nb[3];
        float acc[4][4];
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[r][c] = 0.0f;

        for (int64_t k0 = 0; k0 < K; k0 += kTK) {
            for (int e = threadIdx.x; e < kTK * kTM; e += 256) {
                const int kk = e / kTM, ii = e % kTM;
                const int64_t k = k0 + kk, i = i0 + ii;
                As[kk][ii] = (k < K && i < M) ? *reinterpret_cast<const float*>(pa + k * a.nb[0] + i * a.nb[1]) : 0.0f;
            }
            for (int e = threadIdx.x; e < kTK * kTN; e += 256) {
                const int kk = e / kTN, jj = e % kTN;
                const int64_t k = k0 + kk, j = j0 + jj;
                Bs[kk][jj] = (k < K && j < N) ? *reinterpret_cast<const float*>(pb + k * b.nb[0] + j * b.nb[1]) : 0.0f;
            }
            __syncthreads();
            const int kmax = static_cast<int>(min(static_cast<int64_t>(kTK), K - k0));
            for (int kk = 0; kk < kmax; ++kk) {
                float av[4], bv[4];
#pragma unroll
                for (int r = 0; r < 4; ++r) av[r] = As[kk][ty * 4 + r];
#pragma unroll
                for (int c = 0; c < 4; ++c) bv[c] = Bs[kk][tx * 4 + c];
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int c = 0; c < 4; ++c) acc[r][c] = __fadd_rn(acc[r][c], __fmul_rn(av[r], bv[c]));
            }
            __syncthreads();
        }
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) total[r][c] = red2 * red3 == 1 ? acc[r][c] : __fadd_rn(total[r][c], acc[r][c]);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const int64_t i = i0 + ty * 4 + r;
        if (i >= M) continue;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int64_t j = j0 + tx * 4 + c;
            if (j >= N) continue;
            float* o = reinterpret_cast<float*>(pd + i * d.nb[0] + j * d.nb[1]);
            *o = accumulate ? __fadd_rn(*o, total[r][c]) : total[r][c];
        }
    }
}

}  // namespace

int mul_mat_simt(const trc_cuda_view& a, const trc_cuda_view& b, const trc_cuda_view& d, bool accumulate,
                 cudaStream_t stream) {
    const int64_t M = a.ne[1], N = b.ne[1];
    const int64_t planes = d.ne[2] * d.ne[3];  // output planes (fewer than b's when repeat_back is fused)
    const int64_t gx = (M + kTM - 1) / kTM, gy = (N + kTN - 1) / kTN;
    if (gx >= (1ll << 31) || gy >= 65536) return TRC_CUDA_EUNSUPPORTED;
    for (int64_t p0 = 0; p0 < planes; p0 += 65535) {
        const unsigned gz = static_cast<unsigned>(std::min<int64_t>(65535, planes - p0));
        mm_simt_kernel<<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy), gz), 256, 0, stream>>>(
            to_view4(a), to_view4(b), to_view4(d), accumulate ? 1 : 0, p0);
        note_launch();
        const int st = check_launch();
        if (st != TRC_CUDA_OK) return st;
    }
    return TRC_CUDA_OK;
}

}  // namespace trc
