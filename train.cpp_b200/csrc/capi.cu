// capi.cu -- extern "C" entry points of libtrc_cuda.so that are not kernels themselves: status
// reporting, the device error word, argument checks that mirror the reference's shape rules, and
// dispatch between the tensor-core and SIMT mul_mat kernels.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <mutex>

#include "trc_internal.h"
#include "trc_ptx.cuh"

namespace trc {

__device__ int g_device_error = 0;

namespace {
std::atomic<uint64_t> g_launches{0};
thread_local int      g_last_cuda_error = 0;
}  // namespace

void note_launch(int n) { g_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed); }

// One CTA waits, with the library's bounded wait, on an mbarrier no thread ever arrives on: the
// wait runs out after limit_ns, records TRC_DEVERR_SELFTEST and the kernel returns normally.
__global__ void selftest_wait_kernel(uint64_t limit_ns, int* out) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) out[0] = mbar_wait_limit(&bar, 0, TRC_DEVERR_SELFTEST, limit_ns) ? 1 : 0;
}

int cuda_fail(cudaError_t e) {
    g_last_cuda_error = static_cast<int>(e);
    return TRC_CUDA_ECUDA;
}

int check_launch() {
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TRC_CUDA_OK : cuda_fail(e);
}

int sm_count_current() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return -1;
    static int cache[64] = {0};
    if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    if (dev >= 0 && dev < 64) cache[dev] = n;
    return n;
}

namespace {

// The copy stream and the two events of the chunked host upload, one set per device, created on
// first use (and kept for the process).
struct UploadCtx {
    std::mutex   mu;
    cudaStream_t copy    = nullptr;
    cudaEvent_t  start   = nullptr;  // recorded on the caller's stream: staging is free from here
    cudaEvent_t  landed  = nullptr;  // recorded on the copy stream after each chunk
    bool         ready   = false;
};
UploadCtx g_upload[64];

// From this many columns of b on, trc_cuda_mul_mat_q dequantizes W into scratch and runs the F32
// kernel: the dequant pass costs about 88 / N of the GEMM, while the fused kernel's in-loop decode
// costs it 12-20 % at N = 2048 on B200.
constexpr int64_t kTwoStepMinColumns = 1024;

// A pipelined upload: chunks of up to kUploadChunkBytes of packed bytes, then two short chunks of
// about kUploadTail1 and kUploadTail2, so that only a small dequant is left exposed; uploads of
// kPipelineMinBytes or more are pipelined. Measured on B200 (five 4096 x 11008 tensors per step,
// share of a plain pinned copy of the same bytes): chunks of 4 / 8 / 16 / 32 MB reach 0.92 / 0.94 /
// 0.95 / 0.955 (every chunk costs its own copy and event round trip); one chunk for the whole
// front 0.957, but then a large tensor's whole dequant would be exposed.
constexpr size_t kUploadChunkBytes = size_t(32) << 20;
constexpr size_t kUploadTail1      = size_t(2) << 20;
constexpr size_t kUploadTail2      = size_t(1) << 20;
constexpr size_t kPipelineMinBytes = size_t(16) << 20;
constexpr int64_t kRunBlocks       = 256;  // chunks start on whole runs of the dequant kernel

}  // namespace

// trc_cuda_load_quant with the host copy cut into chunks on a second stream: chunk c + 1 crosses
// PCIe while the caller's stream dequantizes chunk c, so the upload of a large tensor costs its
// copy time plus one chunk's dequant instead of copy + dequant. The first copy waits for the
// caller's earlier work (the staging buffer may still be read by a previous dequant), and every
// dequant waits for its own chunk.
int load_quant_pipelined(int type, const uint8_t* host, int64_t n_blocks, uint8_t* staging, float* out,
                         cudaStream_t s) {
    const size_t bb = trc_cuda_block_bytes(type);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    if (dev < 0 || dev >= 64) return TRC_CUDA_EUNSUPPORTED;
    UploadCtx& u = g_upload[dev];
    std::lock_guard<std::mutex> lock(u.mu);
    if (!u.ready) {
        if ((e = cudaStreamCreateWithFlags(&u.copy, cudaStreamNonBlocking)) != cudaSuccess) return cuda_fail(e);
        if ((e = cudaEventCreateWithFlags(&u.start, cudaEventDisableTiming)) != cudaSuccess) return cuda_fail(e);
        if ((e = cudaEventCreateWithFlags(&u.landed, cudaEventDisableTiming)) != cudaSuccess) return cuda_fail(e);
        u.ready = true;
    }
    // Front chunks of up to kUploadChunkBytes, then the two tail chunks: only the last chunk's
    // dequant runs with no copy beside it, so it is kept small. Every chunk starts on a whole run
    // (the last one ends with the tensor's ragged end).
    const auto blocks_of = [&](size_t bytes) {
        return std::max<int64_t>(kRunBlocks, static_cast<int64_t>(bytes / bb) / kRunBlocks * kRunBlocks);
    };
    const int64_t tail1 = blocks_of(kUploadTail1);
    const int64_t front = (n_blocks - tail1 - blocks_of(kUploadTail2)) / kRunBlocks * kRunBlocks;
    const int64_t n_front = (front + blocks_of(kUploadChunkBytes) - 1) / blocks_of(kUploadChunkBytes);
    int64_t chunk = (front + n_front - 1) / n_front;
    chunk = (chunk + kRunBlocks - 1) / kRunBlocks * kRunBlocks;
    if ((e = cudaEventRecord(u.start, s)) != cudaSuccess) return cuda_fail(e);
    if ((e = cudaStreamWaitEvent(u.copy, u.start, 0)) != cudaSuccess) return cuda_fail(e);
    for (int64_t b0 = 0; b0 < n_blocks;) {
        const int64_t nb = b0 < front ? std::min(chunk, front - b0) : b0 == front ? tail1 : n_blocks - b0;
        const size_t off = static_cast<size_t>(b0) * bb;
        e = cudaMemcpyAsync(staging + off, host + off, static_cast<size_t>(nb) * bb, cudaMemcpyHostToDevice, u.copy);
        if (e != cudaSuccess) return cuda_fail(e);
        if ((e = cudaEventRecord(u.landed, u.copy)) != cudaSuccess) return cuda_fail(e);
        if ((e = cudaStreamWaitEvent(s, u.landed, 0)) != cudaSuccess) return cuda_fail(e);
        const int st = trc_cuda_dequant(type, staging + off, nb, out + b0 * 32, s);
        if (st != TRC_CUDA_OK) return st;
        b0 += nb;
    }
    return TRC_CUDA_OK;
}

// trc_cuda_mul_mat_q in two steps: W dequantized into pooled, stream-ordered scratch, then
// trc_cuda_mul_mat on a view of it (transposed for a_transposed). TRC_CUDA_EUNSUPPORTED, with
// nothing launched, when the scratch cannot be allocated.
int mul_mat_q_two_step(int type, const void* w_blocks, int64_t w_ne0, int64_t w_ne1, int a_transposed,
                       const trc_cuda_view& b, const trc_cuda_view& d, uint32_t flags, cudaStream_t s) {
    const int64_t n = w_ne0 * w_ne1;
    retain_pool_once();
    void* wf = nullptr;
    if (cudaMallocAsync(&wf, static_cast<size_t>(n) * sizeof(float), s) != cudaSuccess) {
        cudaGetLastError();
        return TRC_CUDA_EUNSUPPORTED;
    }
    int st = trc_cuda_dequant(type, w_blocks, n / 32, static_cast<float*>(wf), s);
    if (st == TRC_CUDA_OK) {
        trc_cuda_view a;
        a.data = wf;
        a.ne[0] = a_transposed ? w_ne1 : w_ne0;
        a.ne[1] = a_transposed ? w_ne0 : w_ne1;
        a.ne[2] = a.ne[3] = 1;
        a.nb[0] = a_transposed ? 4 * w_ne0 : 4;
        a.nb[1] = a_transposed ? 4 : 4 * w_ne0;
        a.nb[2] = a.nb[3] = 4 * n;
        st = trc_cuda_mul_mat(&a, &b, &d, flags & ~(TRC_CUDA_MM_FUSED | TRC_CUDA_MM_NO_PRETAIL | TRC_CUDA_MM_TWO_STEP), s);
    }
    cudaFreeAsync(wf, s);
    return st;
}

// The upload as one copy and one dequant, both on the caller's stream: no stream, event or memory
// of the library's own is created (the allocation-free loader relies on this).
int load_quant_direct(int type, const void* host_blocks, int64_t n_blocks, void* staging, float* out,
                      cudaStream_t s) {
    const size_t bb = trc_cuda_block_bytes(type);
    const cudaError_t e =
        cudaMemcpyAsync(staging, host_blocks, static_cast<size_t>(n_blocks) * bb, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return cuda_fail(e);
    return trc_cuda_dequant(type, staging, n_blocks, out, s);
}

}  // namespace trc

using namespace trc;

extern "C" {

int trc_cuda_abi_version(void) { return TRC_CUDA_ABI_VERSION; }

const char* trc_cuda_status_string(int status) {
    switch (status) {
        case TRC_CUDA_OK: return "ok";
        case TRC_CUDA_EINVAL: return "invalid argument (null pointer, bad size or shape rule violated)";
        case TRC_CUDA_EUNSUPPORTED: return "unsupported type or layout";
        case TRC_CUDA_EDEVICE: return "a kernel hit its wait limit (device error word set)";
        case TRC_CUDA_ECUDA: return "CUDA runtime error";
        case TRC_CUDA_ENOMEM: return "device allocation failed";
        case TRC_CUDA_ETOOBIG: return "tensor larger than the fixed 64 MiB static staging buffer";
        default: return "unknown status";
    }
}

int trc_cuda_last_cuda_error(void) { return g_last_cuda_error; }

int trc_cuda_selftest_wait_timeout(uint64_t limit_ns, int* completed) {
    if (completed == nullptr || limit_ns == 0 || limit_ns > 5000000000ull) return TRC_CUDA_EINVAL;
    int* d = nullptr;
    cudaError_t e = cudaMalloc(&d, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e);
    selftest_wait_kernel<<<1, 32>>>(limit_ns, d);
    note_launch();
    e = cudaMemcpy(completed, d, sizeof(int), cudaMemcpyDeviceToHost);
    cudaFree(d);
    return e == cudaSuccess ? TRC_CUDA_OK : cuda_fail(e);
}

int trc_cuda_device_error(int* code, int reset) {
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e);
    if (code != nullptr) *code = v;
    if (reset != 0 && v != 0) {
        const int zero = 0;
        e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
        if (e != cudaSuccess) return cuda_fail(e);
    }
    return TRC_CUDA_OK;
}

uint64_t trc_cuda_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int trc_cuda_sm_count(void) { return sm_count_current(); }

size_t trc_cuda_block_bytes(int type) {
    switch (type) {
        case TRC_CUDA_TYPE_Q4_0: return 18;
        case TRC_CUDA_TYPE_Q4_1: return 20;
        case TRC_CUDA_TYPE_Q5_0: return 22;
        case TRC_CUDA_TYPE_Q5_1: return 24;
        case TRC_CUDA_TYPE_Q8_0: return 34;
        default: return 0;
    }
}

int trc_cuda_dequant(int type, const void* blocks, int64_t n_blocks, float* out, void* stream) {
    if (trc_cuda_block_bytes(type) == 0) return TRC_CUDA_EUNSUPPORTED;
    trc_cuda_dequant_job job;
    job.blocks   = blocks;
    job.out      = out;
    job.n_blocks = n_blocks;
    job.type     = type;
    job.reserved = 0;
    return dequant_jobs(&job, 1, static_cast<cudaStream_t>(stream));
}

int trc_cuda_dequant_many(const trc_cuda_dequant_job* jobs, int n_jobs, void* stream) {
    return dequant_jobs(jobs, n_jobs, static_cast<cudaStream_t>(stream));
}

int trc_cuda_dequant_many_to_peers(const trc_cuda_dequant_job* jobs, int n_jobs, const void* local_base,
                                   void* const* peer_bases, int n_peers, void* stream) {
    return dequant_jobs_peers(jobs, n_jobs, local_base, peer_bases, n_peers, static_cast<cudaStream_t>(stream));
}

int trc_cuda_load_quant(int type, const void* host_blocks, int64_t n_blocks, void* staging, float* out,
                        void* stream) {
    const size_t bb = trc_cuda_block_bytes(type);
    if (bb == 0) return TRC_CUDA_EUNSUPPORTED;
    if (n_blocks < 0) return TRC_CUDA_EINVAL;
    if (n_blocks == 0) return TRC_CUDA_OK;
    if (host_blocks == nullptr || staging == nullptr || out == nullptr) return TRC_CUDA_EINVAL;
    if ((reinterpret_cast<uint64_t>(staging) & 15u) != 0) return TRC_CUDA_EINVAL;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (static_cast<size_t>(n_blocks) * bb >= kPipelineMinBytes)
        return load_quant_pipelined(type, static_cast<const uint8_t*>(host_blocks), n_blocks,
                                    static_cast<uint8_t*>(staging), out, s);
    return load_quant_direct(type, host_blocks, n_blocks, staging, out, s);
}

// Shape rules of the mul_mat constructor (src/ops/trc_ops.cpp:366-385).
static int check_mul_mat_shapes(const trc_cuda_view* a, const trc_cuda_view* b, const trc_cuda_view* d) {
    if (!view_ok(a) || !view_ok(b) || !view_ok(d)) return TRC_CUDA_EINVAL;
    if (a->ne[0] != b->ne[0]) return TRC_CUDA_EINVAL;
    if (a->ne[2] <= 0 || a->ne[3] <= 0 || b->ne[2] % a->ne[2] != 0 || b->ne[3] % a->ne[3] != 0)
        return TRC_CUDA_EINVAL;
    if (d->ne[0] != a->ne[1] || d->ne[1] != b->ne[1] || d->ne[2] != b->ne[2] || d->ne[3] != b->ne[3])
        return TRC_CUDA_EINVAL;
    return TRC_CUDA_OK;
}

int trc_cuda_mul_mat(const trc_cuda_view* a, const trc_cuda_view* b, const trc_cuda_view* d, uint32_t flags,
                     void* stream) {
    int st = check_mul_mat_shapes(a, b, d);
    if (st != TRC_CUDA_OK) return st;
    if (nelements(*d) == 0) return TRC_CUDA_OK;
    const bool acc = (flags & TRC_CUDA_MM_ACCUMULATE) != 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (a->ne[0] == 0) {  // empty reduction: d = 0 (or unchanged when accumulating)
        if (acc) return TRC_CUDA_OK;
        return mul_mat_simt(*a, *b, *d, false, s);
    }
    if ((flags & TRC_CUDA_MM_SIMT) == 0) {
        st = mul_mat_tc(*a, *b, *d, flags, s);
        if (st != TRC_CUDA_EUNSUPPORTED) return st;
    }
    return mul_mat_simt(*a, *b, *d, acc, s);
}

int trc_cuda_mul_mat_repeat_back(const trc_cuda_view* a, const trc_cuda_view* b, const trc_cuda_view* d,
                                 uint32_t flags, void* stream) {
    if (!view_ok(a) || !view_ok(b) || !view_ok(d)) return TRC_CUDA_EINVAL;
    if (a->ne[0] != b->ne[0]) return TRC_CUDA_EINVAL;
    if (a->ne[2] <= 0 || a->ne[3] <= 0 || b->ne[2] % a->ne[2] != 0 || b->ne[3] % a->ne[3] != 0) return TRC_CUDA_EINVAL;
    if (d->ne[0] != a->ne[1] || d->ne[1] != b->ne[1] || d->ne[2] <= 0 || d->ne[3] <= 0 ||
        b->ne[2] % d->ne[2] != 0 || b->ne[3] % d->ne[3] != 0)
        return TRC_CUDA_EINVAL;
    if (nelements(*d) == 0) return TRC_CUDA_OK;
    const bool acc = (flags & TRC_CUDA_MM_ACCUMULATE) != 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (a->ne[0] == 0) {
        if (acc) return TRC_CUDA_OK;
        return mul_mat_simt(*a, *b, *d, false, s);
    }
    if ((flags & TRC_CUDA_MM_SIMT) == 0) {
        const int st = mul_mat_tc(*a, *b, *d, flags, s);
        if (st != TRC_CUDA_EUNSUPPORTED) return st;
    }
    return mul_mat_simt(*a, *b, *d, acc, s);
}

int trc_cuda_mul_mat_kernel(const trc_cuda_view* a, const trc_cuda_view* b, const trc_cuda_view* d, uint32_t flags) {
    const int st = check_mul_mat_shapes(a, b, d);
    if (st != TRC_CUDA_OK) return st;
    if ((flags & TRC_CUDA_MM_SIMT) != 0 || nelements(*d) == 0 || a->ne[0] == 0) return TRC_CUDA_KERNEL_SIMT;
    return mul_mat_tc_eligible(*a, *b, *d) ? TRC_CUDA_KERNEL_TCGEN05 : TRC_CUDA_KERNEL_SIMT;
}

int trc_cuda_mul_mat_q(int type, const void* w_blocks, int64_t w_ne0, int64_t w_ne1, int a_transposed,
                       const trc_cuda_view* b, const trc_cuda_view* d, uint32_t flags, void* stream) {
    if (trc_cuda_block_bytes(type) == 0) return TRC_CUDA_EUNSUPPORTED;
    if (w_blocks == nullptr || w_ne0 <= 0 || w_ne1 <= 0 || (w_ne0 % 32) != 0) return TRC_CUDA_EINVAL;
    if (!view_ok(b) || !view_ok(d)) return TRC_CUDA_EINVAL;
    const int64_t K = a_transposed ? w_ne1 : w_ne0;
    const int64_t M = a_transposed ? w_ne0 : w_ne1;
    if (b->ne[0] != K || d->ne[0] != M || d->ne[1] != b->ne[1] || d->ne[2] != b->ne[2] || d->ne[3] != b->ne[3])
        return TRC_CUDA_EINVAL;
    if (nelements(*d) == 0) return TRC_CUDA_OK;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Two steps with TRC_CUDA_MM_SIMT (the bit-exact mode) or TRC_CUDA_MM_TWO_STEP, and by default from
    // kTwoStepMinColumns columns on where the fused kernel cannot stage the packed bytes by TMA;
    // the fused kernel otherwise (TRC_CUDA_MM_FUSED forces it).
    const bool fused = (flags & TRC_CUDA_MM_FUSED) != 0;
    const bool two_step = (flags & (TRC_CUDA_MM_SIMT | TRC_CUDA_MM_TWO_STEP)) != 0 ||
                          (b->ne[1] >= kTwoStepMinColumns &&
                           !mul_mat_q_tma_staged(type, w_blocks, w_ne0, w_ne1, a_transposed, flags));
    if (!fused && two_step) {
        const int st = mul_mat_q_two_step(type, w_blocks, w_ne0, w_ne1, a_transposed, *b, *d, flags, s);
        if (st != TRC_CUDA_EUNSUPPORTED) return st;  // else: no scratch memory, the fused kernel runs
    }
    return mul_mat_q_tc(type, w_blocks, w_ne0, w_ne1, a_transposed, *b, *d, flags, s);
}

}  // extern "C"
