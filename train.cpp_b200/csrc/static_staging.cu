// static_staging.cu -- trc_cuda_load_quant_static: the GGUF device loader without any allocation.
//
// Some callers cannot call cudaMalloc (their device memory belongs to another allocator or has a
// fixed budget). For them the packed blocks are staged in a fixed array of this library instead of
// a caller-provided buffer: a file-scope static __device__ array that each GPU loading the
// library holds until the process exits. In host code the array's name only stands in for the
// symbol; its device address for the current device is looked up once with cudaGetSymbolAddress
// (the first call on a device does this, before any stream capture should begin) and passed on.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "trc_internal.h"

namespace {

static __device__ __align__(256) uint8_t g_static_staging[TRC_CUDA_STATIC_STAGING_BYTES];

constexpr int kMaxDevices = 64;

// Device address of g_static_staging on the current device (looked up once per device).
int static_staging_address(void** out) {
    static std::mutex mu;
    static void*      addr[kMaxDevices] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return trc::cuda_fail(e);
    if (dev < 0 || dev >= kMaxDevices) return TRC_CUDA_EUNSUPPORTED;
    std::lock_guard<std::mutex> lock(mu);
    if (addr[dev] == nullptr) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_static_staging);
        if (e != cudaSuccess) return trc::cuda_fail(e);
        addr[dev] = p;
    }
    *out = addr[dev];
    return TRC_CUDA_OK;
}

}  // namespace

extern "C" int trc_cuda_load_quant_static(int type, const void* host_blocks, int64_t n_blocks, float* out,
                                          void* stream) {
    const size_t bb = trc_cuda_block_bytes(type);
    if (bb == 0) return TRC_CUDA_EUNSUPPORTED;
    if (n_blocks < 0) return TRC_CUDA_EINVAL;
    if (n_blocks == 0) return TRC_CUDA_OK;
    if (host_blocks == nullptr || out == nullptr) return TRC_CUDA_EINVAL;
    if (static_cast<uint64_t>(n_blocks) > TRC_CUDA_STATIC_STAGING_BYTES / bb) return TRC_CUDA_ETOOBIG;
    void* staging = nullptr;
    const int st = static_staging_address(&staging);
    if (st != TRC_CUDA_OK) return st;
    // One copy and one dequant on the caller's stream, whatever the size: the chunked upload of
    // trc_cuda_load_quant would create a copy stream and events of the library's own.
    return trc::load_quant_direct(type, host_blocks, n_blocks, staging, out, static_cast<cudaStream_t>(stream));
}
