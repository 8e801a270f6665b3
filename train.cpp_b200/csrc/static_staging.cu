// static_staging.cu -- trc_cuda_load_quant_static: the GGUF device loader without any allocation.
//
// Some callers cannot call cudaMalloc (their device memory belongs to another allocator or has a
// fixed budget). For them the packed blocks are staged in a fixed array of this library instead of
// a caller-provided buffer: a file-scope static __device__ array that each GPU holds from the moment
// the library's device code is loaded there until the process exits. In host code the array's name
// only stands in for the symbol; its device address on the current device is looked up with
// cudaGetSymbolAddress on every call (a host-side lookup once the module is loaded, and never stale
// after a device reset re-creates the context) and passed to the copy and the kernel.
#include <cuda_runtime.h>

#include <cstdint>

#include "trc_internal.h"

namespace {

static __device__ __align__(256) uint8_t g_static_staging[TRC_CUDA_STATIC_STAGING_BYTES];

// Device address of g_static_staging on the current device. The first use of the library's device
// code on a device loads its module (lazy loading) and with it reserves the array; later lookups
// are host-side only.
int static_staging_address(void** out) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_static_staging);
    if (e != cudaSuccess) return trc::cuda_fail(e);
    *out = p;
    return TRC_CUDA_OK;
}

}  // namespace

extern "C" int trc_cuda_load_quant_static(int type, const void* host_blocks, int64_t n_blocks, float* out,
                                          void* stream) {
    const size_t bb = trc_cuda_block_bytes(type);
    if (bb == 0) return TRC_CUDA_EUNSUPPORTED;
    if (n_blocks < 0) return TRC_CUDA_EINVAL;
    if (static_cast<uint64_t>(n_blocks) > TRC_CUDA_STATIC_STAGING_BYTES / bb) return TRC_CUDA_ETOOBIG;
    // the lookup comes first, so that a zero-size warm-up call also loads the module on this device
    void* staging = nullptr;
    const int st = static_staging_address(&staging);
    if (st != TRC_CUDA_OK) return st;
    if (n_blocks == 0) return TRC_CUDA_OK;
    if (host_blocks == nullptr || out == nullptr) return TRC_CUDA_EINVAL;
    // One copy and one dequant on the caller's stream, whatever the size: the chunked upload of
    // trc_cuda_load_quant would create a copy stream and events of the library's own.
    return trc::load_quant_direct(type, host_blocks, n_blocks, staging, out, static_cast<cudaStream_t>(stream));
}
