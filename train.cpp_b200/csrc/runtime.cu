// runtime.cu -- device-management entry points of the C ABI (include/trc_cuda_runtime.h): the
// C++ backend allocates, copies and synchronises only through these, so the process uses the one
// CUDA runtime linked into libtrc_cuda.so.
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>

#include "../../include/trc_cuda_runtime.h"
#include "trc_internal.h"

using namespace trc;

namespace {
int rt(cudaError_t e) { return e == cudaSuccess ? TRC_CUDA_OK : cuda_fail(e); }
}  // namespace

extern "C" {

int trc_cuda_rt_device_count(int* count) {
    if (count == nullptr) return TRC_CUDA_EINVAL;
    *count = 0;
    const cudaError_t e = cudaGetDeviceCount(count);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
        cudaGetLastError();
        *count = 0;
        return TRC_CUDA_OK;
    }
    return rt(e);
}

int trc_cuda_rt_set_device(int ordinal) { return rt(cudaSetDevice(ordinal)); }

int trc_cuda_rt_get_device(int* ordinal) {
    if (ordinal == nullptr) return TRC_CUDA_EINVAL;
    return rt(cudaGetDevice(ordinal));
}

int trc_cuda_rt_device_info(int ordinal, char* name, size_t name_len, int* cc_major, int* cc_minor) {
    cudaDeviceProp prop;
    const int st = rt(cudaGetDeviceProperties(&prop, ordinal));
    if (st != TRC_CUDA_OK) return st;
    if (name != nullptr && name_len > 0) {
        std::strncpy(name, prop.name, name_len - 1);
        name[name_len - 1] = '\0';
    }
    if (cc_major != nullptr) *cc_major = prop.major;
    if (cc_minor != nullptr) *cc_minor = prop.minor;
    return TRC_CUDA_OK;
}

int trc_cuda_rt_mem_info(size_t* free_bytes, size_t* total_bytes) {
    if (free_bytes == nullptr || total_bytes == nullptr) return TRC_CUDA_EINVAL;
    return rt(cudaMemGetInfo(free_bytes, total_bytes));
}

const char* trc_cuda_rt_error_string(int cuda_error) { return cudaGetErrorString(static_cast<cudaError_t>(cuda_error)); }

int trc_cuda_rt_malloc(void** ptr, size_t bytes) {
    if (ptr == nullptr) return TRC_CUDA_EINVAL;
    const cudaError_t e = cudaMalloc(ptr, bytes == 0 ? 256 : bytes);
    if (e == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        *ptr = nullptr;
        return TRC_CUDA_ENOMEM;
    }
    return rt(e);
}

int trc_cuda_rt_free(void* ptr) { return rt(cudaFree(ptr)); }

static std::atomic<uint64_t> g_host_allocs{0};

uint64_t trc_cuda_rt_host_alloc_count(void) { return g_host_allocs.load(std::memory_order_relaxed); }

int trc_cuda_rt_malloc_host(void** ptr, size_t bytes) {
    if (ptr == nullptr) return TRC_CUDA_EINVAL;
    const cudaError_t e = cudaMallocHost(ptr, bytes == 0 ? 1 : bytes);
    if (e == cudaErrorMemoryAllocation) {
        cudaGetLastError();
        *ptr = nullptr;
        return TRC_CUDA_ENOMEM;
    }
    if (e == cudaSuccess) g_host_allocs.fetch_add(1, std::memory_order_relaxed);
    return rt(e);
}

int trc_cuda_rt_free_host(void* ptr) { return rt(cudaFreeHost(ptr)); }

int trc_cuda_rt_memcpy(void* dst, const void* src, size_t bytes, int kind) {
    if (bytes == 0) return TRC_CUDA_OK;
    if (dst == nullptr || src == nullptr) return TRC_CUDA_EINVAL;
    const cudaMemcpyKind k = kind == 0 ? cudaMemcpyHostToDevice : kind == 1 ? cudaMemcpyDeviceToHost
                                                                             : cudaMemcpyDeviceToDevice;
    if (kind < 0 || kind > 2) return TRC_CUDA_EINVAL;
    return rt(cudaMemcpy(dst, src, bytes, k));
}

int trc_cuda_rt_memcpy_async(void* dst, const void* src, size_t bytes, int kind, void* stream) {
    if (bytes == 0) return TRC_CUDA_OK;
    if (dst == nullptr || src == nullptr || kind < 0 || kind > 2) return TRC_CUDA_EINVAL;
    const cudaMemcpyKind k = kind == 0 ? cudaMemcpyHostToDevice : kind == 1 ? cudaMemcpyDeviceToHost
                                                                             : cudaMemcpyDeviceToDevice;
    return rt(cudaMemcpyAsync(dst, src, bytes, k, static_cast<cudaStream_t>(stream)));
}

int trc_cuda_rt_memset(void* dst, int value, size_t bytes) {
    if (bytes == 0) return TRC_CUDA_OK;
    if (dst == nullptr) return TRC_CUDA_EINVAL;
    return rt(cudaMemset(dst, value, bytes));
}

int trc_cuda_rt_stream_create(void** stream) {
    if (stream == nullptr) return TRC_CUDA_EINVAL;
    cudaStream_t s = nullptr;
    const int st = rt(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    *stream = s;
    return st;
}

int trc_cuda_rt_stream_destroy(void* stream) { return rt(cudaStreamDestroy(static_cast<cudaStream_t>(stream))); }

int trc_cuda_rt_stream_sync(void* stream) { return rt(cudaStreamSynchronize(static_cast<cudaStream_t>(stream))); }

int trc_cuda_rt_event_create(void** event) {
    if (event == nullptr) return TRC_CUDA_EINVAL;
    cudaEvent_t e = nullptr;
    const int st = rt(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    *event = e;
    return st;
}

int trc_cuda_rt_event_destroy(void* event) { return rt(cudaEventDestroy(static_cast<cudaEvent_t>(event))); }

int trc_cuda_rt_event_record(void* event, void* stream) {
    if (event == nullptr) return TRC_CUDA_EINVAL;
    return rt(cudaEventRecord(static_cast<cudaEvent_t>(event), static_cast<cudaStream_t>(stream)));
}

int trc_cuda_rt_event_sync(void* event) {
    if (event == nullptr) return TRC_CUDA_EINVAL;
    return rt(cudaEventSynchronize(static_cast<cudaEvent_t>(event)));
}

static_assert(sizeof(cudaIpcMemHandle_t) == TRC_CUDA_IPC_HANDLE_BYTES, "IPC handle size");

int trc_cuda_rt_ipc_get_handle(void* ptr, void* handle) {
    if (ptr == nullptr || handle == nullptr) return TRC_CUDA_EINVAL;
    cudaIpcMemHandle_t h;
    const int st = rt(cudaIpcGetMemHandle(&h, ptr));
    if (st == TRC_CUDA_OK) std::memcpy(handle, &h, sizeof(h));
    return st;
}

int trc_cuda_rt_ipc_open(const void* handle, void** ptr) {
    if (handle == nullptr || ptr == nullptr) return TRC_CUDA_EINVAL;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    *ptr = nullptr;
    return rt(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int trc_cuda_rt_ipc_close(void* ptr) {
    if (ptr == nullptr) return TRC_CUDA_EINVAL;
    return rt(cudaIpcCloseMemHandle(ptr));
}

int trc_cuda_rt_can_access_peer(int device, int peer, int* can_access) {
    if (can_access == nullptr) return TRC_CUDA_EINVAL;
    *can_access = 0;
    return rt(cudaDeviceCanAccessPeer(can_access, device, peer));
}

}  // extern "C"
