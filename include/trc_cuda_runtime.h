/* trc_cuda_runtime.h -- device-management part of the C ABI of libtrc_cuda.so.
 *
 * The C++ backend (train.cpp_b200/backend/trc_cuda_backend.cpp) manages device memory, copies and
 * streams only through these calls, so one CUDA runtime instance (the one inside libtrc_cuda.so)
 * serves the whole process. They back the reference's BufferType::alloc_buffer,
 * Buffer::set_tensor / get_tensor / clear and Device::props
 * (include/traincpp/trc_backend.h:33-88 of train.cpp). Every function returns a TRC_CUDA_* status
 * (include/trc_cuda.h); a failed CUDA call returns TRC_CUDA_ECUDA and leaves its cudaError_t in
 * trc_cuda_last_cuda_error(). Allocation failure returns TRC_CUDA_ENOMEM and does not abort.
 */
#ifndef TRC_CUDA_RUNTIME_H
#define TRC_CUDA_RUNTIME_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

int         trc_cuda_rt_device_count(int* count);       /* 0 devices is not an error */
int         trc_cuda_rt_set_device(int ordinal);
int         trc_cuda_rt_get_device(int* ordinal);
/* name (NUL-terminated, truncated to name_len), compute capability, memory */
int         trc_cuda_rt_device_info(int ordinal, char* name, size_t name_len, int* cc_major, int* cc_minor);
int         trc_cuda_rt_mem_info(size_t* free_bytes, size_t* total_bytes);
const char* trc_cuda_rt_error_string(int cuda_error);

int trc_cuda_rt_malloc(void** ptr, size_t bytes);        /* device memory of the current device */
int trc_cuda_rt_free(void* ptr);
int trc_cuda_rt_malloc_host(void** ptr, size_t bytes);   /* pinned host memory */
/* Number of successful trc_cuda_rt_malloc_host calls in this process (page-locking is a system
 * call; loaders that reuse their pinned staging keep this constant across repeated loads). */
uint64_t trc_cuda_rt_host_alloc_count(void);
int trc_cuda_rt_free_host(void* ptr);

/* kind: 0 host->device, 1 device->host, 2 device->device. Synchronous. */
int trc_cuda_rt_memcpy(void* dst, const void* src, size_t bytes, int kind);
int trc_cuda_rt_memset(void* dst, int value, size_t bytes);
/* Asynchronous on `stream`; a host side must be pinned (trc_cuda_rt_malloc_host) to overlap. */
int trc_cuda_rt_memcpy_async(void* dst, const void* src, size_t bytes, int kind, void* stream);

int trc_cuda_rt_stream_create(void** stream);           /* non-blocking stream of the current device */
int trc_cuda_rt_stream_destroy(void* stream);
int trc_cuda_rt_stream_sync(void* stream);

/* Events (timing disabled): mark a point of a stream's work and wait for it from the host, e.g.
 * before a pinned staging buffer that an asynchronous copy reads is refilled. */
int trc_cuda_rt_event_create(void** event);
int trc_cuda_rt_event_destroy(void* event);
int trc_cuda_rt_event_record(void* event, void* stream);
int trc_cuda_rt_event_sync(void* event);

/* Peer memory between the processes of one node (one process per GPU), for the dequant
 * all-gather over NVLink (trc_cuda_dequant_many_to_peers). Plain CUDA IPC mappings: peer loads
 * and stores, no multicast object. ptr must be the base of a trc_cuda_rt_malloc allocation; the
 * handle is TRC_CUDA_IPC_HANDLE_BYTES opaque bytes that another process passes to
 * trc_cuda_rt_ipc_open, which maps the allocation into the current device's address space
 * (peer access enabled on first use). trc_cuda_rt_ipc_close unmaps it. */
#define TRC_CUDA_IPC_HANDLE_BYTES 64
int trc_cuda_rt_ipc_get_handle(void* ptr, void* handle);
int trc_cuda_rt_ipc_open(const void* handle, void** ptr);
int trc_cuda_rt_ipc_close(void* ptr);
int trc_cuda_rt_can_access_peer(int device, int peer, int* can_access);

#ifdef __cplusplus
}
#endif

#endif /* TRC_CUDA_RUNTIME_H */
