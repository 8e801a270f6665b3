// trc_cuda_backend.h -- CUDA (B200, sm_100a) backend for train.cpp, behind its abstract backend
// interface (include/traincpp/trc_backend.h:33-88). Drop-in: the GGUF reader, op constructors,
// autograd, graph_first_unsupported and graph_compute callers stay unchanged; this file only adds
// a Device / BufferType / Buffer implementation whose kernels live in libtrc_cuda.so
// (include/trc_cuda.h).
//
// Registration mirrors the reference's backend entry points (src/core/trc_backends.h:14-22):
// cuda_device(i) returns the process-lifetime device of GPU i; cuda_register_devices() appends every
// visible GPU to the registry with backend_register_device() (src/core/trc_backend_reg.cpp:89-92),
// after which device_by_type(DeviceType::GPU) and TRC_TEST_DEVICE-style selection find it.
#pragma once

#include "traincpp/traincpp.h"

#include <cstddef>
#include <cstdint>
#include <vector>

namespace traincpp {

// Number of CUDA devices visible to the process (0 when no driver/GPU is present).
int cuda_device_count();

// The CUDA device for GPU `ordinal` (created on first use), or nullptr if there is no such GPU.
Device* cuda_device(int ordinal = 0);

// Registers every visible GPU with the backend registry (idempotent). Returns how many are registered.
int cuda_register_devices();

// Device-side gguf_load_tensor (src/io/trc_gguf.cpp:1051-1094) for a quantized file tensor and an F32
// destination allocated on a CUDA buffer: the packed blocks are read from `path` into pinned host
// staging, copied to the device (4-8x fewer bytes than the F32 result) and dequantized there,
// bit-exact with the reference. Non-quantized file types and non-CUDA destinations fall back to
// the reference's own gguf_load_tensor. Returns false (and logs) where the reference would.
bool cuda_gguf_load_tensor(const GgufFile* f, const char* path, const char* name, Tensor* dst);

// The file tensors rank `rank` of `world` loads when a whole model is dealt to one process per GPU:
// a byte-balanced greedy LPT over each tensor's load bytes (bytes read + F32 bytes written),
// largest first, ties by file order, each tensor to the least-loaded rank (ties to the lowest).
// Returns this rank's tensor indices in file order; the ranks' lists partition the file.
std::vector<int64_t> gguf_shard_tensors(const GgufFile* f, int rank, int world);

// Streams `count` file tensors into their F32 destinations on one CUDA device (the GGUF reader can
// have been opened with load_data = false: nothing of the data segment is held on the host).
// Packed blocks are read from `path` in chunks of whole blocks into two pinned staging buffers of
// `staging_bytes`; the file read of the next chunk overlaps the copy and dequant of the current one
// on the device; F32 file tensors are copied the same way. Other file types (F16), and destinations
// that are not on a CUDA buffer, go through the reference's gguf_load_tensor (which needs the data
// segment loaded). Bit-exact with gguf_load_tensor; returns false (and logs) where the reference
// would.
bool cuda_gguf_load_tensors(const GgufFile* f, const char* path, const char* const* names, Tensor* const* dsts,
                            size_t count, size_t staging_bytes = size_t(64) << 20);

// ---- frozen quantized weights that never exist as F32 in device memory ----------------------
//
// A second buffer type of GPU `ordinal`, "CUDA<i>_Q", for frozen weights kept as their packed GGUF
// blocks. Tensors allocated from it (buffer_alloc_ctx_tensors on a context holding only such
// weights) stay ordinary F32 graph tensors, so train.cpp's op constructors, autograd and
// nn::Linear accept them unchanged (mul_mat requires a->type == b->type, src/ops/trc_ops.cpp:368,
// and quantized types are not allocatable, src/core/trc_types.cpp:104-118). Their F32 bytes are
// never backed: the buffer holds, per weight, the packed blocks loaded into it, described by
// Tensor::extra (include/traincpp/trc_tensor.h:62). The CUDA device runs mul_mat(W, x) and
// mul_mat(transpose(W), g) -- a Linear's forward and its dX -- with the dequant-in-prologue GEMM,
// which decodes the blocks inside the GEMM and writes no F32 copy of W anywhere. Rules:
//   - a weight is 2-D (ne[2] = ne[3] = 1), F32-typed, with ne[0] a multiple of 32, and must be
//     loaded (cuda_gguf_load_tensor, cuda_gguf_load_tensors or cuda_set_tensor_from_quant) before a
//     graph reads it; the weight is frozen (its blocks change only by another load);
//   - supports_op answers false for every node that would read a packed weight other than
//     mul_mat with the weight (or its transpose) as the first operand, so graph_first_unsupported
//     reports such graphs; tensor_get dequantizes (bit-exact with the reference's host
//     dequantizers); tensor_set of F32 data is refused (the library does not quantize).
// With TRC_CUDA_PACKED_TWO_STEP=1, every product dequantizes W into stream-ordered scratch for the
// duration of one GEMM instead (same results, bit for bit).
BufferType* cuda_packed_buffer_type(int ordinal = 0);

// True when t (or the root of the view t) lives on a packed-weight buffer.
bool cuda_tensor_is_packed(const Tensor* t);

// The Buffer::set_tensor_from_quant hook of this backend: makes `bytes` of packed GGUF blocks of
// `type` (HOST memory) the data of the F32 tensor `dst`. On a packed-weight buffer the blocks are
// stored as they are; on an ordinary CUDA buffer they are uploaded and dequantized on the device
// (bit-exact with the reference). Returns false (and logs) for a non-legacy type, a size that does
// not match dst's element count, a non-contiguous dst, or a dst that is not on this backend.
bool cuda_set_tensor_from_quant(Tensor* dst, Type type, const void* packed, size_t bytes);

}  // namespace traincpp

extern "C" {
// C entry points of the backend library, for hosts that do not link C++ (ctypes, cgo, ...).
int trc_cuda_backend_register(void);
void* trc_cuda_backend_device(int ordinal);
// gguf_shard_tensors of the file at `path` (read without its data segment): writes up to `capacity`
// tensor indices of rank `rank` and returns how many the rank has, or -1 on a bad argument / file.
// Needs no GPU.
int64_t trc_cuda_backend_gguf_shard_plan(const char* path, int rank, int world, int64_t* indices, int64_t capacity);
}
