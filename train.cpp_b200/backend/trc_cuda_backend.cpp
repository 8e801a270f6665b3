// trc_cuda_backend.cpp -- train.cpp's abstract backend (include/traincpp/trc_backend.h:33-88)
// implemented for NVIDIA B200 on top of the C ABI of libtrc_cuda.so (include/trc_cuda.h).
//
//   CudaBufferType  device() / name() "CUDA<i>" / alignment() 256 / alloc_buffer() -> nullptr on
//                   failure, so the core prints need/available and aborts as it does for every
//                   backend (src/core/trc_backend_reg.cpp:248-264)
//   CudaBuffer      device-local memory: base() is nullptr and tensors are located by
//                   Tensor::data_offset (src/core/trc_backend_reg.cpp:276-279); set/get_tensor are
//                   host<->device copies; clear() a device memset
//   CudaDevice      supports_op() answers for every node without aborting; graph_compute() runs
//                   each node's kernel on the device's stream and returns when results are ready
//                   (the synchronous contract of trc_backend.h:78); fill_tensors() is a device fill
//
// Fatal errors abort with file:line and a message, like the reference's TRC_ABORT
// (src/core/trc_impl.h:118-125); a kernel that gave up a bounded wait is reported the same way.
#include "trc_cuda_backend.h"

#include <cstdarg>
#include <cstdio>
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <condition_variable>
#include <mutex>
#include <thread>
#include <string>
#include <unordered_map>
#include <vector>

#include "trc_cuda.h"
#include "trc_cuda_runtime.h"

namespace traincpp {

namespace {

[[noreturn]] void backend_abort(const char* file, int line, const char* fmt, ...) {
    std::fprintf(stderr, "[traincpp] 致命错误 %s:%d: ", file, line);
    va_list ap;
    va_start(ap, fmt);
    std::vfprintf(stderr, fmt, ap);
    va_end(ap);
    std::fprintf(stderr, "\n");
    std::fflush(stderr);
    std::abort();
}

#define CB_ABORT(...) backend_abort(__FILE__, __LINE__, __VA_ARGS__)
#define CB_CUDA(call)                                                                                   \
    do {                                                                                                \
        const int s_ = (call);                                                                          \
        if (s_ != TRC_CUDA_OK)                                                                          \
            CB_ABORT("CUDA: %s -> %s (%s)", #call, trc_cuda_status_string(s_),                          \
                     trc_cuda_rt_error_string(trc_cuda_last_cuda_error()));                             \
    } while (0)
#define CB_TRC(call, what)                                                                          \
    do {                                                                                            \
        const int s_ = (call);                                                                      \
        if (s_ != TRC_CUDA_OK)                                                                      \
            CB_ABORT("CUDA: %s failed: %s (cudaError %d)", what, trc_cuda_status_string(s_),         \
                     trc_cuda_last_cuda_error());                                                   \
    } while (0)

// Host-side failure injection for tests (no GPU fault involved): TRC_CUDA_FAIL_ALLOC=n makes the
// n-th buffer allocation of the process fail as if the device were out of memory.
bool fake_alloc_failure() {
    static std::mutex mu;
    static long counter = 0;
    const char* env = std::getenv("TRC_CUDA_FAIL_ALLOC");
    if (env == nullptr) return false;
    std::lock_guard<std::mutex> lock(mu);
    ++counter;
    return counter == std::atol(env);
}

class CudaDevice;

// Host <-> device copies of one tensor through the device's two pinned chunks (below): the host
// copy of one chunk overlaps the DMA of the other. Synchronous like cudaMemcpy. Measured on B200
// for a 235 MB tensor: a pageable cudaMemcpy moves 10.9 GB/s, a pinned one 53.1 GB/s, and a host
// memcpy into pinned memory 45.5 GB/s.
constexpr size_t kStagedCopyMin = size_t(4) << 20;   // below this a plain cudaMemcpy
constexpr size_t kStagedChunk   = size_t(8) << 20;
void staged_h2d(CudaDevice* dev, void* dst, const void* src, size_t bytes);
void staged_d2h(CudaDevice* dev, void* dst, const void* src, size_t bytes);

class CudaBufferType : public BufferType {
public:
    explicit CudaBufferType(CudaDevice* dev, int ordinal) : dev_(dev) {
        std::snprintf(name_, sizeof(name_), "CUDA%d", ordinal);
    }
    Device* device() const override;
    const char* name() const override { return name_; }
    size_t alignment() const override { return 256; }
    Buffer* alloc_buffer(size_t size) override;

private:
    CudaDevice* dev_;
    char        name_[16];
};

class CudaBuffer : public Buffer {
public:
    CudaBuffer(CudaBufferType* buft, int ordinal, char* dptr, size_t size)
        : buft_(buft), ordinal_(ordinal), dptr_(dptr), size_(size) {}
    ~CudaBuffer() override {
        int prev = 0;
        trc_cuda_rt_get_device(&prev);
        trc_cuda_rt_set_device(ordinal_);
        trc_cuda_rt_free(dptr_);
        trc_cuda_rt_set_device(prev);
    }
    BufferType* buffer_type() const override { return buft_; }
    size_t size() const override { return size_; }
    void* base() override { return nullptr; }  // device-local: not mappable by the host
    bool is_host() const override { return false; }

    // Large copies go through the device's pinned chunks (pageable host memory otherwise limits the
    // copy to about a fifth of what PCIe carries): the reference's tensor_set / tensor_get, and with
    // them gguf_load_tensor's and checkpoint_load's uploads, run at pinned-copy speed.
    void set_tensor(Tensor* t, size_t offset, const void* data, size_t size) override {
        check_range(t, offset, size, "set_tensor");
        CB_CUDA(trc_cuda_rt_set_device(ordinal_));
        if (size >= kStagedCopyMin) staged_h2d(device_of(), dptr_ + t->data_offset + offset, data, size);
        else CB_CUDA(trc_cuda_rt_memcpy(dptr_ + t->data_offset + offset, data, size, 0));
    }
    void get_tensor(const Tensor* t, size_t offset, void* data, size_t size) const override {
        check_range(t, offset, size, "get_tensor");
        CB_CUDA(trc_cuda_rt_set_device(ordinal_));
        if (size >= kStagedCopyMin) staged_d2h(device_of(), data, dptr_ + t->data_offset + offset, size);
        else CB_CUDA(trc_cuda_rt_memcpy(data, dptr_ + t->data_offset + offset, size, 1));
    }
    void clear() override {
        CB_CUDA(trc_cuda_rt_set_device(ordinal_));
        CB_CUDA(trc_cuda_rt_memset(dptr_, 0, size_));
    }

    char* device_ptr() const { return dptr_; }
    int   ordinal() const { return ordinal_; }
    CudaDevice* device_of() const;

private:
    void check_range(const Tensor* t, size_t offset, size_t size, const char* what) const {
        if (t->data_offset + offset + size > size_)
            CB_ABORT("CudaBuffer::%s: 越界 (data_offset=%zu offset=%zu size=%zu buffer=%zu)", what, t->data_offset,
                     offset, size, size_);
    }

    CudaBufferType* buft_;
    int             ordinal_;
    char*           dptr_;
    size_t          size_;
};

// Root buffer of a tensor (views resolve through view_src: src/core/trc_backend_reg.cpp:61-67).
CudaBuffer* cuda_buffer_of(const Tensor* t) {
    while (t != nullptr && t->buffer == nullptr && t->view_src != nullptr) t = t->view_src;
    if (t == nullptr || t->buffer == nullptr) return nullptr;
    return dynamic_cast<CudaBuffer*>(t->buffer);
}

trc_cuda_view view_of(const Tensor* t) {
    CudaBuffer* b = cuda_buffer_of(t);
    if (b == nullptr) CB_ABORT("CUDA: 张量 %s 不在 CUDA buffer 上", t->name);
    trc_cuda_view v;
    v.data = b->device_ptr() + t->data_offset;
    for (int i = 0; i < 4; ++i) {
        v.ne[i] = t->ne[i];
        v.nb[i] = static_cast<int64_t>(t->nb[i]);
    }
    return v;
}

// ---------------------------------------------------------------- packed-weight buffers
// A frozen quantized weight is an F32 graph tensor whose bytes are never backed: the buffer keeps
// the packed GGUF blocks loaded into it, and Tensor::extra of the weight points at their
// descriptor. Only mul_mat(W, x) and mul_mat(transpose(W), g) read it on the device (through the
// dequant-in-prologue GEMM); tensor_get dequantizes.
struct PackedWeight {
    const Buffer* owner = nullptr;  // the buffer that holds the blocks
    Type          type = TYPE_F32;  // Q4_0 .. Q8_0
    int64_t       ne0 = 0, ne1 = 0; // the F32 tensor's extents (2-D)
    void*         blocks = nullptr; // device memory: ne0 * ne1 / 32 blocks
    size_t        bytes = 0;
    size_t        capacity = 0;     // bytes allocated at `blocks`
};

class CudaPackedBufferType : public BufferType {
public:
    CudaPackedBufferType(CudaDevice* dev, int ordinal) : dev_(dev), ordinal_(ordinal) {
        std::snprintf(name_, sizeof(name_), "CUDA%d_Q", ordinal);
    }
    Device* device() const override;
    const char* name() const override { return name_; }
    size_t alignment() const override { return 256; }
    Buffer* alloc_buffer(size_t size) override;  // bookkeeping only: the blocks arrive with each load
    CudaDevice* cuda_device() const { return dev_; }
    int ordinal() const { return ordinal_; }

private:
    CudaDevice* dev_;
    int         ordinal_;
    char        name_[16];
};

Tensor* view_root(Tensor* t) {
    while (t->view_src != nullptr) t = t->view_src;
    return t;
}
const Tensor* view_root(const Tensor* t) {
    while (t->view_src != nullptr) t = t->view_src;
    return t;
}

class CudaPackedBuffer : public Buffer {
public:
    CudaPackedBuffer(CudaPackedBufferType* buft, size_t size) : buft_(buft), size_(size) {}
    ~CudaPackedBuffer() override {
        int prev = 0;
        trc_cuda_rt_get_device(&prev);
        trc_cuda_rt_set_device(buft_->ordinal());
        for (auto& kv : weights_) trc_cuda_rt_free(kv.second->blocks);
        trc_cuda_rt_set_device(prev);
    }
    BufferType* buffer_type() const override { return buft_; }
    size_t size() const override { return size_; }
    void* base() override { return nullptr; }
    bool is_host() const override { return false; }

    void set_tensor(Tensor* t, size_t, const void*, size_t) override {
        CB_ABORT("%s: 张量 %s 是冻结的量化权重，只能载入 GGUF 量化块（cuda_gguf_load_tensor / "
                 "cuda_set_tensor_from_quant）；本后端不做量化", buft_->name(), t->name);
    }
    void get_tensor(const Tensor* t, size_t offset, void* data, size_t size) const override;
    void clear() override;

    // Makes `bytes` of packed blocks (HOST memory) the data of root tensor t; false + log on a
    // mismatch. Synchronous.
    bool store(Tensor* t, Type type, const void* host, size_t bytes);

    const PackedWeight* weight_of(const Tensor* root) const {
        const auto it = weights_.find(root);
        if (it == weights_.end() || root->extra != it->second.get()) return nullptr;
        return it->second.get();
    }

private:
    CudaPackedBufferType* buft_;
    size_t                size_;
    std::unordered_map<const Tensor*, std::unique_ptr<PackedWeight>> weights_;
};

CudaPackedBuffer* packed_buffer_of(const Tensor* t) {
    if (t == nullptr) return nullptr;
    const Tensor* r = view_root(t);
    return r->buffer == nullptr ? nullptr : dynamic_cast<CudaPackedBuffer*>(r->buffer);
}

// How a graph operand refers to a packed weight: not at all, as W itself, as transpose(W) (the
// two forms the GEMM reads), or through a view the GEMM cannot take.
enum class PackedUse { none, plain, transposed, unsupported };

PackedUse packed_use(const Tensor* t, const PackedWeight** w_out) {
    CudaPackedBuffer* buf = packed_buffer_of(t);
    if (buf == nullptr) return PackedUse::none;
    const Tensor* r = view_root(t);
    const PackedWeight* w = buf->weight_of(r);
    if (w_out != nullptr) *w_out = w;
    if (r->ne[2] != 1 || r->ne[3] != 1 || t->ne[2] != 1 || t->ne[3] != 1) return PackedUse::unsupported;
    if (t->data_offset != r->data_offset && t != r) return PackedUse::unsupported;
    const int64_t ne0 = r->ne[0], ne1 = r->ne[1];
    if (t->ne[0] == ne0 && t->ne[1] == ne1 && t->nb[0] == 4 && t->nb[1] == static_cast<size_t>(4 * ne0))
        return PackedUse::plain;
    if (t->ne[0] == ne1 && t->ne[1] == ne0 && t->nb[1] == 4 && t->nb[0] == static_cast<size_t>(4 * ne0))
        return PackedUse::transposed;
    return PackedUse::unsupported;
}

bool all_f32(const Tensor* t) {
    if (t->type != TYPE_F32) return false;
    for (int i = 0; i < t->nsrc; ++i)
        if (t->src[i] != nullptr && t->src[i]->type != TYPE_F32) return false;
    return true;
}

class CudaDevice : public Device {
public:
    explicit CudaDevice(int ordinal) : ordinal_(ordinal), buft_(this, ordinal), packed_buft_(this, ordinal) {
        char name[256];
        int  major = 0, minor = 0;
        CB_CUDA(trc_cuda_rt_device_info(ordinal, name, sizeof(name), &major, &minor));
        CB_CUDA(trc_cuda_rt_set_device(ordinal));
        CB_CUDA(trc_cuda_rt_stream_create(&stream_));
        props_.name        = std::string("CUDA") + std::to_string(ordinal);
        props_.description = std::string(name) + " (sm_" + std::to_string(major) + std::to_string(minor) +
                             "a, tcgen05 3xTF32 mul_mat, device dequant)";
        props_.type           = DeviceType::GPU;
        props_.unified_memory = false;
        refresh_memory();
    }

    const DeviceProps& props() const override {
        const_cast<CudaDevice*>(this)->refresh_memory();
        return props_;
    }
    BufferType* default_buffer_type() override { return &buft_; }

    bool supports_op(const Tensor* t) const override {
        if (t == nullptr) return false;
        const int reads_packed = packed_reads(t);
        if (reads_packed < 0) return false;
        if (reads_packed > 0) return t->op == OP_MUL_MAT && all_f32(t);  // the dequant-in-prologue GEMM
        switch (t->op) {
            case OP_NONE:
            case OP_RESHAPE:
            case OP_VIEW:
            case OP_PERMUTE:
            case OP_TRANSPOSE:
                return true;  // leaves and views: nothing to compute
            case OP_MUL_MAT:
            case OP_SUM:
            case OP_REPEAT:
            case OP_ACC:
                return all_f32(t);
            case OP_CONT:
            case OP_DUP:
                return all_f32(t);
            case OP_REPEAT_BACK:
                return all_f32(t) && tensor_is_contiguous(t);
            case OP_ADD:
            case OP_SUB:
            case OP_MUL:
            case OP_DIV:
                return all_f32(t) && t->src[1] != nullptr && tensor_can_repeat(t->src[1], t->src[0]);
            case OP_SQR:
            case OP_SQRT:
            case OP_ABS:
            case OP_NEG:
            case OP_SGN:
            case OP_STEP:
            case OP_SCALE:
                return all_f32(t) && t->src[0] != nullptr && tensor_are_same_shape(t, t->src[0]);
            case OP_SUM_ROWS:
            case OP_MEAN:
                return all_f32(t) && t->src[0] != nullptr;
            case OP_OPT_STEP_ADAMW:
            case OP_OPT_STEP_SGD: {
                // the optimizer graph's nodes (src/optim/trc_optim.cpp:372-388): flat in-place updates
                const int nstate = t->op == OP_OPT_STEP_ADAMW ? 4 : 3;
                if (!all_f32(t)) return false;
                for (int i = 0; i < nstate; ++i) {
                    const Tensor* s = t->src[i];
                    if (s == nullptr || !tensor_is_contiguous(s) ||
                        tensor_nelements(s) != tensor_nelements(t->src[0]))
                        return false;
                }
                return true;
            }
            case OP_SUM_SQR_ACC:
                return all_f32(t) && t->src[1] != nullptr && tensor_is_contiguous(t->src[1]);
            case OP_CLIP_SCALE_INPLACE:
                return all_f32(t) && t->src[0] != nullptr && tensor_is_contiguous(t->src[0]);
            default:
                return false;
        }
    }

    bool graph_compute(Graph* graph) override {
        if (graph == nullptr) CB_ABORT("CudaDevice::graph_compute: graph 为空");
        CB_CUDA(trc_cuda_rt_set_device(ordinal_));
        plan_fusions(graph);
        for (Tensor* node : graph->nodes) compute_node(node);
        CB_CUDA(trc_cuda_rt_stream_sync(stream_));
        int code = 0;
        CB_TRC(trc_cuda_device_error(&code, 1), "trc_cuda_device_error");
        if (code != 0) CB_ABORT("CUDA: kernel 等待超时（设备错误码 %d），结果无效", code);
        return true;
    }

    bool fill_tensors(const TensorFill* fills, size_t count) override {
        CB_CUDA(trc_cuda_rt_set_device(ordinal_));
        for (size_t i = 0; i < count; ++i) {
            Tensor* t = fills[i].tensor;
            if (t == nullptr || t->type != TYPE_F32 || !tensor_is_contiguous(t))
                CB_ABORT("fill_tensors: 仅支持连续 F32 张量");
            const trc_cuda_view v = view_of(t);
            CB_TRC(trc_cuda_fill(static_cast<float*>(v.data), tensor_nelements(t), fills[i].value, stream_),
                   "trc_cuda_fill");
        }
        CB_CUDA(trc_cuda_rt_stream_sync(stream_));
        return true;
    }

    int          ordinal() const { return ordinal_; }
    void*        stream() const { return stream_; }
    BufferType*  packed_buffer_type() { return &packed_buft_; }

    // Device scratch, grown on demand (sum partials, GGUF staging). Stream-ordered use only.
    void* scratch(size_t bytes) {
        if (bytes > scratch_bytes_) {
            CB_CUDA(trc_cuda_rt_stream_sync(stream_));
            if (scratch_ != nullptr) CB_CUDA(trc_cuda_rt_free(scratch_));
            scratch_ = nullptr;
            scratch_bytes_ = 0;
            CB_CUDA(trc_cuda_rt_malloc(&scratch_, bytes));
            scratch_bytes_ = bytes;
        }
        return scratch_;
    }

    // Two pinned chunks and their events for the staged tensor copies (created on first use, kept
    // for the device's lifetime).
    struct CopyRing {
        void* host[2] = {nullptr, nullptr};
        void* done[2] = {nullptr, nullptr};
    };
    CopyRing& copy_ring() {
        if (ring_.host[0] == nullptr) {
            for (int k = 0; k < 2; ++k) {
                CB_CUDA(trc_cuda_rt_malloc_host(&ring_.host[k], kStagedChunk));
                CB_CUDA(trc_cuda_rt_event_create(&ring_.done[k]));
            }
        }
        return ring_;
    }

    // Pinned host staging for the single-tensor GGUF loader, grown on demand and kept for the
    // device's lifetime (page-locking is a system call; a warm start loads hundreds of tensors).
    // The caller synchronizes the stream before the next use.
    void* pinned(size_t bytes) {
        if (bytes > pinned_bytes_) {
            CB_CUDA(trc_cuda_rt_stream_sync(stream_));
            if (pinned_ != nullptr) CB_CUDA(trc_cuda_rt_free_host(pinned_));
            pinned_ = nullptr;
            pinned_bytes_ = 0;
            CB_CUDA(trc_cuda_rt_malloc_host(&pinned_, bytes));
            pinned_bytes_ = bytes;
        }
        return pinned_;
    }

private:
    void refresh_memory() {
        size_t free_b = 0, total_b = 0;
        int prev = 0;
        trc_cuda_rt_get_device(&prev);
        if (trc_cuda_rt_set_device(ordinal_) == TRC_CUDA_OK && trc_cuda_rt_mem_info(&free_b, &total_b) == TRC_CUDA_OK) {
            props_.memory_free  = free_b;
            props_.memory_total = total_b;
        }
        trc_cuda_rt_set_device(prev);
    }

    // Whether node t reads a packed weight: 0 no; 1 as the first operand of a mul_mat in one of the
    // two forms the dequant-in-prologue GEMM takes (W, or transpose(W)) with an ordinary second
    // operand; -1 in any other way (no kernel of this device reads it so), or t itself lives on a
    // packed buffer. Views of a packed weight compute nothing and count as 0.
    static int packed_reads(const Tensor* t) {
        switch (t->op) {
            case OP_NONE:
            case OP_RESHAPE:
            case OP_VIEW:
            case OP_PERMUTE:
            case OP_TRANSPOSE:
                return 0;
            default:
                break;
        }
        if (packed_buffer_of(t) != nullptr) return -1;
        int found = 0;
        for (int i = 0; i < t->nsrc; ++i) {
            const PackedUse u = packed_use(t->src[i], nullptr);
            if (u == PackedUse::none) continue;
            if (t->op != OP_MUL_MAT || i != 0 || u == PackedUse::unsupported) return -1;
            found = 1;
        }
        return found;
    }

    // ---------------------------------------------------------------- graph-level fusion
    // The composed backward (src/core/trc_autograd.cpp:60-77, 487-503) materialises intermediates
    // that the GEMM can write or accumulate directly when nothing else reads them:
    //   dW:  mul_mat M -> permute P -> cont C -> acc(inplace, whole grad_acc)   => GEMM into T(grad_acc), +=
    //   dB:  mul_mat M -> acc(inplace, whole grad_acc)                          => GEMM into grad_acc, +=
    //   dA of a broadcast operand:
    //        mul_mat M -> permute P -> repeat_back R -> acc(inplace, grad_acc)  => plane-reducing GEMM into
    //                                                                              T(grad_acc), +=
    //        mul_mat M -> permute P -> repeat_back R (other readers)           => plane-reducing GEMM into T(R)
    // Every output element still receives one fp32 add from the fused acc, as in the unfused graph.
    // TRC_CUDA_NO_FUSION=1 executes every node as written.
    struct Fused {
        const Tensor* target;      // tensor the GEMM writes (grad_acc, or the repeat_back output)
        bool          transposed;  // write through the transposed view of target
        bool          reduce;      // sum broadcast planes (repeat_back) in the GEMM
        bool          accumulate;  // target += product
    };
    std::unordered_map<const Tensor*, Fused> fused_gemm_;  // mul_mat node -> fusion
    std::unordered_map<const Tensor*, bool>  skipped_;     // nodes whose work the fused GEMM does

    void plan_fusions(Graph* g) {
        fused_gemm_.clear();
        skipped_.clear();
        const char* off = std::getenv("TRC_CUDA_NO_FUSION");
        if (off != nullptr && off[0] == '1') return;
        std::unordered_map<const Tensor*, int> readers;
        for (Tensor* n : g->nodes)
            for (int i = 0; i < n->nsrc; ++i)
                if (n->src[i] != nullptr) readers[n->src[i]]++;
        auto private_to = [&](const Tensor* t) {
            return readers[t] == 1 && (t->flags & (TENSOR_FLAG_OUTPUT | TENSOR_FLAG_PARAM | TENSOR_FLAG_LOSS)) == 0;
        };
        auto is_transpose_of_private_mul_mat = [&](const Tensor* P) {
            if (P == nullptr || P->op != OP_PERMUTE || !private_to(P)) return false;
            const int* ax = P->op_params;
            const Tensor* M = P->src[0];
            return ax[0] == 1 && ax[1] == 0 && ax[2] == 2 && ax[3] == 3 && M != nullptr && M->op == OP_MUL_MAT &&
                   private_to(M) && fused_gemm_.count(M) == 0;
        };
        for (Tensor* n : g->nodes) {
            if (n->op == OP_ACC && n->nsrc >= 2 && n->op_params[4] != 0) {  // in-place acc into a whole tensor
                const Tensor* G = n->src[0];
                const Tensor* C = n->src[1];
                if (!tensor_is_contiguous(G) || !tensor_are_same_shape(G, C) || n->op_params[3] != 0) continue;
                if (static_cast<size_t>(n->op_params[0]) != G->nb[1] || static_cast<size_t>(n->op_params[1]) != G->nb[2] ||
                    static_cast<size_t>(n->op_params[2]) != G->nb[3])
                    continue;
                if (C->op == OP_MUL_MAT && private_to(C) && fused_gemm_.count(C) == 0) {
                    fused_gemm_[C] = {G, false, false, true};
                    skipped_[n]    = true;
                } else if ((C->op == OP_CONT || C->op == OP_REPEAT_BACK) && private_to(C) &&
                           is_transpose_of_private_mul_mat(C->src[0])) {
                    fused_gemm_[C->src[0]->src[0]] = {G, true, C->op == OP_REPEAT_BACK, true};
                    skipped_[C] = true;
                    skipped_[n] = true;
                }
            }
        }
        // second pass: a repeat_back whose consumer is not a fusable acc is written by the GEMM directly
        for (Tensor* n : g->nodes) {
            if (n->op == OP_REPEAT_BACK && skipped_.count(n) == 0 && tensor_is_contiguous(n) &&
                is_transpose_of_private_mul_mat(n->src[0])) {
                fused_gemm_[n->src[0]->src[0]] = {n, true, true, false};
                skipped_[n] = true;
            }
        }
    }

    // ---------------------------------------------------------------- per-node execution
    void compute_node(Tensor* t) {
        if (skipped_.count(t) != 0) return;
        const int reads_packed = packed_reads(t);
        if (reads_packed < 0)
            CB_ABORT("CUDA: 算子 %s（张量 %s）不能读取冻结的量化权重：只有 mul_mat(W, x) 与 "
                     "mul_mat(transpose(W), g) 支持；请先用 graph_first_unsupported 预检", op_name(t->op), t->name);
        if (reads_packed > 0) {
            compute_packed_mul_mat(t);
            return;
        }
        switch (t->op) {
            case OP_NONE:
            case OP_RESHAPE:
            case OP_VIEW:
            case OP_PERMUTE:
            case OP_TRANSPOSE:
                return;
            case OP_MUL_MAT: {
                const trc_cuda_view a = view_of(t->src[0]), b = view_of(t->src[1]);
                const auto it = fused_gemm_.find(t);
                if (it == fused_gemm_.end()) {
                    const trc_cuda_view d = view_of(t);
                    CB_TRC(trc_cuda_mul_mat(&a, &b, &d, mm_flags(), stream_), "trc_cuda_mul_mat");
                } else {
                    const Fused& f = it->second;
                    trc_cuda_view d = view_of(f.target);
                    if (f.transposed) {  // D[i, j] lands on target[j, i]
                        std::swap(d.ne[0], d.ne[1]);
                        std::swap(d.nb[0], d.nb[1]);
                    }
                    const uint32_t flags = (f.accumulate ? TRC_CUDA_MM_ACCUMULATE : 0u) | mm_flags();
                    if (f.reduce)
                        CB_TRC(trc_cuda_mul_mat_repeat_back(&a, &b, &d, flags, stream_), "trc_cuda_mul_mat_repeat_back (fused)");
                    else
                        CB_TRC(trc_cuda_mul_mat(&a, &b, &d, flags, stream_), "trc_cuda_mul_mat (fused)");
                }
                return;
            }
            case OP_ADD:
            case OP_SUB:
            case OP_MUL:
            case OP_DIV: {
                const int op = t->op == OP_ADD ? TRC_CUDA_BIN_ADD
                             : t->op == OP_SUB ? TRC_CUDA_BIN_SUB
                             : t->op == OP_MUL ? TRC_CUDA_BIN_MUL
                                               : TRC_CUDA_BIN_DIV;
                const trc_cuda_view a = view_of(t->src[0]), b = view_of(t->src[1]), d = view_of(t);
                CB_TRC(trc_cuda_binary(op, &a, &b, &d, stream_), "trc_cuda_binary");
                return;
            }
            case OP_SUM: {
                const trc_cuda_view a = view_of(t->src[0]), d = view_of(t);
                const size_t ws = trc_cuda_sum_workspace_bytes(tensor_nelements(t->src[0]));
                CB_TRC(trc_cuda_sum(&a, static_cast<float*>(d.data), scratch(ws), ws, stream_), "trc_cuda_sum");
                return;
            }
            case OP_REPEAT: {
                const trc_cuda_view a = view_of(t->src[0]), d = view_of(t);
                CB_TRC(trc_cuda_repeat(&a, &d, stream_), "trc_cuda_repeat");
                return;
            }
            case OP_REPEAT_BACK: {
                const trc_cuda_view a = view_of(t->src[0]), d = view_of(t);
                CB_TRC(trc_cuda_repeat_back(&a, &d, stream_), "trc_cuda_repeat_back");
                return;
            }
            case OP_CONT:
            case OP_DUP: {
                const trc_cuda_view a = view_of(t->src[0]), d = view_of(t);
                CB_TRC(trc_cuda_cont(&a, &d, stream_), "trc_cuda_cont");
                return;
            }
            case OP_ACC: {
                // op_params: int32 nb1, nb2, nb3, offset, inplace (src/core/trc_tensor.cpp:353-358)
                const int32_t* p = t->op_params;
                const trc_cuda_view b = view_of(t->src[1]);
                const trc_cuda_view d = view_of(t);
                if (p[4] == 0) {  // not in place: dst = a, then the region += b
                    const trc_cuda_view a = view_of(t->src[0]);
                    CB_TRC(trc_cuda_cont(&a, &d, stream_), "trc_cuda_cont (acc copy)");
                }
                CB_TRC(trc_cuda_acc(d.data, static_cast<int64_t>(tensor_nbytes(t)), &b, p[0], p[1], p[2], p[3], stream_),
                       "trc_cuda_acc");
                return;
            }
            case OP_SQR:
            case OP_SQRT:
            case OP_ABS:
            case OP_NEG:
            case OP_SGN:
            case OP_STEP:
            case OP_SCALE: {
                const int op = t->op == OP_SQR    ? TRC_CUDA_UNARY_SQR
                             : t->op == OP_SQRT   ? TRC_CUDA_UNARY_SQRT
                             : t->op == OP_ABS    ? TRC_CUDA_UNARY_ABS
                             : t->op == OP_NEG    ? TRC_CUDA_UNARY_NEG
                             : t->op == OP_SGN    ? TRC_CUDA_UNARY_SGN
                             : t->op == OP_STEP   ? TRC_CUDA_UNARY_STEP
                                                  : TRC_CUDA_UNARY_SCALE;
                float param = 0.0f;
                if (t->op == OP_SCALE) std::memcpy(&param, t->op_params, sizeof(float));  // src/ops/trc_ops.cpp:113
                const trc_cuda_view a = view_of(t->src[0]), d = view_of(t);
                CB_TRC(trc_cuda_unary(op, &a, &d, param, stream_), "trc_cuda_unary");
                return;
            }
            case OP_SUM_ROWS:
            case OP_MEAN: {
                const trc_cuda_view a = view_of(t->src[0]), d = view_of(t);
                CB_TRC(trc_cuda_sum_rows(&a, &d, t->op == OP_MEAN ? 1 : 0, stream_), "trc_cuda_sum_rows");
                return;
            }
            case OP_OPT_STEP_ADAMW:
            case OP_OPT_STEP_SGD: {
                // the node is a full view of the parameter; op_params float[6] (src/ops/trc_ops.cpp:792-811)
                float ps[6];
                std::memcpy(ps, t->op_params, sizeof(ps));
                float* p = static_cast<float*>(view_of(t).data);
                const float* g = static_cast<const float*>(view_of(t->src[1]).data);
                float* m = static_cast<float*>(view_of(t->src[2]).data);
                const int64_t n = tensor_nelements(t->src[0]);
                if (t->op == OP_OPT_STEP_ADAMW) {
                    float* v = static_cast<float*>(view_of(t->src[3]).data);
                    CB_TRC(trc_cuda_opt_step_adamw(p, g, m, v, n, ps, stream_), "trc_cuda_opt_step_adamw");
                } else {
                    CB_TRC(trc_cuda_opt_step_sgd(p, g, m, n, ps, stream_), "trc_cuda_opt_step_sgd");
                }
                return;
            }
            case OP_SUM_SQR_ACC: {
                // the node is a full view of the one-element accumulator (src/ops/trc_ops.cpp:815-828)
                float* acc = static_cast<float*>(view_of(t).data);
                const Tensor* a = t->src[1];
                const int64_t n = tensor_nelements(a);
                const size_t ws = trc_cuda_sum_sqr_workspace_bytes(n);
                CB_TRC(trc_cuda_sum_sqr_acc(acc, static_cast<const float*>(view_of(a).data), n, scratch(ws), ws, stream_),
                       "trc_cuda_sum_sqr_acc");
                return;
            }
            case OP_CLIP_SCALE_INPLACE: {
                float ps[2];  // max_norm, eps (src/ops/trc_ops.cpp:830-844)
                std::memcpy(ps, t->op_params, sizeof(ps));
                float* a = static_cast<float*>(view_of(t).data);
                const float* norm = static_cast<const float*>(view_of(t->src[1]).data);
                CB_TRC(trc_cuda_clip_scale_inplace(a, tensor_nelements(t->src[0]), norm, ps[0], ps[1], stream_),
                       "trc_cuda_clip_scale_inplace");
                return;
            }
            default:
                CB_ABORT("CUDA: 不支持的算子 %s（张量 %s）；请先用 graph_first_unsupported 预检", op_name(t->op),
                         t->name);
        }
    }

    // mul_mat whose first operand is a packed weight W or transpose(W): the dequant-in-prologue GEMM
    // (trc_cuda_mul_mat_q with TRC_CUDA_MM_FUSED), which decodes W's blocks inside the GEMM and
    // writes no F32 copy of W. The graph-level fusion into grad_acc (dX of a parameter input)
    // applies as for any mul_mat. Views the tensor-core kernel cannot address fall back to the
    // dequant + SIMT kernel (W dequantized into stream-ordered scratch for that one product).
    void compute_packed_mul_mat(Tensor* t) {
        const PackedWeight* w = nullptr;
        const PackedUse u = packed_use(t->src[0], &w);
        if (w == nullptr)
            CB_ABORT("CUDA: 冻结的量化权重 %s 尚未载入（cuda_gguf_load_tensor / cuda_set_tensor_from_quant）",
                     view_root(t->src[0])->name);
        const trc_cuda_view b = view_of(t->src[1]);
        trc_cuda_view d;
        uint32_t flags = mm_flags();
        const auto it = fused_gemm_.find(t);
        if (it == fused_gemm_.end()) {
            d = view_of(t);
        } else {
            const Fused& f = it->second;
            if (f.reduce) CB_ABORT("CUDA: 量化权重不会作为广播操作数（张量 %s）", t->name);
            d = view_of(f.target);
            if (f.transposed) {
                std::swap(d.ne[0], d.ne[1]);
                std::swap(d.nb[0], d.nb[1]);
            }
            if (f.accumulate) flags |= TRC_CUDA_MM_ACCUMULATE;
        }
        if ((flags & TRC_CUDA_MM_SIMT) == 0) flags |= packed_two_step() ? TRC_CUDA_MM_TWO_STEP : TRC_CUDA_MM_FUSED;
        const int tr = u == PackedUse::transposed ? 1 : 0;
        int st = trc_cuda_mul_mat_q(static_cast<int>(w->type), w->blocks, w->ne0, w->ne1, tr, &b, &d, flags, stream_);
        if (st == TRC_CUDA_EUNSUPPORTED)  // a view TMA cannot address: dequant + the SIMT kernel
            st = trc_cuda_mul_mat_q(static_cast<int>(w->type), w->blocks, w->ne0, w->ne1, tr, &b, &d,
                                    (flags & ~static_cast<uint32_t>(TRC_CUDA_MM_FUSED)) | TRC_CUDA_MM_SIMT, stream_);
        CB_TRC(st, "trc_cuda_mul_mat_q (packed weight)");
    }

    // TRC_CUDA_PACKED_TWO_STEP=1: packed weights take mul_mat_q's two-step path (W dequantized into
    // scratch for one product; same bits); by default no F32 copy of W is ever written.
    static bool packed_two_step() {
        static const bool on = [] {
            const char* e = std::getenv("TRC_CUDA_PACKED_TWO_STEP");
            return e != nullptr && *e != '\0' && *e != '0';
        }();
        return on;
    }

    // TRC_CUDA_MM_SIMT=1 runs every mul_mat on the SIMT kernel, which sums in the reference's order,
    // so whole training runs can be compared bit for bit with the CPU device.
    static uint32_t mm_flags() {
        static const uint32_t flags = [] {
            const char* e = std::getenv("TRC_CUDA_MM_SIMT");
            return (e != nullptr && *e != '\0' && *e != '0') ? static_cast<uint32_t>(TRC_CUDA_MM_SIMT) : 0u;
        }();
        return flags;
    }

    int            ordinal_;
    CudaBufferType buft_;
    CudaPackedBufferType packed_buft_;
    DeviceProps    props_;
    void*          stream_ = nullptr;
    void*          scratch_ = nullptr;
    size_t         scratch_bytes_ = 0;
    void*          pinned_ = nullptr;
    size_t         pinned_bytes_ = 0;
    CopyRing       ring_;
};

Device* CudaBufferType::device() const { return dev_; }

Buffer* CudaBufferType::alloc_buffer(size_t size) {
    if (fake_alloc_failure()) return nullptr;
    const int ordinal = static_cast<CudaDevice*>(dev_)->ordinal();
    if (trc_cuda_rt_set_device(ordinal) != TRC_CUDA_OK) return nullptr;
    void* p = nullptr;
    if (trc_cuda_rt_malloc(&p, size) != TRC_CUDA_OK) return nullptr;
    return new CudaBuffer(this, ordinal, static_cast<char*>(p), size);
}

CudaDevice* CudaBuffer::device_of() const { return static_cast<CudaDevice*>(buft_->device()); }

// Host memcpy on several threads: one host thread copies about 10 GB/s, the pinned DMA it feeds
// runs at 40-55 GB/s. A small pool of worker threads, created on first use, splits each copy into
// slices; the calling thread copies one slice itself and waits for the rest.
class CopyPool {
public:
    // Never destroyed: its workers wait on its condition variable for the life of the process, and
    // destroying a condition variable that threads still wait on blocks (glibc) at exit.
    static CopyPool& get() {
        static CopyPool* pool = new CopyPool;
        return *pool;
    }
    void copy(void* dst, const void* src, size_t bytes) {
        const size_t slices = std::min<size_t>(workers_.size() + 1, std::max<size_t>(1, bytes / (size_t(1) << 20)));
        if (slices <= 1) {
            std::memcpy(dst, src, bytes);
            return;
        }
        const size_t per = (bytes + slices - 1) / slices;
        std::lock_guard<std::mutex> one_job(job_mu_);  // callers on several threads take turns
        {
            std::lock_guard<std::mutex> lock(mu_);
            dst_ = static_cast<char*>(dst);
            src_ = static_cast<const char*>(src);
            bytes_ = bytes;
            per_ = per;
            next_ = 1;  // slice 0 is the caller's
            total_ = slices;
            pending_ = slices - 1;
            ++generation_;
        }
        cv_.notify_all();
        std::memcpy(dst, src, std::min(per, bytes));
        std::unique_lock<std::mutex> lock(mu_);
        done_cv_.wait(lock, [&] { return pending_ == 0; });
    }

private:
    CopyPool() {
        const unsigned hw = std::thread::hardware_concurrency();
        const unsigned n = std::max(1u, std::min(7u, hw > 1 ? hw - 1 : 1u));
        for (unsigned i = 0; i < n; ++i) workers_.emplace_back([this] { run(); });
        for (auto& w : workers_) w.detach();  // process-lifetime workers
    }
    void run() {
        uint64_t seen = 0;
        for (;;) {
            std::unique_lock<std::mutex> lock(mu_);
            cv_.wait(lock, [&] { return generation_ != seen && next_ < total_; });
            const size_t i = next_++;
            if (next_ >= total_) seen = generation_;
            char* d = dst_;
            const char* s = src_;
            const size_t off = i * per_, len = std::min(per_, bytes_ - std::min(bytes_, off));
            lock.unlock();
            if (len > 0) std::memcpy(d + off, s + off, len);
            lock.lock();
            if (--pending_ == 0) done_cv_.notify_one();
        }
    }
    std::mutex job_mu_, mu_;
    std::condition_variable cv_, done_cv_;
    std::vector<std::thread> workers_;
    char* dst_ = nullptr;
    const char* src_ = nullptr;
    size_t bytes_ = 0, per_ = 0, next_ = 0, total_ = 0, pending_ = 0;
    uint64_t generation_ = 0;
};

void staged_h2d(CudaDevice* dev, void* dst, const void* src, size_t bytes) {
    CudaDevice::CopyRing& r = dev->copy_ring();
    const char* s = static_cast<const char*>(src);
    char*       d = static_cast<char*>(dst);
    size_t c = 0;
    for (size_t off = 0; off < bytes; off += kStagedChunk, ++c) {
        const int    k   = static_cast<int>(c & 1u);
        const size_t len = std::min(kStagedChunk, bytes - off);
        if (c >= 2) CB_CUDA(trc_cuda_rt_event_sync(r.done[k]));  // the DMA that read chunk k finished
        CopyPool::get().copy(r.host[k], s + off, len);
        CB_CUDA(trc_cuda_rt_memcpy_async(d + off, r.host[k], len, 0, dev->stream()));
        CB_CUDA(trc_cuda_rt_event_record(r.done[k], dev->stream()));
    }
    CB_CUDA(trc_cuda_rt_stream_sync(dev->stream()));
}

void staged_d2h(CudaDevice* dev, void* dst, const void* src, size_t bytes) {
    CudaDevice::CopyRing& r = dev->copy_ring();
    const char* s = static_cast<const char*>(src);
    char*       d = static_cast<char*>(dst);
    const size_t n = (bytes + kStagedChunk - 1) / kStagedChunk;
    auto issue = [&](size_t c) {
        const int    k   = static_cast<int>(c & 1u);
        const size_t off = c * kStagedChunk;
        CB_CUDA(trc_cuda_rt_memcpy_async(r.host[k], s + off, std::min(kStagedChunk, bytes - off), 1, dev->stream()));
        CB_CUDA(trc_cuda_rt_event_record(r.done[k], dev->stream()));
    };
    issue(0);
    for (size_t c = 0; c < n; ++c) {
        if (c + 1 < n) issue(c + 1);  // its chunk's previous contents were copied out in step c - 1
        const int    k   = static_cast<int>(c & 1u);
        const size_t off = c * kStagedChunk;
        CB_CUDA(trc_cuda_rt_event_sync(r.done[k]));
        CopyPool::get().copy(d + off, r.host[k], std::min(kStagedChunk, bytes - off));
    }
}

Device* CudaPackedBufferType::device() const { return dev_; }

Buffer* CudaPackedBufferType::alloc_buffer(size_t size) {
    if (fake_alloc_failure()) return nullptr;
    return new CudaPackedBuffer(this, size);
}

bool CudaPackedBuffer::store(Tensor* t, Type type, const void* host, size_t bytes) {
    const size_t bb = trc_cuda_block_bytes(static_cast<int>(type));
    if (t->buffer != this || t->view_src != nullptr) CB_ABORT("%s: 张量 %s 不是本 buffer 的根张量", buft_->name(), t->name);
    if (bb == 0 || t->type != TYPE_F32 || !tensor_is_contiguous(t) || t->ne[2] != 1 || t->ne[3] != 1 ||
        t->ne[0] % 32 != 0) {
        std::fprintf(stderr, "[traincpp] %s: 张量 %s 须为二维连续 F32（ne0 为 32 的倍数），数据须为 Q4_0/Q4_1/Q5_0/Q5_1/Q8_0\n",
                     buft_->name(), t->name);
        return false;
    }
    if (static_cast<size_t>(tensor_nelements(t) / 32) * bb != bytes) {
        std::fprintf(stderr, "[traincpp] %s: 张量 %s 的量化块字节数不符（%zu）\n", buft_->name(), t->name, bytes);
        return false;
    }
    std::unique_ptr<PackedWeight>& slot = weights_[t];
    if (!slot) slot = std::make_unique<PackedWeight>();
    PackedWeight& w = *slot;
    CB_CUDA(trc_cuda_rt_set_device(buft_->ordinal()));
    const size_t want = (bytes + 255) / 256 * 256;
    if (w.capacity < want) {
        if (w.blocks != nullptr) CB_CUDA(trc_cuda_rt_free(w.blocks));
        w.blocks = nullptr;
        w.capacity = 0;
        const int st = trc_cuda_rt_malloc(&w.blocks, want);
        if (st != TRC_CUDA_OK) {
            std::fprintf(stderr, "[traincpp] %s: 量化块显存分配失败（%zu 字节）\n", buft_->name(), want);
            return false;
        }
        w.capacity = want;
    }
    CB_CUDA(trc_cuda_rt_memcpy(w.blocks, host, bytes, 0));
    w.owner = this;
    w.type = type;
    w.ne0 = t->ne[0];
    w.ne1 = t->ne[1];
    w.bytes = bytes;
    t->extra = &w;
    return true;
}

void CudaPackedBuffer::get_tensor(const Tensor* t, size_t offset, void* data, size_t size) const {
    const Tensor* r = view_root(t);
    const PackedWeight* w = weight_of(r);
    if (w == nullptr) CB_ABORT("%s: 张量 %s 尚未载入量化块", buft_->name(), r->name);
    // the bytes asked for, as positions in the root's F32 layout (views address the root's bytes)
    const size_t pos = t->data_offset - r->data_offset + offset;
    if (pos + size > tensor_nbytes(r)) CB_ABORT("%s::get_tensor: 越界", buft_->name());
    if (size == 0) return;
    const int64_t b0 = static_cast<int64_t>(pos / 128), b1 = static_cast<int64_t>((pos + size + 127) / 128);
    CudaDevice* dev = buft_->cuda_device();
    CB_CUDA(trc_cuda_rt_set_device(buft_->ordinal()));
    const size_t bb = trc_cuda_block_bytes(static_cast<int>(w->type));
    float* tmp = static_cast<float*>(dev->scratch(static_cast<size_t>(b1 - b0) * 128));
    CB_TRC(trc_cuda_dequant(static_cast<int>(w->type), static_cast<const uint8_t*>(w->blocks) + b0 * bb, b1 - b0, tmp,
                            dev->stream()),
           "trc_cuda_dequant (tensor_get of a packed weight)");
    CB_CUDA(trc_cuda_rt_stream_sync(dev->stream()));
    CB_CUDA(trc_cuda_rt_memcpy(data, reinterpret_cast<const char*>(tmp) + (pos - static_cast<size_t>(b0) * 128), size, 1));
}

void CudaPackedBuffer::clear() {
    CB_CUDA(trc_cuda_rt_set_device(buft_->ordinal()));
    for (auto& kv : weights_)  // all-zero blocks decode to 0.0f (scale 0)
        if (kv.second->blocks != nullptr) CB_CUDA(trc_cuda_rt_memset(kv.second->blocks, 0, kv.second->bytes));
}

std::mutex& registry_mutex() {
    static std::mutex mu;
    return mu;
}

std::vector<std::unique_ptr<CudaDevice>>& devices() {
    static std::vector<std::unique_ptr<CudaDevice>> d;
    return d;
}

bool is_legacy_quant(Type t) {
    return t == TYPE_Q4_0 || t == TYPE_Q4_1 || t == TYPE_Q5_0 || t == TYPE_Q5_1 || t == TYPE_Q8_0;
}

}  // namespace

int cuda_device_count() {
    int n = 0;
    if (trc_cuda_rt_device_count(&n) != TRC_CUDA_OK) return 0;
    return n;
}

Device* cuda_device(int ordinal) {
    std::lock_guard<std::mutex> lock(registry_mutex());
    const int n = cuda_device_count();
    if (ordinal < 0 || ordinal >= n) return nullptr;
    auto& d = devices();
    if (d.size() < static_cast<size_t>(n)) d.resize(static_cast<size_t>(n));
    if (!d[ordinal]) d[ordinal] = std::make_unique<CudaDevice>(ordinal);
    return d[ordinal].get();
}

int cuda_register_devices() {
    static std::mutex mu;
    static int        registered = -1;
    std::lock_guard<std::mutex> lock(mu);
    if (registered >= 0) return registered;
    registered = 0;
    for (int i = 0; i < cuda_device_count(); ++i) {
        if (Device* d = cuda_device(i)) {
            backend_register_device(d);
            ++registered;
        }
    }
    return registered;
}

BufferType* cuda_packed_buffer_type(int ordinal) {
    Device* d = cuda_device(ordinal);
    return d == nullptr ? nullptr : static_cast<CudaDevice*>(d)->packed_buffer_type();
}

bool cuda_tensor_is_packed(const Tensor* t) { return packed_buffer_of(t) != nullptr; }

bool cuda_set_tensor_from_quant(Tensor* dst, Type type, const void* packed, size_t bytes) {
    if (dst == nullptr || (packed == nullptr && bytes != 0)) CB_ABORT("cuda_set_tensor_from_quant: 参数为空");
    if (CudaPackedBuffer* pb = packed_buffer_of(dst)) {
        if (dst->view_src != nullptr) {
            std::fprintf(stderr, "[traincpp] cuda_set_tensor_from_quant: 量化权重 %s 须按根张量载入\n", dst->name);
            return false;
        }
        return pb->store(dst, type, packed, bytes);
    }
    CudaBuffer* buf = cuda_buffer_of(dst);
    const size_t bb = trc_cuda_block_bytes(static_cast<int>(type));
    if (buf == nullptr || bb == 0 || dst->type != TYPE_F32 || !tensor_is_contiguous(dst) ||
        tensor_nelements(dst) % 32 != 0 || static_cast<size_t>(tensor_nelements(dst) / 32) * bb != bytes) {
        std::fprintf(stderr, "[traincpp] cuda_set_tensor_from_quant: 张量 %s 须为 CUDA 上的连续 F32 张量，"
                     "数据须为与元素数一致的 Q4_0/Q4_1/Q5_0/Q5_1/Q8_0 块\n", dst->name);
        return false;
    }
    if (bytes == 0) return true;
    CB_CUDA(trc_cuda_rt_set_device(buf->ordinal()));
    CudaDevice* dev = static_cast<CudaDevice*>(buf->buffer_type()->device());
    void* staging = dev->scratch((bytes + 15) / 16 * 16);
    float* out = reinterpret_cast<float*>(buf->device_ptr() + dst->data_offset);
    CB_TRC(trc_cuda_load_quant(static_cast<int>(type), packed, tensor_nelements(dst) / 32, staging, out, dev->stream()),
           "trc_cuda_load_quant");
    CB_CUDA(trc_cuda_rt_stream_sync(dev->stream()));
    int code = 0;
    CB_TRC(trc_cuda_device_error(&code, 1), "trc_cuda_device_error");
    if (code != 0) CB_ABORT("CUDA: dequant kernel 等待超时（设备错误码 %d）", code);
    return true;
}

bool cuda_gguf_load_tensor(const GgufFile* f, const char* path, const char* name, Tensor* dst) {
    if (f == nullptr || path == nullptr || name == nullptr || dst == nullptr)
        CB_ABORT("cuda_gguf_load_tensor: 参数为空");
    const int64_t ti = gguf_find_tensor(f, name);
    if (ti < 0) {
        std::fprintf(stderr, "[traincpp] GGUF: 张量不存在 %s\n", name);
        return false;
    }
    const GgufTensorInfo* info = gguf_tensor_info(f, ti);
    CudaBuffer* buf = cuda_buffer_of(dst);
    CudaPackedBuffer* pbuf = packed_buffer_of(dst);
    if (pbuf != nullptr && !is_legacy_quant(info->type)) {
        std::fprintf(stderr, "[traincpp] GGUF: 张量 %s 的类型 %s 不能载入量化权重 buffer\n", name, type_name(info->type));
        return false;
    }
    if (pbuf == nullptr && (!is_legacy_quant(info->type) || dst->type != TYPE_F32 || buf == nullptr))
        return gguf_load_tensor(f, name, dst);  // the reference path (also reports its errors)
    // the reference's destination checks (src/io/trc_gguf.cpp:1060-1076)
    if (!tensor_is_contiguous(dst)) {
        std::fprintf(stderr, "[traincpp] GGUF: 目标张量 %s 必须连续\n", name);
        return false;
    }
    if (tensor_nelements(dst) != gguf_tensor_nelements(f, ti)) {
        std::fprintf(stderr, "[traincpp] GGUF: 张量 %s 元素数不匹配\n", name);
        return false;
    }
    const int64_t n_blocks = gguf_tensor_nelements(f, ti) / 32;
    const size_t  bytes    = info->nbytes;
    FILE* fp = std::fopen(path, "rb");
    if (fp == nullptr) {
        std::fprintf(stderr, "[traincpp] GGUF: 无法打开 %s\n", path);
        return false;
    }
    CudaDevice* dev = static_cast<CudaDevice*>(pbuf != nullptr ? pbuf->buffer_type()->device()
                                                               : buf->buffer_type()->device());
    CB_CUDA(trc_cuda_rt_set_device(dev->ordinal()));
    void* host = dev->pinned(bytes);  // reused across calls: no page-locking per tensor
    const long pos = static_cast<long>(gguf_data_offset(f) + info->offset);
    const bool ok = std::fseek(fp, pos, SEEK_SET) == 0 && std::fread(host, 1, bytes, fp) == bytes;
    std::fclose(fp);
    if (!ok) {
        std::fprintf(stderr, "[traincpp] GGUF: 张量 %s 数据越界\n", name);
        return false;
    }
    if (pbuf != nullptr) return pbuf->store(dst, info->type, host, bytes);  // the blocks as they are
    void* staging = dev->scratch((bytes + 15) / 16 * 16);
    float* out = reinterpret_cast<float*>(buf->device_ptr() + dst->data_offset);
    CB_TRC(trc_cuda_load_quant(static_cast<int>(info->type), host, n_blocks, staging, out, dev->stream()),
           "trc_cuda_load_quant");
    CB_CUDA(trc_cuda_rt_stream_sync(dev->stream()));  // the pinned and device staging are free again
    int code = 0;
    CB_TRC(trc_cuda_device_error(&code, 1), "trc_cuda_device_error");
    if (code != 0) CB_ABORT("CUDA: dequant kernel 等待超时（设备错误码 %d）", code);
    return true;
}

// Algorithmic bytes of loading one file tensor: what is read (packed or F32) plus the F32 written.
static int64_t load_bytes(const GgufFile* f, int64_t ti) {
    const GgufTensorInfo* info = gguf_tensor_info(f, ti);
    return static_cast<int64_t>(info->nbytes) + 4 * gguf_tensor_nelements(f, ti);
}

std::vector<int64_t> gguf_shard_tensors(const GgufFile* f, int rank, int world) {
    if (f == nullptr || world <= 0 || rank < 0 || rank >= world) CB_ABORT("gguf_shard_tensors: 参数无效");
    const int64_t n = gguf_tensor_count(f);
    std::vector<int64_t> order(static_cast<size_t>(n));
    for (int64_t i = 0; i < n; ++i) order[static_cast<size_t>(i)] = i;
    // largest first, ties by file order; each tensor to the least-loaded rank, ties to the lowest rank
    std::stable_sort(order.begin(), order.end(),
                     [&](int64_t a, int64_t b) { return load_bytes(f, a) > load_bytes(f, b); });
    std::vector<int64_t> loads(static_cast<size_t>(world), 0);
    std::vector<int64_t> mine;
    for (const int64_t ti : order) {
        const auto least = std::min_element(loads.begin(), loads.end());
        *least += load_bytes(f, ti);
        if (least - loads.begin() == rank) mine.push_back(ti);
    }
    std::sort(mine.begin(), mine.end());
    return mine;
}

bool cuda_gguf_load_tensors(const GgufFile* f, const char* path, const char* const* names, Tensor* const* dsts,
                            size_t count, size_t staging_bytes) {
    if (f == nullptr || path == nullptr || (count > 0 && (names == nullptr || dsts == nullptr)))
        CB_ABORT("cuda_gguf_load_tensors: 参数为空");
    struct Job {
        const GgufTensorInfo* info;
        int64_t               n_units;  // 32-weight blocks, or floats for an F32 file tensor
        float*                out;
    };
    std::vector<Job> jobs;
    std::vector<size_t> fallback;  // tensors the reference loader handles (not quantized / not on CUDA)
    std::vector<size_t> packed;    // destinations on a packed-weight buffer
    CudaDevice* dev = nullptr;
    for (size_t i = 0; i < count; ++i) {
        const int64_t ti = gguf_find_tensor(f, names[i]);
        if (ti < 0) {
            std::fprintf(stderr, "[traincpp] GGUF: 张量不存在 %s\n", names[i]);
            return false;
        }
        const GgufTensorInfo* info = gguf_tensor_info(f, ti);
        CudaBuffer* buf = cuda_buffer_of(dsts[i]);
        if (packed_buffer_of(dsts[i]) != nullptr) {  // frozen quantized weight: its blocks as they are
            packed.push_back(i);
            continue;
        }
        if ((!is_legacy_quant(info->type) && info->type != TYPE_F32) || dsts[i]->type != TYPE_F32 || buf == nullptr) {
            fallback.push_back(i);
            continue;
        }
        if (!tensor_is_contiguous(dsts[i]) || tensor_nelements(dsts[i]) != gguf_tensor_nelements(f, ti)) {
            std::fprintf(stderr, "[traincpp] GGUF: 目标张量 %s 必须连续且元素数一致\n", names[i]);
            return false;
        }
        CudaDevice* d = static_cast<CudaDevice*>(buf->buffer_type()->device());
        if (dev != nullptr && d != dev) CB_ABORT("cuda_gguf_load_tensors: 目标张量须在同一 CUDA 设备上");
        dev = d;
        const bool quant = info->type != TYPE_F32;
        jobs.push_back({info, quant ? gguf_tensor_nelements(f, ti) / 32 : gguf_tensor_nelements(f, ti),
                        reinterpret_cast<float*>(buf->device_ptr() + dsts[i]->data_offset)});
    }
    bool ok = true;
    if (!jobs.empty()) {
        const size_t S = std::max<size_t>(staging_bytes / 16 * 16, 4096);
        FILE* fp = std::fopen(path, "rb");
        if (fp == nullptr) {
            std::fprintf(stderr, "[traincpp] GGUF: 无法打开 %s\n", path);
            return false;
        }
        CB_CUDA(trc_cuda_rt_set_device(dev->ordinal()));
        void* host[2] = {nullptr, nullptr};
        void* done[2] = {nullptr, nullptr};
        for (int k = 0; k < 2; ++k) {
            CB_CUDA(trc_cuda_rt_malloc_host(&host[k], S));
            CB_CUDA(trc_cuda_rt_event_create(&done[k]));
        }
        uint8_t* staging = static_cast<uint8_t*>(dev->scratch(2 * S));
        // chunks of whole blocks; chunk c uses pinned buffer and device staging c % 2, refilled only
        // after the copy of chunk c - 2 has read it (its event)
        uint64_t c = 0;
        for (const Job& J : jobs) {
            const bool    quant = J.info->type != TYPE_F32;
            const size_t  bb = quant ? trc_cuda_block_bytes(static_cast<int>(J.info->type)) : sizeof(float);
            const int64_t per_chunk = static_cast<int64_t>(S / bb);
            for (int64_t b0 = 0; ok && b0 < J.n_units; b0 += per_chunk, ++c) {
                const int64_t nb = std::min(per_chunk, J.n_units - b0);
                const int k = static_cast<int>(c & 1u);
                if (c >= 2) CB_CUDA(trc_cuda_rt_event_sync(done[k]));
                const long pos = static_cast<long>(gguf_data_offset(f) + J.info->offset + static_cast<uint64_t>(b0) * bb);
                const size_t bytes = static_cast<size_t>(nb) * bb;
                if (std::fseek(fp, pos, SEEK_SET) != 0 || std::fread(host[k], 1, bytes, fp) != bytes) {
                    std::fprintf(stderr, "[traincpp] GGUF: 张量 %s 数据越界\n", J.info->name);
                    ok = false;
                    break;
                }
                if (quant)
                    CB_TRC(trc_cuda_load_quant(static_cast<int>(J.info->type), host[k], nb, staging + k * S,
                                               J.out + b0 * 32, dev->stream()),
                           "trc_cuda_load_quant");
                else  // F32 file tensor: a plain copy (the reference's F32 branch, src/io/trc_gguf.cpp:1079)
                    CB_CUDA(trc_cuda_rt_memcpy_async(J.out + b0, host[k], bytes, 0, dev->stream()));
                CB_CUDA(trc_cuda_rt_event_record(done[k], dev->stream()));
            }
            if (!ok) break;
        }
        std::fclose(fp);
        CB_CUDA(trc_cuda_rt_stream_sync(dev->stream()));
        for (int k = 0; k < 2; ++k) {
            trc_cuda_rt_event_destroy(done[k]);
            trc_cuda_rt_free_host(host[k]);
        }
        int code = 0;
        CB_TRC(trc_cuda_device_error(&code, 1), "trc_cuda_device_error");
        if (code != 0) CB_ABORT("CUDA: dequant kernel 等待超时（设备错误码 %d）", code);
    }
    for (const size_t i : packed) ok = ok && cuda_gguf_load_tensor(f, path, names[i], dsts[i]);
    for (const size_t i : fallback) ok = ok && gguf_load_tensor(f, names[i], dsts[i]);
    return ok;
}

}  // namespace traincpp

extern "C" int trc_cuda_backend_register(void) { return traincpp::cuda_register_devices(); }

extern "C" void* trc_cuda_backend_device(int ordinal) { return traincpp::cuda_device(ordinal); }

extern "C" int64_t trc_cuda_backend_gguf_shard_plan(const char* path, int rank, int world, int64_t* indices,
                                                    int64_t capacity) {
    if (path == nullptr || world <= 0 || rank < 0 || rank >= world || capacity < 0) return -1;
    traincpp::GgufFile* f = traincpp::gguf_open(path, false);
    if (f == nullptr) return -1;
    const std::vector<int64_t> mine = traincpp::gguf_shard_tensors(f, rank, world);
    traincpp::gguf_close(f);
    for (size_t i = 0; i < mine.size() && static_cast<int64_t>(i) < capacity; ++i) indices[i] = mine[i];
    return static_cast<int64_t>(mine.size());
}
