// ref_shim.cpp -- TEST INFRASTRUCTURE, not product code.
//
// A thin extern "C" wrapper over the reference library (train.cpp / traincpp, compiled from its own
// sources by oracle/Makefile into oracle/_ref/libtrc_ref.so). It lets the Python tests and the CPU
// baseline of bench.py call the reference's own CPU code paths without linking C++:
//
//   * fp16 <-> fp32 conversion           src/core/trc_float.h:23-63
//   * GGUF open + host dequantization    src/io/trc_gguf.cpp:748-775 (gguf_open),
//                                        :966-1049 (gguf_tensor_to_f32) -> :320-417 (dequantize_*)
//   * ggml mul_mat on the CPU device     src/ops/trc_ops.cpp:366-385, src/backends/cpu/trc_cpu_ops.cpp:182-216
//   * mul_mat forward + composed backward through the reference autograd
//                                        src/core/trc_autograd.cpp:487-503 (OP_MUL_MAT rule),
//                                        loss = sum(mul(D, G)) injects dL/dD = G exactly (:247-257, :420)
//   * the rest of a training step on the CPU device: unaries (neg/abs_op/sqr/sqrt_op/sgn/step/scale),
//     sum_rows / mean, opt_step_adamw / opt_step_sgd and the grad-norm clip pair sum_sqr_acc /
//     clip_scale_inplace (src/ops/trc_ops.cpp, src/backends/cpu/trc_cpu_ops.cpp)
//
// Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm load this.
#include "traincpp/traincpp.h"
#include "core/trc_float.h"

#include <cstdint>
#include <cstring>

using namespace traincpp;

namespace {

Tensor* make_operand(Context* ctx, const int64_t* ne, int trans, Tensor** base_out) {
    Tensor* base = new_tensor_4d(ctx, TYPE_F32, ne[0], ne[1], ne[2], ne[3]);
    *base_out = base;
    return trans ? transpose(ctx, base) : base;
}

size_t nbytes4(const int64_t* ne) {
    return (size_t) (ne[0] * ne[1] * ne[2] * ne[3]) * sizeof(float);
}

} // namespace

extern "C" {

uint32_t ref_fp16_to_fp32_bits(uint16_t h) {
    return fp32_to_bits(fp16_to_fp32(h));
}

uint16_t ref_fp32_to_fp16(float f) {
    return fp32_to_fp16(f);
}

// GGUF handle API: the caller writes the file; the reference parses it (load_data=true).
void* ref_gguf_open(const char* path) {
    return (void*) gguf_open(path, true);
}

void ref_gguf_close(void* f) {
    gguf_close((GgufFile*) f);
}

int64_t ref_gguf_tensor_nelements(void* f, const char* name) {
    const int64_t i = gguf_find_tensor((GgufFile*) f, name);
    return i < 0 ? -1 : gguf_tensor_nelements((GgufFile*) f, i);
}

// Host dequantization exactly as the reference's loader performs it. 0 = ok, -1 = rejected.
int ref_gguf_tensor_to_f32(void* f, const char* name, float* out, int64_t n) {
    return gguf_tensor_to_f32((GgufFile*) f, name, out, n) ? 0 : -1;
}

// D = mul_mat(A, B) on the reference CPU device. a_ne/b_ne describe the contiguous stored
// tensors; a_trans/b_trans make the operand transpose(stored) (a permute(1,0,2,3) view, the form
// the composed backward produces). d receives the contiguous result [A.ne1, B.ne1, B.ne2, B.ne3].
int ref_mul_mat(const float* a, const int64_t* a_ne, int a_trans,
                const float* b, const int64_t* b_ne, int b_trans, float* d) {
    Context* ctx = context_new((size_t) 1 << 20);
    Graph*   g   = graph_new(ctx);
    Tensor *abase = nullptr, *bbase = nullptr;
    Tensor* A   = make_operand(ctx, a_ne, a_trans, &abase);
    Tensor* B   = make_operand(ctx, b_ne, b_trans, &bbase);
    Tensor* out = mul_mat(ctx, A, B);
    graph_build_forward_expand(ctx, g, out);
    Device* cpu = device_cpu();
    Buffer* buf = buffer_alloc_ctx_tensors(ctx, cpu->default_buffer_type());
    tensor_set(abase, a, 0, nbytes4(a_ne));
    tensor_set(bbase, b, 0, nbytes4(b_ne));
    const bool ok = cpu->graph_compute(g);
    tensor_get(out, d, 0, tensor_nbytes(out));
    buffer_free(buf);
    graph_free(g);
    context_free(ctx);
    return ok ? 0 : -1;
}

// One training step of D = mul_mat(A, B) through the reference autograd: A and B are PARAMs,
// loss = sum(mul(D, G)), so dL/dD = G. Writes D, dA (= A's grad_acc) and dB (= B's grad_acc).
// This is the Linear forward + composed backward of the configs (A = weight, B = activations)
// and, with ne[2]/ne[3] broadcasting, the batched GQA case (dA goes through repeat_back).
int ref_mul_mat_step(const float* a, const int64_t* a_ne, const float* b, const int64_t* b_ne,
                     const float* gr, float* d, float* da, float* db) {
    Context* ctx = context_new((size_t) 1 << 22);
    Graph*   g   = graph_new(ctx);
    Tensor* A = new_tensor_4d(ctx, TYPE_F32, a_ne[0], a_ne[1], a_ne[2], a_ne[3]);
    Tensor* B = new_tensor_4d(ctx, TYPE_F32, b_ne[0], b_ne[1], b_ne[2], b_ne[3]);
    tensor_set_param(A);
    tensor_set_param(B);
    Tensor* D = mul_mat(ctx, A, B);
    Tensor* G = new_tensor_4d(ctx, TYPE_F32, D->ne[0], D->ne[1], D->ne[2], D->ne[3]);
    Tensor* loss = sum(ctx, mul(ctx, D, G));
    tensor_set_loss(loss);
    graph_build_forward_expand(ctx, g, loss);
    graph_build_backward_expand(g);
    Device* cpu = device_cpu();
    Buffer* buf = buffer_alloc_ctx_tensors(ctx, cpu->default_buffer_type());
    tensor_set(A, a, 0, nbytes4(a_ne));
    tensor_set(B, b, 0, nbytes4(b_ne));
    tensor_set(G, gr, 0, tensor_nbytes(G));
    graph_reset(g);
    const bool ok = cpu->graph_compute(g);
    tensor_get(D, d, 0, tensor_nbytes(D));
    tensor_get(graph_get_grad_acc(g, A), da, 0, tensor_nbytes(A));
    tensor_get(graph_get_grad_acc(g, B), db, 0, tensor_nbytes(B));
    buffer_free(buf);
    graph_free(g);
    context_free(ctx);
    return ok ? 0 : -1;
}

} // extern "C"

namespace {

// One node evaluated on the reference CPU device: `build` creates the inputs and the node,
// `upload` sets the inputs after allocation, `read` reads the results back.
template <class Build, class Upload, class Read>
int run_node(Build build, Upload upload, Read read) {
    Context* ctx = context_new((size_t) 1 << 20);
    Graph*   g   = graph_new(ctx);
    Tensor*  out = build(ctx);
    graph_build_forward_expand(ctx, g, out);
    Device* cpu = device_cpu();
    Buffer* buf = buffer_alloc_ctx_tensors(ctx, cpu->default_buffer_type());
    upload();
    const bool ok = cpu->graph_compute(g);
    read(out);
    buffer_free(buf);
    graph_free(g);
    context_free(ctx);
    return ok ? 0 : -1;
}

} // namespace

extern "C" {

// op: 0 sqr, 1 sqrt, 2 abs, 3 neg, 4 sgn, 5 step, 6 scale(param) -- the library's TRC_CUDA_UNARY_* codes.
int ref_unary(int op, const float* x, const int64_t* ne, float param, float* out) {
    Tensor* a = nullptr;
    return run_node(
        [&](Context* ctx) {
            a = new_tensor_4d(ctx, TYPE_F32, ne[0], ne[1], ne[2], ne[3]);
            switch (op) {
                case 0: return sqr(ctx, a);
                case 1: return sqrt_op(ctx, a);
                case 2: return abs_op(ctx, a);
                case 3: return neg(ctx, a);
                case 4: return sgn(ctx, a);
                case 5: return step(ctx, a);
                default: return scale(ctx, a, param);
            }
        },
        [&] { tensor_set(a, x, 0, nbytes4(ne)); },
        [&](Tensor* o) { tensor_get(o, out, 0, tensor_nbytes(o)); });
}

int ref_sum_rows(const float* x, const int64_t* ne, int take_mean, float* out) {
    Tensor* a = nullptr;
    return run_node(
        [&](Context* ctx) {
            a = new_tensor_4d(ctx, TYPE_F32, ne[0], ne[1], ne[2], ne[3]);
            return take_mean ? mean(ctx, a) : sum_rows(ctx, a);
        },
        [&] { tensor_set(a, x, 0, nbytes4(ne)); },
        [&](Tensor* o) { tensor_get(o, out, 0, tensor_nbytes(o)); });
}

// In place on p, m, v (n floats each); params6 as the optimizer writes them.
int ref_opt_step_adamw(float* p, const float* g, float* m, float* v, int64_t n, const float* ps) {
    Tensor *P = nullptr, *G = nullptr, *M = nullptr, *V = nullptr;
    return run_node(
        [&](Context* ctx) {
            P = new_tensor_1d(ctx, TYPE_F32, n);
            G = new_tensor_1d(ctx, TYPE_F32, n);
            M = new_tensor_1d(ctx, TYPE_F32, n);
            V = new_tensor_1d(ctx, TYPE_F32, n);
            return opt_step_adamw(ctx, P, G, M, V, ps[0], ps[1], ps[2], ps[3], ps[4], ps[5]);
        },
        [&] {
            tensor_set(P, p, 0, n * sizeof(float));
            tensor_set(G, g, 0, n * sizeof(float));
            tensor_set(M, m, 0, n * sizeof(float));
            tensor_set(V, v, 0, n * sizeof(float));
        },
        [&](Tensor*) {
            tensor_get(P, p, 0, n * sizeof(float));
            tensor_get(M, m, 0, n * sizeof(float));
            tensor_get(V, v, 0, n * sizeof(float));
        });
}

int ref_opt_step_sgd(float* p, const float* g, float* mom, int64_t n, const float* ps) {
    Tensor *P = nullptr, *G = nullptr, *M = nullptr;
    return run_node(
        [&](Context* ctx) {
            P = new_tensor_1d(ctx, TYPE_F32, n);
            G = new_tensor_1d(ctx, TYPE_F32, n);
            M = new_tensor_1d(ctx, TYPE_F32, n);
            return opt_step_sgd(ctx, P, G, M, ps[0], ps[1], ps[2], ps[3], ps[4] != 0.0f, ps[5] != 0.0f);
        },
        [&] {
            tensor_set(P, p, 0, n * sizeof(float));
            tensor_set(G, g, 0, n * sizeof(float));
            tensor_set(M, mom, 0, n * sizeof(float));
        },
        [&](Tensor*) {
            tensor_get(P, p, 0, n * sizeof(float));
            tensor_get(M, mom, 0, n * sizeof(float));
        });
}

int ref_sum_sqr_acc(float* acc, const float* x, int64_t n) {
    Tensor *ACC = nullptr, *A = nullptr;
    return run_node(
        [&](Context* ctx) {
            ACC = new_tensor_1d(ctx, TYPE_F32, 1);
            A   = new_tensor_1d(ctx, TYPE_F32, n);
            return sum_sqr_acc(ctx, ACC, A);
        },
        [&] {
            tensor_set(ACC, acc, 0, sizeof(float));
            tensor_set(A, x, 0, n * sizeof(float));
        },
        [&](Tensor*) { tensor_get(ACC, acc, 0, sizeof(float)); });
}

int ref_clip_scale_inplace(float* x, int64_t n, float norm, float max_norm, float eps) {
    Tensor *A = nullptr, *N = nullptr;
    return run_node(
        [&](Context* ctx) {
            A = new_tensor_1d(ctx, TYPE_F32, n);
            N = new_tensor_1d(ctx, TYPE_F32, 1);
            return clip_scale_inplace(ctx, A, N, max_norm, eps);
        },
        [&] {
            tensor_set(A, x, 0, n * sizeof(float));
            tensor_set(N, &norm, 0, sizeof(float));
        },
        [&](Tensor*) { tensor_get(A, x, 0, n * sizeof(float)); });
}

} // extern "C"
