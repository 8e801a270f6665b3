// test_dropin.cpp -- the CUDA backend as a drop-in train.cpp device.
//
// Everything above the backend is train.cpp's own code, unchanged (linked from the library that
// oracle/Makefile compiles from its sources): contexts, op constructors, graph building, autograd,
// buffer allocation, the GGUF reader and nn::Linear. Each case builds the same graph on the
// reference CPU device and on the CUDA device and compares the results, the way the reference's
// backend conformance suite compares its Vulkan device with the CPU
// (tests/test_backend_conformance.cpp:43-128 of train.cpp).
//
// usage: test_dropin [all|alloc_fail|shard|packed|checkpoint] [path] [tokens]
// Exit status 0 when every case passes.
#include "traincpp/traincpp.h"
#include "trc_cuda_backend.h"
#include "trc_cuda_runtime.h"

#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <random>
#include <string>
#include <vector>

using namespace traincpp;

namespace {

int g_failures = 0;

void fail(const std::string& msg) {
    std::printf("    [FAIL] %s\n", msg.c_str());
    ++g_failures;
}

std::vector<float> ramp(size_t n) {  // the conformance suite's input pattern
    std::vector<float> v(n);
    for (size_t i = 0; i < n; ++i) v[i] = (float) ((int) (i % 17) - 8) * 0.25f;
    return v;
}

std::vector<float> gauss(size_t n, unsigned seed, float sigma = 1.0f) {
    std::mt19937 g(seed);
    std::normal_distribution<float> d(0.0f, sigma);
    std::vector<float> v(n);
    for (auto& x : v) x = d(g);
    return v;
}

double normwise(const std::vector<float>& got, const std::vector<float>& want) {
    double num = 0, den = 0;
    for (size_t i = 0; i < want.size(); ++i) {
        num = std::max(num, std::fabs((double) got[i] - want[i]));
        den = std::max(den, std::fabs((double) want[i]));
    }
    return den > 0 ? num / den : num;
}

// The normwise bar max|got - want| / max|want| <= 1e-5 everywhere. The reference's element-wise
// conformance tolerance 1e-5 + 2e-4|ref| (test_backend_conformance.cpp:99) is applied too where it
// is meaningful: its own small-K cases. At K in the hundreds and beyond, the CPU's sequential fp32
// sum is itself off by more than 2e-4 relative on near-zero outputs, so element-wise relative
// error no longer measures the device.
void compare(const char* name, const std::vector<float>& got, const std::vector<float>& want, bool elementwise = false,
             double norm_tol = 1e-5) {
    if (got.size() != want.size()) {
        fail(std::string(name) + ": size mismatch");
        return;
    }
    int64_t bad = 0;
    for (size_t i = 0; elementwise && i < want.size(); ++i)
        if (std::fabs((double) got[i] - want[i]) > 1e-5 + 2e-4 * std::fabs((double) want[i])) ++bad;
    const double nw = normwise(got, want);
    if (bad != 0 || nw > norm_tol) {
        char buf[256];
        std::snprintf(buf, sizeof(buf), "%s: %lld elements outside 1e-5+2e-4|ref|, normwise %.3g", name, (long long) bad, nw);
        fail(buf);
    } else {
        std::printf("    [ OK ] %-34s normwise %.2e\n", name, nw);
    }
}

struct Built {
    Tensor* out;
    std::vector<std::pair<Tensor*, std::vector<float>>> inputs;
};
using BuildFn = std::function<Built(Context*)>;

std::vector<float> run_forward(Device* dev, const BuildFn& build) {
    Context* ctx = context_new(1 << 22);
    Graph*   g   = graph_new(ctx);
    Built    b   = build(ctx);
    Buffer*  buf = buffer_alloc_ctx_tensors(ctx, dev->default_buffer_type());
    for (auto& in : b.inputs) tensor_set(in.first, in.second.data(), 0, in.second.size() * sizeof(float));
    graph_build_forward_expand(ctx, g, b.out);
    if (const Tensor* bad = graph_first_unsupported(g, dev)) {
        fail(std::string("graph_first_unsupported: ") + op_name(bad->op));
    }
    dev->graph_compute(g);
    std::vector<float> out((size_t) tensor_nelements(b.out));
    tensor_get(b.out, out.data(), 0, out.size() * sizeof(float));
    buffer_free(buf);
    graph_free(g);
    context_free(ctx);
    return out;
}

void conformance_matmul(Device* cpu, Device* cuda) {
    std::printf("  conformance_matmul (the reference's cases)\n");
    struct Case {
        const char* name;
        BuildFn     fn;
        bool        elementwise = true;
    };
    std::vector<Case> cases = {
        {"mul_mat_basic", [](Context* c) {
             Tensor* a = new_tensor_2d(c, TYPE_F32, 5, 3);
             Tensor* b = new_tensor_2d(c, TYPE_F32, 5, 4);
             return Built{mul_mat(c, a, b), {{a, ramp(15)}, {b, ramp(20)}}};
         }},
        {"mul_mat_transposed_a", [](Context* c) {
             Tensor* base = new_tensor_2d(c, TYPE_F32, 3, 5);
             Tensor* b    = new_tensor_2d(c, TYPE_F32, 5, 4);
             return Built{mul_mat(c, transpose(c, base), b), {{base, ramp(15)}, {b, ramp(20)}}};
         }},
        {"mul_mat_transposed_b", [](Context* c) {
             Tensor* a    = new_tensor_2d(c, TYPE_F32, 5, 3);
             Tensor* base = new_tensor_2d(c, TYPE_F32, 4, 5);
             return Built{mul_mat(c, a, transpose(c, base)), {{a, ramp(15)}, {base, ramp(20)}}};
         }},
        {"mul_mat_tile_boundary", [](Context* c) {
             Tensor* a = new_tensor_2d(c, TYPE_F32, 33, 70);
             Tensor* b = new_tensor_2d(c, TYPE_F32, 33, 66);
             return Built{mul_mat(c, a, b), {{a, ramp(33 * 70)}, {b, ramp(33 * 66)}}};
         }},
        {"mul_mat_batch", [](Context* c) {
             Tensor* a = new_tensor_4d(c, TYPE_F32, 5, 3, 1, 1);
             Tensor* b = new_tensor_4d(c, TYPE_F32, 5, 4, 2, 3);
             return Built{mul_mat(c, a, b), {{a, ramp(15)}, {b, ramp(120)}}};
         }},
        {"mul_mat_batch_bcast_div", [](Context* c) {
             Tensor* a = new_tensor_4d(c, TYPE_F32, 5, 3, 2, 1);
             Tensor* b = new_tensor_4d(c, TYPE_F32, 5, 4, 4, 1);
             return Built{mul_mat(c, a, b), {{a, ramp(30)}, {b, ramp(80)}}};
         }},
        {"mul_mat_batch_transposed", [](Context* c) {
             Tensor* abase = new_tensor_4d(c, TYPE_F32, 3, 5, 2, 2);
             Tensor* bbase = new_tensor_4d(c, TYPE_F32, 4, 5, 2, 2);
             return Built{mul_mat(c, transpose(c, abase), transpose(c, bbase)), {{abase, ramp(60)}, {bbase, ramp(80)}}};
         }},
        {"mul_mat_batch_tile_boundary", [](Context* c) {
             Tensor* a = new_tensor_4d(c, TYPE_F32, 33, 70, 1, 1);
             Tensor* b = new_tensor_4d(c, TYPE_F32, 33, 66, 2, 2);
             return Built{mul_mat(c, a, b), {{a, ramp(33 * 70)}, {b, ramp(33 * 66 * 4)}}};
         }},
        {"grid_mul_mat_batch_z", [](Context* c) {
             Tensor* a = new_tensor_4d(c, TYPE_F32, 8, 4, 1, 1);
             Tensor* b = new_tensor_4d(c, TYPE_F32, 8, 4, 65, 1);
             return Built{mul_mat(c, a, b), {{a, ramp(32)}, {b, ramp(8 * 4 * 65)}}};
         }},
        // tensor-core eligible shapes (16-byte strides), transposed views, broadcast, ragged tiles
        {"tc_linear_fwd", [](Context* c) {
             Tensor* w = new_tensor_2d(c, TYPE_F32, 1024, 300);
             Tensor* x = new_tensor_2d(c, TYPE_F32, 1024, 72);
             return Built{mul_mat(c, w, x), {{w, gauss(1024 * 300, 1)}, {x, gauss(1024 * 72, 2)}}};
         }, false},
        {"tc_transposed_both", [](Context* c) {
             Tensor* abase = new_tensor_4d(c, TYPE_F32, 132, 520, 2, 1);
             Tensor* bbase = new_tensor_4d(c, TYPE_F32, 260, 520, 4, 1);
             return Built{mul_mat(c, transpose(c, abase), transpose(c, bbase)),
                          {{abase, gauss(132 * 520 * 2, 3)}, {bbase, gauss(260 * 520 * 4, 4)}}};
         }, false},
    };
    for (auto& k : cases) compare(k.name, run_forward(cuda, k.fn), run_forward(cpu, k.fn), k.elementwise);
}

struct StepOut {
    std::vector<float> y, da, db, dbias;
};

// One training step of y = mul_mat(A, B) [+ bias] with loss = sum(mul(y, G)) through the reference
// autograd (trc_autograd.cpp:487-503; the injected gradient dL/dy = G).
StepOut run_step(Device* dev, const int64_t* ane, const int64_t* bne, bool with_bias, unsigned seed) {
    Context* ctx = context_new(1 << 22);
    Graph*   g   = graph_new(ctx);
    Tensor*  A   = new_tensor_4d(ctx, TYPE_F32, ane[0], ane[1], ane[2], ane[3]);
    Tensor*  B   = new_tensor_4d(ctx, TYPE_F32, bne[0], bne[1], bne[2], bne[3]);
    tensor_set_param(A);
    tensor_set_param(B);
    Tensor* y    = mul_mat(ctx, A, B);
    Tensor* bias = nullptr;
    if (with_bias) {
        bias = new_tensor_1d(ctx, TYPE_F32, y->ne[0]);
        tensor_set_param(bias);
        y = add(ctx, y, bias);
    }
    Tensor* G    = new_tensor_4d(ctx, TYPE_F32, y->ne[0], y->ne[1], y->ne[2], y->ne[3]);
    Tensor* loss = sum(ctx, mul(ctx, y, G));
    tensor_set_loss(loss);
    graph_build_forward_expand(ctx, g, loss);
    graph_build_backward_expand(g);
    if (const Tensor* bad = graph_first_unsupported(g, dev)) fail(std::string("preflight: ") + op_name(bad->op));
    Buffer* buf = buffer_alloc_ctx_tensors(ctx, dev->default_buffer_type());
    auto av = gauss((size_t) tensor_nelements(A), seed);
    auto bv = gauss((size_t) tensor_nelements(B), seed + 1);
    auto gv = gauss((size_t) tensor_nelements(G), seed + 2, 1e-2f);
    tensor_set(A, av.data(), 0, av.size() * 4);
    tensor_set(B, bv.data(), 0, bv.size() * 4);
    tensor_set(G, gv.data(), 0, gv.size() * 4);
    if (bias != nullptr) {
        auto bb = gauss((size_t) tensor_nelements(bias), seed + 3);
        tensor_set(bias, bb.data(), 0, bb.size() * 4);
    }
    graph_reset(g);
    dev->graph_compute(g);
    StepOut r;
    r.y.resize((size_t) tensor_nelements(y));
    tensor_get(y, r.y.data(), 0, r.y.size() * 4);
    Tensor* ga = graph_get_grad_acc(g, A);
    Tensor* gb = graph_get_grad_acc(g, B);
    r.da.resize((size_t) tensor_nelements(ga));
    r.db.resize((size_t) tensor_nelements(gb));
    tensor_get(ga, r.da.data(), 0, r.da.size() * 4);
    tensor_get(gb, r.db.data(), 0, r.db.size() * 4);
    if (bias != nullptr) {
        Tensor* gbias = graph_get_grad_acc(g, bias);
        r.dbias.resize((size_t) tensor_nelements(gbias));
        tensor_get(gbias, r.dbias.data(), 0, r.dbias.size() * 4);
    }
    buffer_free(buf);
    graph_free(g);
    context_free(ctx);
    return r;
}

void training_steps(Device* cpu, Device* cuda) {
    std::printf("  training steps through the reference autograd\n");
    struct Case {
        const char* name;
        int64_t     a[4], b[4];
        bool        bias;
    };
    const Case cases[] = {
        {"linear_step (W 1024x384, 96 tokens)", {1024, 384, 1, 1}, {1024, 96, 1, 1}, false},
        {"linear_step_bias", {512, 256, 1, 1}, {512, 80, 1, 1}, true},
        {"linear_step_ragged", {100, 70, 1, 1}, {100, 33, 1, 1}, false},
        {"gqa_step (bcast ne2 x4)", {128, 96, 2, 2}, {128, 80, 8, 2}, false},
    };
    for (const Case& c : cases) {
        const StepOut want = run_step(cpu, c.a, c.b, c.bias, 7);
        const StepOut got  = run_step(cuda, c.a, c.b, c.bias, 7);
        const std::string n = c.name;
        compare((n + " y").c_str(), got.y, want.y);
        compare((n + " dA").c_str(), got.da, want.da);
        compare((n + " dB").c_str(), got.db, want.db);
        if (c.bias) compare((n + " dbias").c_str(), got.dbias, want.dbias);
    }
}

// A Linear model trained for several steps the way the reference trains (its optimizer test
// fixture: graph_reset + graph_compute, then optim_clip_grad_norm and optim_step;
// tests/test_optim.cpp of train.cpp): y = W x + b, loss = mean((y - t)^2). On the CUDA device every
// node -- forward, autograd backward, the optimizer's OP_OPT_STEP_* graph and the clip graph's
// OP_SUM_SQR_ACC / OP_CLIP_SCALE_INPLACE -- runs on the device.
struct LoopOut {
    std::vector<float> w, b;
    float              loss0 = 0, loss1 = 0;
};

LoopOut train_loop(Device* dev, bool use_sgd, int steps, float clip) {
    constexpr int64_t IN = 256, OUT = 160, BATCH = 48;
    Context* ctx = context_new((size_t) 1 << 24);
    Graph*   g   = graph_new(ctx);
    Tensor*  W   = new_tensor_2d(ctx, TYPE_F32, IN, OUT);
    Tensor*  b   = new_tensor_2d(ctx, TYPE_F32, OUT, 1);
    Tensor*  x   = new_tensor_2d(ctx, TYPE_F32, IN, BATCH);
    Tensor*  y   = new_tensor_2d(ctx, TYPE_F32, OUT, BATCH);
    Tensor*  params[2] = {W, b};
    tensor_set_param(W);
    tensor_set_param(b);
    Tensor* pred = add(ctx, mul_mat(ctx, W, x), b);
    Tensor* loss = scale(ctx, sum(ctx, sqr(ctx, sub(ctx, pred, y))), 1.0f / (float) (OUT * BATCH));
    tensor_set_loss(loss);
    graph_build_forward_expand(ctx, g, loss);
    graph_build_backward_expand(g);
    Buffer* buf = buffer_alloc_ctx_tensors(ctx, dev->default_buffer_type());
    if (const Tensor* bad = graph_first_unsupported(g, dev)) fail(std::string("graph_first_unsupported: ") + op_name(bad->op));
    const auto vw = gauss((size_t) (IN * OUT), 21, 0.05f), vb = gauss((size_t) OUT, 22, 0.1f);
    const auto vx = gauss((size_t) (IN * BATCH), 23), vy = gauss((size_t) (OUT * BATCH), 24);
    tensor_set(W, vw.data(), 0, vw.size() * 4);
    tensor_set(b, vb.data(), 0, vb.size() * 4);
    tensor_set(x, vx.data(), 0, vx.size() * 4);
    tensor_set(y, vy.data(), 0, vy.size() * 4);
    Optimizer* opt = nullptr;
    if (use_sgd) {
        SgdOptions o;
        o.lr = 0.05f;
        o.momentum = 0.9f;
        o.weight_decay = 1e-4f;
        o.nesterov = true;
        opt = optim_sgd_new(ctx, params, 2, o);
    } else {
        AdamwOptions o;
        o.lr = 1e-2f;
        opt = optim_adamw_new(ctx, params, 2, o);
    }
    LoopOut r;
    graph_reset(g);
    dev->graph_compute(g);
    tensor_get(loss, &r.loss0, 0, 4);
    for (int it = 0; it < steps; ++it) {
        graph_reset(g);
        dev->graph_compute(g);
        optim_clip_grad_norm(opt, clip);
        optim_step(opt);
    }
    graph_reset(g);
    dev->graph_compute(g);
    tensor_get(loss, &r.loss1, 0, 4);
    r.w.resize(vw.size());
    r.b.resize(vb.size());
    tensor_get(W, r.w.data(), 0, r.w.size() * 4);
    tensor_get(b, r.b.data(), 0, r.b.size() * 4);
    optim_free(opt);
    buffer_free(buf);
    graph_free(g);
    context_free(ctx);
    return r;
}

void training_loops(Device* cpu, Device* cuda) {
    const char* simt = std::getenv("TRC_CUDA_MM_SIMT");
    const bool  exact = simt != nullptr && *simt != '\0' && *simt != '0';
    std::printf("  training loops: Linear + MSE, optimizer and grad-norm clip on the device (%s)\n",
                exact ? "SIMT mul_mat: bit-identical" : "tcgen05 mul_mat: within 1e-5");
    struct Case {
        const char* name;
        bool        sgd;
        float       clip;
    };
    const Case cases[] = {{"adamw, 12 steps, clip 0.5", false, 0.5f}, {"sgd nesterov, 12 steps, no clip", true, 1e9f}};
    for (const Case& c : cases) {
        const LoopOut want = train_loop(cpu, c.sgd, 12, c.clip);
        const LoopOut got  = train_loop(cuda, c.sgd, 12, c.clip);
        const std::string n = c.name;
        if (!(want.loss1 < want.loss0)) fail(n + ": the reference's loss did not decrease");
        if (exact) {
            const bool same = std::memcmp(got.w.data(), want.w.data(), want.w.size() * 4) == 0 &&
                              std::memcmp(got.b.data(), want.b.data(), want.b.size() * 4) == 0 &&
                              std::memcmp(&got.loss1, &want.loss1, 4) == 0;
            if (!same) {
                fail(n + ": parameters not bit-identical to the CPU device");
                compare((n + " W").c_str(), got.w, want.w);
            } else {
                std::printf("    [ OK ] %-34s W, b and loss bit-identical (loss %.6g -> %.6g)\n", c.name,
                            (double) want.loss0, (double) want.loss1);
            }
        } else {
            // AdamW divides every update by sqrt(v): on weights whose gradient is near zero, a last-bit
            // difference of the 3xTF32 GEMM moves the step by O(lr), so after 12 steps W agrees to
            // ~2e-5 normwise; b, the loss and SGD stay at the per-op 1e-5 bar.
            compare((n + " W").c_str(), got.w, want.w, false, c.sgd ? 1e-5 : 1e-4);
            compare((n + " b").c_str(), got.b, want.b);
            compare((n + " loss").c_str(), {got.loss1}, {want.loss1});
        }
    }
}

void gguf_warm_start(Device* cpu, Device* cuda, const char* path) {
    std::printf("  GGUF warm start: device dequant vs the reference loader (%s)\n", path);
    GgufFile* f = gguf_open(path, true);
    if (f == nullptr) {
        fail("gguf_open failed");
        return;
    }
    for (int64_t i = 0; i < gguf_tensor_count(f); ++i) {
        const GgufTensorInfo* info = gguf_tensor_info(f, i);
        Context* ctx = context_new(1 << 20);
        Tensor* w_dev = gguf_new_tensor(ctx, f, info->name, TYPE_F32);  // device dequant target
        Tensor* w_ref = gguf_new_tensor(ctx, f, info->name, TYPE_F32);  // reference loader target
        Buffer* buf   = buffer_alloc_ctx_tensors(ctx, cuda->default_buffer_type());
        const bool ok1 = cuda_gguf_load_tensor(f, path, info->name, w_dev);
        const bool ok2 = gguf_load_tensor(f, info->name, w_ref);  // host dequant + tensor_set (H2D)
        const size_t n = (size_t) tensor_nelements(w_dev);
        std::vector<float> a(n), b(n);
        tensor_get(w_dev, a.data(), 0, n * 4);
        tensor_get(w_ref, b.data(), 0, n * 4);
        if (!ok1 || !ok2 || std::memcmp(a.data(), b.data(), n * 4) != 0) {
            fail(std::string("gguf tensor ") + info->name + " not bit-identical");
        } else {
            std::printf("    [ OK ] %-34s %zu weights bit-identical (%s)\n", info->name, n, type_name(info->type));
        }
        buffer_free(buf);
        context_free(ctx);
    }
    // repeated single-tensor loads reuse the device's pinned staging: no page-locking per tensor
    {
        Context* ctx = context_new(1 << 20);
        std::vector<Tensor*> ws;
        for (int64_t i = 0; i < gguf_tensor_count(f); ++i)
            ws.push_back(gguf_new_tensor(ctx, f, gguf_tensor_info(f, i)->name, TYPE_F32));
        Buffer* buf = buffer_alloc_ctx_tensors(ctx, cuda->default_buffer_type());
        size_t largest = 0;
        for (int64_t i = 0; i < gguf_tensor_count(f); ++i) largest = std::max(largest, gguf_tensor_info(f, i)->nbytes);
        int64_t big = 0;
        for (int64_t i = 0; i < gguf_tensor_count(f); ++i)
            if (gguf_tensor_info(f, i)->nbytes == largest) big = i;
        cuda_gguf_load_tensor(f, path, gguf_tensor_info(f, big)->name, ws[(size_t) big]);  // sizes the staging
        const uint64_t pins = trc_cuda_rt_host_alloc_count();
        bool ok = true;
        for (int rep = 0; rep < 3; ++rep)
            for (int64_t i = 0; i < gguf_tensor_count(f); ++i)
                ok = ok && cuda_gguf_load_tensor(f, path, gguf_tensor_info(f, i)->name, ws[(size_t) i]);
        if (!ok || trc_cuda_rt_host_alloc_count() != pins) fail("repeated cuda_gguf_load_tensor pinned host memory again");
        else std::printf("    [ OK ] %-34s %lld loads, no new pinned allocation\n", "single-tensor loader staging reuse",
                         (long long) (3 * gguf_tensor_count(f)));
        buffer_free(buf);
        context_free(ctx);
    }
    // the warm-started weight feeds nn::Linear (linear_init_weight, src/nn/trc_nn.cpp:209-220)
    const GgufTensorInfo* info = gguf_tensor_info(f, 0);
    std::vector<float> outs[2];
    Device* devs[2] = {cpu, cuda};
    for (int d = 0; d < 2; ++d) {
        Context* ctx = context_new(1 << 20);
        Graph*   g   = graph_new(ctx);
        Tensor*  w   = gguf_new_tensor(ctx, f, info->name, TYPE_F32);
        Linear   lin;
        linear_init_weight(ctx, &lin, w, nullptr);
        Tensor* x = new_tensor_2d(ctx, TYPE_F32, w->ne[0], 40);
        Tensor* y = linear_forward(ctx, &lin, x);
        graph_build_forward_expand(ctx, g, y);
        Buffer* buf = buffer_alloc_ctx_tensors(ctx, devs[d]->default_buffer_type());
        if (d == 1) cuda_gguf_load_tensor(f, path, info->name, w);
        else gguf_load_tensor(f, info->name, w);
        auto xv = gauss((size_t) tensor_nelements(x), 5);
        tensor_set(x, xv.data(), 0, xv.size() * 4);
        devs[d]->graph_compute(g);
        outs[d].resize((size_t) tensor_nelements(y));
        tensor_get(y, outs[d].data(), 0, outs[d].size() * 4);
        buffer_free(buf);
        graph_free(g);
        context_free(ctx);
    }
    compare("linear_forward on warm-started W", outs[1], outs[0]);
    gguf_close(f);
}

// The sharded model loader: every rank's share (gguf_shard_tensors) streamed from the file with
// cuda_gguf_load_tensors through a small staging buffer (so tensors span several chunks), each
// tensor bit-identical to the reference's gguf_load_tensor, the ranks' shares a partition of the
// file. Prints "shard <world> <rank>: <indices>" for the caller to compare with its own LPT plan.
void gguf_sharded_load(Device* cuda, const char* path, int world) {
    std::printf("  sharded GGUF load over %d ranks (%s)\n", world, path);
    GgufFile* meta = gguf_open(path, false);  // header only: nothing of the data segment on the host
    GgufFile* full = gguf_open(path, true);   // the reference loader's view
    if (meta == nullptr || full == nullptr) {
        fail("gguf_open failed");
        return;
    }
    std::vector<int> owner(static_cast<size_t>(gguf_tensor_count(meta)), -1);
    for (int r = 0; r < world; ++r) {
        const std::vector<int64_t> mine = gguf_shard_tensors(meta, r, world);
        std::printf("shard %d %d:", world, r);
        for (int64_t ti : mine) std::printf(" %lld", (long long) ti);
        std::printf("\n");
        Context* ctx = context_new(1 << 20);
        std::vector<const char*> names;
        std::vector<Tensor*> dsts, refs;
        for (int64_t ti : mine) {
            if (owner[static_cast<size_t>(ti)] != -1) fail("tensor dealt to two ranks");
            owner[static_cast<size_t>(ti)] = r;
            const GgufTensorInfo* info = gguf_tensor_info(meta, ti);
            names.push_back(info->name);
            dsts.push_back(gguf_new_tensor(ctx, meta, info->name, TYPE_F32));
            refs.push_back(gguf_new_tensor(ctx, full, info->name, TYPE_F32));
        }
        Buffer* buf = buffer_alloc_ctx_tensors(ctx, cuda->default_buffer_type());
        const int before = g_failures;
        const bool ok = cuda_gguf_load_tensors(meta, path, names.data(), dsts.data(), names.size(), size_t(1) << 20);
        if (!ok) fail("cuda_gguf_load_tensors failed");
        for (size_t i = 0; i < names.size(); ++i) {
            if (!gguf_load_tensor(full, names[i], refs[i])) fail("reference gguf_load_tensor failed");
            const size_t n = (size_t) tensor_nelements(dsts[i]);
            std::vector<float> a(n), b(n);
            tensor_get(dsts[i], a.data(), 0, n * 4);
            tensor_get(refs[i], b.data(), 0, n * 4);
            if (std::memcmp(a.data(), b.data(), n * 4) != 0) fail(std::string("sharded load of ") + names[i] + " differs");
        }
        if (g_failures == before) std::printf("    [ OK ] rank %d: %zu tensors bit-identical\n", r, names.size());
        buffer_free(buf);
        context_free(ctx);
    }
    for (int o : owner)
        if (o < 0) fail("a tensor was dealt to no rank");
    gguf_close(meta);
    gguf_close(full);
}

// Frozen quantized weights on the packed-weight buffer type (CUDA<i>_Q): nn::Linear's forward and
// the gradient of its input through train.cpp's own autograd, with W's packed GGUF blocks decoded
// inside the GEMM. Compared with (a) the same graph on the CUDA device with W as an ordinary F32
// tensor (dequantized on load): bit for bit, since the dequant-in-prologue GEMM and the F32 GEMM
// take the same tile and split-K plan on bit-identical weights; (b) the CPU device with the
// reference loader: normwise 1e-5. Device memory: the packed weight takes its blocks' bytes, not
// its F32 bytes.
struct PackedRun {
    std::vector<float> y, dx, w_head;
    size_t             weight_bytes = 0;  // device memory the loaded weight took
};

size_t device_free(Device* d) { return d->props().memory_free; }

PackedRun packed_linear(Device* dev, int mode, const GgufFile* meta, const GgufFile* full, const char* path,
                        const char* name, int64_t tokens) {
    // mode 0: packed buffer on the CUDA device; 1: F32 weight on the CUDA device; 2: CPU device
    PackedRun r;
    Context* wctx = context_new(1 << 16);
    Tensor*  W    = gguf_new_tensor(wctx, meta, name, TYPE_F32);
    const size_t free0 = mode < 2 ? device_free(dev) : 0;
    Buffer* wbuf = buffer_alloc_ctx_tensors(wctx, mode == 0 ? cuda_packed_buffer_type(0) : dev->default_buffer_type());
    const bool loaded = mode < 2 ? cuda_gguf_load_tensor(meta, path, name, W) : gguf_load_tensor(full, name, W);
    if (!loaded) fail(std::string("loading ") + name);
    if (mode < 2) r.weight_bytes = free0 - device_free(dev);
    Context* ctx = context_new(1 << 22);
    Graph*   g   = graph_new(ctx);
    Linear   lin;
    linear_init_weight(ctx, &lin, W, nullptr);
    tensor_clear_param(W);  // frozen: no gradient for the quantized weight
    Tensor* X = new_tensor_2d(ctx, TYPE_F32, W->ne[0], tokens);
    tensor_set_param(X);
    Tensor* y = linear_forward(ctx, &lin, X);
    Tensor* G = new_tensor_2d(ctx, TYPE_F32, y->ne[0], y->ne[1]);
    Tensor* loss = sum(ctx, mul(ctx, y, G));
    tensor_set_loss(loss);
    graph_build_forward_expand(ctx, g, loss);
    graph_build_backward_expand(g);
    if (const Tensor* bad = graph_first_unsupported(g, dev)) fail(std::string("preflight: ") + op_name(bad->op));
    Buffer* buf = buffer_alloc_ctx_tensors(ctx, dev->default_buffer_type());
    const auto xv = gauss((size_t) tensor_nelements(X), 31), gv = gauss((size_t) tensor_nelements(G), 32, 1e-2f);
    tensor_set(X, xv.data(), 0, xv.size() * 4);
    tensor_set(G, gv.data(), 0, gv.size() * 4);
    graph_reset(g);
    dev->graph_compute(g);
    r.y.resize((size_t) tensor_nelements(y));
    tensor_get(y, r.y.data(), 0, r.y.size() * 4);
    Tensor* gx = graph_get_grad_acc(g, X);
    r.dx.resize((size_t) tensor_nelements(gx));
    tensor_get(gx, r.dx.data(), 0, r.dx.size() * 4);
    r.w_head.resize((size_t) std::min<int64_t>(tensor_nelements(W), 4096 + 37));
    tensor_get(W, r.w_head.data(), 0, r.w_head.size() * 4);  // on the packed buffer: dequantized on read
    buffer_free(buf);
    graph_free(g);
    context_free(ctx);
    buffer_free(wbuf);
    context_free(wctx);
    return r;
}

void packed_weights(Device* cpu, Device* cuda, const char* path, int64_t tokens) {
    std::printf("  frozen quantized weights on %s (%s, %lld tokens)\n", cuda_packed_buffer_type(0)->name(), path,
                (long long) tokens);
    GgufFile* meta = gguf_open(path, false);
    GgufFile* full = gguf_open(path, true);
    if (meta == nullptr || full == nullptr) {
        fail("gguf_open failed");
        return;
    }
    auto same_bits = [](const std::vector<float>& a, const std::vector<float>& b) {
        return a.size() == b.size() && std::memcmp(a.data(), b.data(), a.size() * 4) == 0;
    };
    for (int64_t i = 0; i < gguf_tensor_count(meta); ++i) {
        const GgufTensorInfo* info = gguf_tensor_info(meta, i);
        const PackedRun pk = packed_linear(cuda, 0, meta, full, path, info->name, tokens);
        const PackedRun f32 = packed_linear(cuda, 1, meta, full, path, info->name, tokens);
        const std::string n = std::string(info->name) + " (" + type_name(info->type) + ")";
        if (!same_bits(pk.y, f32.y) || !same_bits(pk.dx, f32.dx)) fail(n + ": packed path differs from the F32 device path");
        else std::printf("    [ OK ] %-34s y and dX bit-identical to the F32 device path\n", n.c_str());
        // the CPU device (single-threaded reference kernels) on the weights small enough for it
        const int64_t cpu_tokens = std::min<int64_t>(tokens, 64);
        if (gguf_tensor_nelements(meta, i) <= (int64_t(1) << 23)) {
            const PackedRun pk_small = cpu_tokens == tokens ? pk : packed_linear(cuda, 0, meta, full, path, info->name, cpu_tokens);
            const PackedRun ref = packed_linear(cpu, 2, meta, full, path, info->name, cpu_tokens);
            if (!same_bits(pk_small.w_head, ref.w_head))
                fail(n + ": tensor_get of the packed weight differs from the reference loader");
            compare((n + " y vs CPU").c_str(), pk_small.y, ref.y);
            compare((n + " dX vs CPU").c_str(), pk_small.dx, ref.dx);
        }
        const size_t f32_bytes = (size_t) gguf_tensor_nelements(meta, i) * 4;
        std::printf("    device memory of the loaded weight: packed %zu B, F32 %zu B (file %zu B packed)\n",
                    pk.weight_bytes, f32.weight_bytes, (size_t) info->nbytes);
        // the packed weight holds its blocks (rounded to the allocator's granularity), never F32 bytes
        if (f32_bytes >= (size_t(64) << 20) && !(pk.weight_bytes < info->nbytes + (size_t(4) << 20) && f32.weight_bytes >= f32_bytes))
            fail(n + ": the packed weight took more device memory than its blocks");
    }
    // what the device refuses on a packed weight: any op other than mul_mat reading it
    {
        const GgufTensorInfo* info = gguf_tensor_info(meta, 0);
        Context* wctx = context_new(1 << 16);
        Tensor*  W    = gguf_new_tensor(wctx, meta, info->name, TYPE_F32);
        Buffer*  wbuf = buffer_alloc_ctx_tensors(wctx, cuda_packed_buffer_type(0));
        cuda_gguf_load_tensor(meta, path, info->name, W);
        Context* ctx = context_new(1 << 20);
        Graph*   g   = graph_new(ctx);
        Tensor*  s   = sum(ctx, sqr(ctx, W));
        graph_build_forward_expand(ctx, g, s);
        const Tensor* bad = graph_first_unsupported(g, cuda);
        if (bad == nullptr || bad->op != OP_SQR) fail("preflight accepted sqr of a packed weight");
        else std::printf("    [ OK ] %-34s preflight reports %s\n", "non-mul_mat reader of a packed W", op_name(bad->op));
        Graph* g2 = graph_new(ctx);
        Tensor* c = cont(ctx, transpose(ctx, W));
        graph_build_forward_expand(ctx, g2, c);
        const Tensor* bad2 = graph_first_unsupported(g2, cuda);
        if (bad2 == nullptr || bad2->op != OP_CONT) fail("preflight accepted cont of a packed weight");
        graph_free(g2);
        graph_free(g);
        context_free(ctx);
        buffer_free(wbuf);
        context_free(wctx);
    }
    gguf_close(meta);
    gguf_close(full);
}

// checkpoint_save / checkpoint_load (src/io/trc_checkpoint.cpp) of a model trained on the CUDA device:
// the reference's own functions, unchanged, over the CUDA buffers (tensor_get / set_tensor). The
// file written from the device is loaded onto a fresh CUDA model and onto a fresh CPU model; every
// parameter and AdamW state tensor must come back bit-identical on both, the optimizer step and
// learning rate restored, and one more step on each device must agree.
struct CkptModel {
    Context*   ctx = nullptr;
    Graph*     g = nullptr;
    Buffer*    buf = nullptr;
    Optimizer* opt = nullptr;
    Tensor*    W = nullptr;
    Tensor*    b = nullptr;
};

CkptModel ckpt_model(Device* dev) {
    constexpr int64_t IN = 128, OUT = 96, BATCH = 40;
    CkptModel m;
    m.ctx = context_new((size_t) 1 << 24);
    m.g   = graph_new(m.ctx);
    m.W   = new_tensor_2d(m.ctx, TYPE_F32, IN, OUT);
    m.b   = new_tensor_2d(m.ctx, TYPE_F32, OUT, 1);
    tensor_set_name(m.W, "lin.weight");
    tensor_set_name(m.b, "lin.bias");
    Tensor* x = new_tensor_2d(m.ctx, TYPE_F32, IN, BATCH);
    Tensor* y = new_tensor_2d(m.ctx, TYPE_F32, OUT, BATCH);
    tensor_set_param(m.W);
    tensor_set_param(m.b);
    Tensor* loss = scale(m.ctx, sum(m.ctx, sqr(m.ctx, sub(m.ctx, add(m.ctx, mul_mat(m.ctx, m.W, x), m.b), y))),
                         1.0f / (float) (OUT * BATCH));
    tensor_set_loss(loss);
    graph_build_forward_expand(m.ctx, m.g, loss);
    graph_build_backward_expand(m.g);
    m.buf = buffer_alloc_ctx_tensors(m.ctx, dev->default_buffer_type());
    const auto vw = gauss((size_t) (IN * OUT), 41, 0.05f), vb = gauss((size_t) OUT, 42, 0.1f);
    const auto vx = gauss((size_t) (IN * BATCH), 43), vy = gauss((size_t) (OUT * BATCH), 44);
    tensor_set(m.W, vw.data(), 0, vw.size() * 4);
    tensor_set(m.b, vb.data(), 0, vb.size() * 4);
    tensor_set(x, vx.data(), 0, vx.size() * 4);
    tensor_set(y, vy.data(), 0, vy.size() * 4);
    Tensor* params[2] = {m.W, m.b};
    AdamwOptions o;
    o.lr = 1e-2f;
    m.opt = optim_adamw_new(m.ctx, params, 2, o);
    optim_alloc_state(m.opt);
    return m;
}

void ckpt_step(Device* dev, CkptModel& m) {
    graph_reset(m.g);
    dev->graph_compute(m.g);
    optim_step(m.opt);
}

std::vector<std::vector<float>> ckpt_tensors(const CkptModel& m) {
    std::vector<std::vector<float>> out;
    std::vector<Tensor*> ts = {m.W, m.b};
    for (int64_t i = 0; i < optim_state_count(m.opt); ++i) ts.push_back(optim_state(m.opt, i));
    for (Tensor* t : ts) {
        std::vector<float> v((size_t) tensor_nelements(t));
        tensor_get(t, v.data(), 0, v.size() * 4);
        out.push_back(std::move(v));
    }
    return out;
}

void ckpt_free(CkptModel& m) {
    optim_free(m.opt);
    buffer_free(m.buf);
    graph_free(m.g);
    context_free(m.ctx);
}

void checkpoint_roundtrip(Device* cpu, Device* cuda, const char* path) {
    std::printf("  checkpoint_save / checkpoint_load on the CUDA device (%s)\n", path);
    CkptModel src = ckpt_model(cuda);
    for (int s = 0; s < 3; ++s) ckpt_step(cuda, src);
    CheckpointItems items;
    items.optimizer = src.opt;
    if (!checkpoint_save(path, items, "dropin")) {
        fail("checkpoint_save from the CUDA device");
        return;
    }
    const auto saved = ckpt_tensors(src);
    CkptModel on_cuda = ckpt_model(cuda), on_cpu = ckpt_model(cpu);
    CheckpointItems a, b;
    a.optimizer = on_cuda.opt;
    b.optimizer = on_cpu.opt;
    if (!checkpoint_load(path, a) || !checkpoint_load(path, b)) {
        fail("checkpoint_load");
        return;
    }
    const auto got_cuda = ckpt_tensors(on_cuda), got_cpu = ckpt_tensors(on_cpu);
    bool same = got_cuda.size() == saved.size() && got_cpu.size() == saved.size();
    for (size_t i = 0; same && i < saved.size(); ++i)
        same = std::memcmp(got_cuda[i].data(), saved[i].data(), saved[i].size() * 4) == 0 &&
               std::memcmp(got_cpu[i].data(), saved[i].data(), saved[i].size() * 4) == 0;
    if (!same) fail("checkpoint tensors differ between the saved model, the CUDA load and the CPU load");
    else std::printf("    [ OK ] %-34s %zu tensors bit-identical (CUDA load = CPU load = saved)\n", "checkpoint round trip",
                     saved.size());
    if (optim_step_count(on_cuda.opt) != optim_step_count(src.opt) || optim_step_count(on_cpu.opt) != optim_step_count(src.opt) ||
        optim_get_lr(on_cuda.opt) != optim_get_lr(src.opt))
        fail("optimizer step / learning rate not restored");
    ckpt_step(cuda, on_cuda);
    ckpt_step(cpu, on_cpu);
    const auto next_cuda = ckpt_tensors(on_cuda), next_cpu = ckpt_tensors(on_cpu);
    compare("step after resume: W (CUDA vs CPU)", next_cuda[0], next_cpu[0], false, 5e-5);
    compare("step after resume: b (CUDA vs CPU)", next_cuda[1], next_cpu[1], false, 5e-5);
    ckpt_free(src);
    ckpt_free(on_cuda);
    ckpt_free(on_cpu);
}

// Bandwidth of checkpoint_load onto the CUDA device, and of plain tensor_set / tensor_get, for a
// model of six 2048 x 4096 F32 parameters with AdamW states (a 576 MB checkpoint). train.cpp's
// checkpoint_load reads the whole file and uploads every tensor with tensor_set, which the CUDA
// buffer runs through its pinned chunks. Prints the rates; checks the loaded tensors bit-identical.
void checkpoint_bandwidth(Device* cuda, const char* path) {
    constexpr int kParams = 6;
    constexpr int64_t R = 2048, C = 4096;
    auto make = [&](std::vector<Tensor*>& ps, Context*& ctx, Buffer*& buf, Optimizer*& opt) {
        ctx = context_new((size_t) 1 << 20);
        for (int i = 0; i < kParams; ++i) {
            Tensor* t = new_tensor_2d(ctx, TYPE_F32, C, R);
            tensor_set_name(t, "big.%d", i);
            tensor_set_param(t);
            ps.push_back(t);
        }
        buf = buffer_alloc_ctx_tensors(ctx, cuda->default_buffer_type());
        opt = optim_adamw_new(ctx, ps.data(), kParams, AdamwOptions{});
        optim_alloc_state(opt);
    };
    std::vector<Tensor*> src, dst;
    Context *c0 = nullptr, *c1 = nullptr;
    Buffer *b0 = nullptr, *b1 = nullptr;
    Optimizer *o0 = nullptr, *o1 = nullptr;
    make(src, c0, b0, o0);
    const size_t n = (size_t) (R * C);
    std::vector<float> host(n);
    using clk = std::chrono::steady_clock;
    double set_s = 0, get_s = 0;
    tensor_set(src[0], host.data(), 0, n * 4);  // first staged copy: creates the pinned chunks and copy threads
    for (int i = 0; i < kParams; ++i) {
        for (size_t j = 0; j < n; ++j) host[j] = (float) ((i * 1315423911u + j * 2654435761u) % 1000003) * 1e-6f;
        const auto t0 = clk::now();
        tensor_set(src[(size_t) i], host.data(), 0, n * 4);
        set_s += std::chrono::duration<double>(clk::now() - t0).count();
    }
    CheckpointItems items;
    items.optimizer = o0;
    if (!checkpoint_save(path, items, "bandwidth")) {
        fail("checkpoint_save (bandwidth case)");
        return;
    }
    make(dst, c1, b1, o1);
    CheckpointItems items1;
    items1.optimizer = o1;
    const auto t0 = clk::now();
    const bool ok = checkpoint_load(path, items1);
    const double load_s = std::chrono::duration<double>(clk::now() - t0).count();
    bool same = ok;
    std::vector<float> a(n), b(n);
    for (int i = 0; same && i < kParams; ++i) {
        const auto g0 = clk::now();
        tensor_get(dst[(size_t) i], a.data(), 0, n * 4);
        get_s += std::chrono::duration<double>(clk::now() - g0).count();
        tensor_get(src[(size_t) i], b.data(), 0, n * 4);
        same = std::memcmp(a.data(), b.data(), n * 4) == 0;
    }
    const double bytes = 3.0 * kParams * (double) n * 4;  // parameters + AdamW m and v
    if (!same) fail("checkpoint_load of the 576 MB model differs");
    else std::printf("    [ OK ] %-34s %.0f MB in %.3f s = %.1f GB/s (file read + upload); tensor_set %.1f GB/s, "
                     "tensor_get %.1f GB/s\n", "checkpoint_load onto CUDA", bytes / 1e6, load_s, bytes / load_s / 1e9,
                     kParams * (double) n * 4 / set_s / 1e9, kParams * (double) n * 4 / get_s / 1e9);
    optim_free(o0);
    optim_free(o1);
    buffer_free(b0);
    buffer_free(b1);
    context_free(c0);
    context_free(c1);
}

}  // namespace

int main(int argc, char** argv) {
    const std::string mode = argc > 1 ? argv[1] : "all";
    const int n = cuda_register_devices();
    Device* cuda = device_by_type(DeviceType::GPU);
    Device* cpu  = device_cpu();
    if (n == 0 || cuda == nullptr || cpu == nullptr) {
        std::printf("no CUDA device registered\n");
        return 77;
    }
    std::printf("devices: %zu registered; CUDA device: %s (%s)\n", device_count(), cuda->props().name.c_str(),
                cuda->props().description.c_str());
    if (mode == "alloc_fail") {
        // TRC_CUDA_FAIL_ALLOC=1 in the environment: the first buffer allocation fails and the core
        // aborts with its need/available message (src/core/trc_backend_reg.cpp:248-264).
        Context* ctx = context_new(1 << 16);
        new_tensor_2d(ctx, TYPE_F32, 1024, 1024);
        buffer_alloc_ctx_tensors(ctx, cuda->default_buffer_type());
        std::printf("allocation unexpectedly succeeded\n");
        return 0;
    }
    if (mode == "packed" && argc > 2) {
        packed_weights(cpu, cuda, argv[2], argc > 3 ? std::atoll(argv[3]) : 64);
        std::printf("%s: %d failure(s)\n", g_failures == 0 ? "PASS" : "FAIL", g_failures);
        return g_failures == 0 ? 0 : 1;
    }
    if (mode == "checkpoint" && argc > 2) {
        checkpoint_roundtrip(cpu, cuda, argv[2]);
        checkpoint_bandwidth(cuda, argv[2]);
        std::printf("%s: %d failure(s)\n", g_failures == 0 ? "PASS" : "FAIL", g_failures);
        return g_failures == 0 ? 0 : 1;
    }
    if (mode == "shard" && argc > 2) {
        for (int world : {1, 2, 3}) gguf_sharded_load(cuda, argv[2], world);
        std::printf("%s: %d failure(s)\n", g_failures == 0 ? "PASS" : "FAIL", g_failures);
        return g_failures == 0 ? 0 : 1;
    }
    conformance_matmul(cpu, cuda);
    training_steps(cpu, cuda);
    training_loops(cpu, cuda);
    if (argc > 2) gguf_warm_start(cpu, cuda, argv[2]);
    std::printf("%s: %d failure(s)\n", g_failures == 0 ? "PASS" : "FAIL", g_failures);
    return g_failures == 0 ? 0 : 1;
}
