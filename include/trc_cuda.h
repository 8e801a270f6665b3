/* trc_cuda.h -- C ABI of libtrc_cuda.so: B200 (sm_100a) kernels for train.cpp's quantized-weight
 * hot path (GGUF legacy-block dequantization + ggml-semantics F32 mul_mat and the graph ops of its
 * composed backward).
 *
 * This is the drop-in boundary. train.cpp's abstract backend interface
 * (include/traincpp/trc_backend.h:33-88: BufferType / Buffer / Device) is implemented in C++ by
 * train.cpp_b200/backend/trc_cuda_backend.cpp, which calls only the functions below. Each entry
 * point names the reference code it replaces. Paths are relative to the train.cpp source tree.
 *
 * Conventions
 *   - Plain C: pointers, sizes, and a `void* stream` that is a cudaStream_t (NULL = legacy stream).
 *   - Every function returns an int status: TRC_CUDA_OK (0) or a negative TRC_CUDA_E* code. No
 *     function aborts; the C++ backend maps a failure to train.cpp's TRC_ABORT with the message of
 *     trc_cuda_status_string(), mirroring how the reference backends report fatal errors
 *     (src/core/trc_impl.h:118-125).
 *   - Device pointers are device-local memory of the current CUDA device. Kernels are enqueued on
 *     `stream` and return without synchronising, except where a function says otherwise.
 *   - Tensor views follow ggml: ne[0] is the innermost extent, nb[] are byte strides
 *     (include/traincpp/trc_tensor.h:1-5, 37-70).
 *   - There is no CPU fallback. Every compute entry point runs a kernel of this library.
 */
#ifndef TRC_CUDA_H
#define TRC_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TRC_CUDA_ABI_VERSION 1

/* ------------------------------------------------------------------ status codes */
enum {
    TRC_CUDA_OK           = 0,
    TRC_CUDA_EINVAL       = -1, /* null pointer, bad size, or a shape rule of the reference violated */
    TRC_CUDA_EUNSUPPORTED = -2, /* element type or layout this library does not compute */
    TRC_CUDA_EDEVICE      = -3, /* a kernel hit its wait limit; see trc_cuda_device_error() */
    TRC_CUDA_ECUDA        = -4, /* a CUDA runtime call failed; see trc_cuda_last_cuda_error() */
    TRC_CUDA_ENOMEM       = -5, /* a device allocation failed */
    TRC_CUDA_ETOOBIG      = -6  /* larger than the fixed static buffer of an allocation-free entry point */
};

/* ggml / GGUF type ids of the legacy quantized blocks (include/traincpp/trc_types.h:11-49). */
enum {
    TRC_CUDA_TYPE_F32  = 0,
    TRC_CUDA_TYPE_Q4_0 = 2,
    TRC_CUDA_TYPE_Q4_1 = 3,
    TRC_CUDA_TYPE_Q5_0 = 6,
    TRC_CUDA_TYPE_Q5_1 = 7,
    TRC_CUDA_TYPE_Q8_0 = 8
};

/* One ggml tensor view in device memory (the fields of Tensor that the kernels need:
 * include/traincpp/trc_tensor.h:37-70; data = buffer base + Tensor::data_offset). */
typedef struct trc_cuda_view {
    void*   data;  /* device address of element (0,0,0,0) */
    int64_t ne[4]; /* extents, ne[0] innermost */
    int64_t nb[4]; /* byte strides */
} trc_cuda_view;

/* ------------------------------------------------------------------ library / diagnostics */

/* TRC_CUDA_ABI_VERSION of the loaded library. */
int trc_cuda_abi_version(void);

/* Human-readable text for a status code (static storage). */
const char* trc_cuda_status_string(int status);

/* The cudaError_t of the last failed CUDA runtime call in this thread (0 if none). */
int trc_cuda_last_cuda_error(void);

/* Reads (and, if reset != 0, clears) the device-side error word of the current device. A nonzero
 * *code means a kernel gave up a bounded wait; its results are not valid. Synchronous. */
int trc_cuda_device_error(int* code, int reset);

/* Failure-detection self-test: launches one CTA that waits, with the library's bounded mbarrier
 * wait, on a barrier nothing arrives on. After limit_ns (at most 5 s) the wait gives up, the device
 * error word records 8 (TRC_DEVERR_SELFTEST) and the kernel returns: *completed = 0 shows that the
 * wait ran out, and the context stays usable. No fault, trap or hang is involved. Synchronous. */
int trc_cuda_selftest_wait_timeout(uint64_t limit_ns, int* completed);

/* Number of kernels this library has launched in this process (all devices). The bench reports
 * the difference across its timed region as the count of native launches. */
uint64_t trc_cuda_launch_count(void);

/* Number of SMs of the current device (148 on B200). */
int trc_cuda_sm_count(void);

/* ------------------------------------------------------------------ GGUF legacy-block dequant */

/* Bytes of one 32-weight block: Q4_0 18, Q4_1 20, Q5_0 22, Q5_1 24, Q8_0 34; 0 for other types.
 * Replaces the block-size column of the type table (src/core/trc_types.cpp:22-32). */
size_t trc_cuda_block_bytes(int type);

/* Dequantize n_blocks consecutive blocks at `blocks` into 32*n_blocks floats at `out`, bit-exact
 * with the reference. Replaces the Q* branch of gguf_tensor_to_f32 (src/io/trc_gguf.cpp:1040-1044)
 * -> dequantize_q4_0 .. dequantize_q8_0 (src/io/trc_gguf.cpp:320-417).
 * EUNSUPPORTED for a type that is not one of the five legacy formats (the reference rejects the
 * others too: src/io/trc_gguf.cpp:1045-1047). */
int trc_cuda_dequant(int type, const void* blocks, int64_t n_blocks, float* out, void* stream);

/* One tensor of a batched dequantization. */
typedef struct trc_cuda_dequant_job {
    const void* blocks;   /* device address of the packed blocks */
    float*      out;      /* device address of 32*n_blocks floats */
    int64_t     n_blocks; /* >= 0 */
    int32_t     type;     /* TRC_CUDA_TYPE_Q* */
    int32_t     reserved;
} trc_cuda_dequant_job;

/* Dequantize many tensors (a whole model's shard) in as few launches as possible. `jobs` is a
 * HOST array; it is passed to the kernel by value, 256 jobs per launch. Equivalent to calling
 * gguf_load_tensor (src/io/trc_gguf.cpp:1051-1094) for each tensor, minus the host F32 copy. */
int trc_cuda_dequant_many(const trc_cuda_dequant_job* jobs, int n_jobs, void* stream);

/* Dequantize-and-all-gather: trc_cuda_dequant_many whose every output float is also written, in
 * the same launch, at the same offset of up to 8 peer GPUs' buffers over NVLink. Each job's `out`
 * lies in the local buffer starting at `local_base`; its copy on peer p is at
 * peer_bases[p] + (out - local_base), peer_bases being the peers' buffers mapped into this
 * process by trc_cuda_rt_ipc_open (plain peer stores, no multicast). With every rank
 * dequantizing its own rows of a tensor, one call per rank leaves the whole F32 tensor on every
 * GPU: the NCCL all-gather a sharded dequantized tensor would otherwise need, fused into the
 * dequant kernel's stores. The copies are complete when the launch is: synchronize the stream,
 * then barrier across the ranks before a peer reads. EINVAL when n_peers is outside 0..8, a peer
 * base is null or not a multiple of 16 bytes away from local_base, or an output lies below
 * local_base. */
int trc_cuda_dequant_many_to_peers(const trc_cuda_dequant_job* jobs, int n_jobs, const void* local_base,
                                   void* const* peer_bases, int n_peers, void* stream);

/* Device-side gguf_load_tensor for a quantized tensor with an F32 destination
 * (src/io/trc_gguf.cpp:1082-1089): copies the packed blocks from HOST memory `host_blocks` into
 * the caller's device staging buffer (>= n_blocks*block_bytes bytes, 16-byte aligned), then
 * dequantizes into `out`. Only the packed bytes cross PCIe (the reference copies the 4-8x larger
 * F32 result). Pinned host memory makes the copy asynchronous; pageable memory is also accepted.
 * Tensors of 16 MB packed or more are uploaded in chunks of up to 32 MB (the last two about 2 MB
 * and 1 MB) on the library's own copy stream, and `stream` dequantizes each chunk once it has
 * landed, so copy and dequant overlap.
 * The first chunk waits for the work already queued on `stream`, so the staging buffer may be
 * reused by consecutive calls on one stream. */
int trc_cuda_load_quant(int type, const void* host_blocks, int64_t n_blocks, void* staging, float* out,
                        void* stream);

/* Allocation-free variant of trc_cuda_load_quant, for callers that cannot call cudaMalloc: code
 * that must not grow device memory (a process whose device memory is owned by another allocator or
 * has a fixed budget, or a loader running while other work owns the allocator). It needs no
 * caller staging buffer: the packed blocks are staged in a fixed array inside the library, a
 * file-scope static __device__ array of TRC_CUDA_STATIC_STAGING_BYTES (64 MiB). The call itself
 * allocates nothing and calls no allocating routine.
 *   - When the memory is taken: the array is part of the library's device code, which CUDA loads
 *     on a device at the library's first kernel launch or symbol lookup there (lazy module loading,
 *     the default since CUDA 12.2), or at process start under CUDA_MODULE_LOADING=EAGER. From then
 *     on that GPU holds the 64 MiB until the process exits. A caller with a fixed budget makes one
 *     call per device before fixing it; a call with n_blocks = 0 is enough (it loads the module
 *     and copies nothing). Make that first call before any stream capture begins.
 *   - Tensors whose packed bytes exceed TRC_CUDA_STATIC_STAGING_BYTES are rejected with
 *     TRC_CUDA_ETOOBIG before any device work.
 *   - Every call looks up the array's address on the current device (cudaGetSymbolAddress, a host
 *     lookup once the module is loaded), so a device reset that re-creates the context is safe.
 *   - All calls share the one array per device and it keeps the last call's bytes; each call
 *     overwrites the bytes it uses before reading them, so nothing needs clearing. Calls whose
 *     copies or kernels overlap on the GPU (different streams without ordering) race on the array.
 * This entry point has no counterpart in the reference, which dequantizes on the host. */
#define TRC_CUDA_STATIC_STAGING_BYTES ((size_t) 64 << 20)
int trc_cuda_load_quant_static(int type, const void* host_blocks, int64_t n_blocks, float* out, void* stream);

/* ------------------------------------------------------------------ mul_mat */

enum {
    TRC_CUDA_MM_ACCUMULATE = 1u, /* d += a*b instead of d = a*b */
    TRC_CUDA_MM_SIMT       = 2u, /* force the fp32 SIMT kernel (exact reference summation order);
                                    the default picks the tcgen05 3xTF32 kernel when the layout allows */
    TRC_CUDA_MM_ONE_CTA    = 4u, /* tcgen05 kernel with one CTA per 128 x 256 tile (cta_group::1); the
                                    default runs 256 x 256 tiles on CTA pairs (cta_group::2, a cluster
                                    of two SMs sharing the B tile) when M spans more than 128 rows */
    TRC_CUDA_MM_NO_PRETAIL = 8u, /* fused trc_cuda_mul_mat_q whose split warps load the packed words
                                    from global memory (single CTAs, or packed rows that are not
                                    16-byte aligned): split B into TF32 head and tail inside every tile
                                    instead of once before the launch (by default that kernel computes
                                    B's tails in one pass into stream-ordered scratch when B is reused
                                    by two or more row tiles; same results). The TMA-staged fused
                                    kernel always splits B in the loop */
    TRC_CUDA_MM_FUSED      = 16u, /* trc_cuda_mul_mat_q: always run the fused dequant-in-prologue
                                     kernel, which allocates no copy of W (the default wherever the
                                     packed bytes can be staged by TMA; see trc_cuda_mul_mat_q) */
    TRC_CUDA_MM_TWO_STEP   = 32u  /* trc_cuda_mul_mat_q: dequantize W into stream-ordered scratch, then
                                     run the F32 kernel (same results as the fused kernel) */
};

/* ggml mul_mat: for every plane (i2, i3) of b,
 *     d[i, j, i2, i3] (+)= sum_k a[k, i, i2 % a.ne2, i3 % a.ne3] * b[k, j, i2, i3]
 * with a.ne0 == b.ne0 == K, d.ne = {a.ne1, b.ne1, b.ne2, b.ne3}, b.ne2 % a.ne2 == 0 and
 * b.ne3 % a.ne3 == 0 (the rules of the constructor, src/ops/trc_ops.cpp:366-385). Any byte strides
 * are accepted, including the transposed views the composed backward builds
 * (src/core/trc_autograd.cpp:487-503). F32 in, F32 out.
 * Replaces compute_mul_mat (src/backends/cpu/trc_cpu_ops.cpp:182-216).
 * Accuracy: the tcgen05 kernel splits each operand into a TF32 head and tail (3xTF32) and stays
 * within 1e-5 normwise (max|gpu - cpu| / max|cpu|) of the reference. The SIMT kernel reproduces
 * the reference's summation bit for bit. */
int trc_cuda_mul_mat(const trc_cuda_view* a, const trc_cuda_view* b, const trc_cuda_view* d, uint32_t flags,
                     void* stream);

/* d = repeat_back(mul_mat(a, b)) in one kernel: d may have fewer planes than b (b.ne2 % d.ne2 == 0,
 * b.ne3 % d.ne3 == 0) and output plane (q2, q3) receives the sum of the products of every source
 * plane (p2, p3) with p2 % d.ne2 == q2 and p3 % d.ne3 == q3. This is the dA of a broadcast mul_mat in
 * the composed backward (src/core/trc_autograd.cpp:490-496: mul_mat, transpose, repeat_back) without
 * the intermediate; with d a transposed view and TRC_CUDA_MM_ACCUMULATE it also performs the
 * following acc into the parameter's grad_acc. Replaces compute_mul_mat + compute_repeat_back
 * (src/backends/cpu/trc_cpu_ops.cpp:182-216, 932-951). The SIMT kernel keeps the reference's order
 * and rounding (each plane's product rounded, then added in plane order) bit for bit; the tcgen05
 * kernel accumulates the planes in its K loop, within the same 1e-5 normwise bar. */
int trc_cuda_mul_mat_repeat_back(const trc_cuda_view* a, const trc_cuda_view* b, const trc_cuda_view* d,
                                 uint32_t flags, void* stream);

enum { TRC_CUDA_KERNEL_TCGEN05 = 1, TRC_CUDA_KERNEL_SIMT = 2 };

/* Which kernel trc_cuda_mul_mat would run for these views and flags: TRC_CUDA_KERNEL_TCGEN05 (the
 * TMA-fed 3xTF32 tensor-core kernel) or TRC_CUDA_KERNEL_SIMT; a negative status if the call would be
 * rejected. Host-only; launches nothing. */
int trc_cuda_mul_mat_kernel(const trc_cuda_view* a, const trc_cuda_view* b, const trc_cuda_view* d, uint32_t flags);

/* dequant + mul_mat: like trc_cuda_mul_mat, but operand a is a frozen quantized weight held as
 * packed blocks. The weight's logical F32 tensor W has ne = {w_ne0, w_ne1, 1, 1} (blocks run along
 * ne0, rows are contiguous). a_transposed = 0 uses a = W, a_transposed = 1 uses a = transpose(W)
 * (the dX = W^T dY product of the backward). Two implementations, with the same results (W
 * dequantized bit-exactly, then the same tile and split-K plan of the tensor-core kernel):
 *   - fused: the GEMM's split warps decode the blocks into shared memory, and the F32 weight never
 *     exists in HBM. On CTA pairs (more than 128 rows of a) with 16-byte aligned packed rows the
 *     producer stages each stage's packed bytes by TMA; on B200 (Q5_0 4096 x 14336, 2048
 *     columns) that kernel is faster than the two steps below (forward ~228 vs ~220 TFLOP/s, dX
 *     ~235 vs ~222). The default wherever it applies, below 1024 columns, with TRC_CUDA_MM_FUSED,
 *     and when the scratch below cannot be allocated;
 *   - two steps: W is dequantized into stream-ordered scratch from the device's memory pool
 *     (w_ne0 * w_ne1 * 4 bytes, freed on the stream), then trc_cuda_mul_mat runs. The default from
 *     1024 columns on where the fused kernel cannot stage the packed bytes by TMA (there the two
 *     steps are faster), and with TRC_CUDA_MM_TWO_STEP. With TRC_CUDA_MM_SIMT the product is the
 *     SIMT kernel's, so the whole call is bit-exact with the reference. */
int trc_cuda_mul_mat_q(int type, const void* w_blocks, int64_t w_ne0, int64_t w_ne1, int a_transposed,
                       const trc_cuda_view* b, const trc_cuda_view* d, uint32_t flags, void* stream);

/* ------------------------------------------------------------------ graph ops of the backward */

/* dst = src (same shape, any strides). Replaces compute_dup for OP_CONT / OP_DUP
 * (src/backends/cpu/trc_cpu_ops.cpp:219-236). Bit-exact. */
int trc_cuda_cont(const trc_cuda_view* src, const trc_cuda_view* dst, void* stream);

/* In-place acc: for every element (i0..i3) of b,
 *     dst_bytes[offset + i0*4 + i1*nb1 + i2*nb2 + i3*nb3] += b[i0, i1, i2, i3]
 * where dst points at the contiguous destination tensor of total size dst_bytes bytes. The caller
 * guarantees the region fits (the constructor asserts it, src/core/trc_tensor.cpp:322-360).
 * Replaces compute_acc with inplace=1 (src/backends/cpu/trc_cpu_ops.cpp:954-998). Bit-exact. */
int trc_cuda_acc(void* dst, int64_t dst_bytes, const trc_cuda_view* b, int64_t nb1, int64_t nb2, int64_t nb3,
                 int64_t offset, void* stream);

/* dst (contiguous) = sum of src over the dimensions it repeats: element i of src adds into element
 * (i0 % dst.ne0, ..., i3 % dst.ne3), in the reference's order. Replaces compute_repeat_back
 * (src/backends/cpu/trc_cpu_ops.cpp:932-951). Bit-exact. */
int trc_cuda_repeat_back(const trc_cuda_view* src, const trc_cuda_view* dst, void* stream);

/* dst = src tiled to dst's shape (index i_d % src.ne_d). Replaces compute_repeat (OP_REPEAT). */
int trc_cuda_repeat(const trc_cuda_view* src, const trc_cuda_view* dst, void* stream);

enum { TRC_CUDA_BIN_ADD = 0, TRC_CUDA_BIN_SUB = 1, TRC_CUDA_BIN_MUL = 2, TRC_CUDA_BIN_DIV = 3 };

/* dst = a (op) b with b broadcast onto a's shape by index modulo (ggml_can_repeat(b, a)).
 * Replaces the F32 cases of OP_ADD / OP_SUB / OP_MUL / OP_DIV. Bit-exact. */
int trc_cuda_binary(int op, const trc_cuda_view* a, const trc_cuda_view* b, const trc_cuda_view* dst, void* stream);

/* Bytes of device workspace trc_cuda_sum needs for a tensor of n elements (at most 8 KiB). */
size_t trc_cuda_sum_workspace_bytes(int64_t n);

/* *dst (one float, device) = sum of every element of src, accumulated in double like the
 * reference and rounded once to float. Deterministic two-pass reduction: the first pass writes one
 * partial per thread block into the caller's device `workspace` (>= trc_cuda_sum_workspace_bytes,
 * 8-byte aligned), the second pass adds the partials in a fixed order.
 * Replaces compute_sum (OP_SUM, src/backends/cpu/trc_cpu_ops.cpp:302-315); agrees with it within
 * double-precision summation error before the final rounding. */
int trc_cuda_sum(const trc_cuda_view* src, float* dst, void* workspace, size_t workspace_bytes, void* stream);

/* dst[0..n) = value. Replaces the host fill of Device::fill_tensors
 * (src/core/trc_backend_reg.cpp:539-544) for device-local F32 tensors. */
int trc_cuda_fill(float* dst, int64_t n, float value, void* stream);

/* ------------------------------------------------------------------ the rest of a training step
 * The graph ops a Linear training step emits besides mul_mat and its backward, for a model that
 * lives on the device: a loss's element-wise unaries, row sums, and the optimizer graph train.cpp
 * builds when parameters, gradients and states share one non-CPU device
 * (src/optim/trc_optim.cpp:330-420, 760-860). Results are bit-exact with the CPU backend except
 * trc_cuda_sum_sqr_acc (see there). */

enum {
    TRC_CUDA_UNARY_SQR = 0,   /* x * x                 fn_sqr   (src/backends/cpu/trc_cpu_ops.cpp:86) */
    TRC_CUDA_UNARY_SQRT = 1,  /* sqrt(x)               fn_sqrt  (:87) */
    TRC_CUDA_UNARY_ABS = 2,   /* |x|                   fn_abs   (:85) */
    TRC_CUDA_UNARY_NEG = 3,   /* -x                    fn_neg   (:84) */
    TRC_CUDA_UNARY_SGN = 4,   /* sign(x), 0 for 0/NaN  fn_sgn   (:93) */
    TRC_CUDA_UNARY_STEP = 5,  /* x > 0 ? 1 : 0         fn_step  (:94) */
    TRC_CUDA_UNARY_SCALE = 6  /* x * param             compute_scale (:139-149) */
};

/* dst = op(src) element by element (same ne; any strides). Replaces compute_unary / compute_scale
 * (src/backends/cpu/trc_cpu_ops.cpp:119-149) for OP_SQR, OP_SQRT, OP_ABS, OP_NEG, OP_SGN, OP_STEP,
 * OP_SCALE. */
int trc_cuda_unary(int op, const trc_cuda_view* src, const trc_cuda_view* dst, float param, void* stream);

/* dst[0, i1, i2, i3] = sum over i0 of src (take_mean: divided by src.ne0), each row summed in
 * double in index order and rounded once to float. Replaces compute_sum_rows_or_mean
 * (src/backends/cpu/trc_cpu_ops.cpp:317-333), OP_SUM_ROWS and OP_MEAN. */
int trc_cuda_sum_rows(const trc_cuda_view* src, const trc_cuda_view* dst, int take_mean, void* stream);

/* In-place AdamW on n contiguous floats; params6 (HOST) = {step_sz, bc2_sqrt, decay, beta1, beta2,
 * eps} as the optimizer writes them into the node's op_params. Replaces compute_opt_step_adamw
 * (src/backends/cpu/trc_cpu_ops.cpp:1506-1538), OP_OPT_STEP_ADAMW. */
int trc_cuda_opt_step_adamw(float* param, const float* grad, float* m, float* v, int64_t n, const float* params6,
                            void* stream);

/* In-place SGD on n contiguous floats; params6 (HOST) = {lr, momentum, dampening, weight_decay,
 * nesterov, is_first}. momentum may be null when params6[1] == 0. Replaces compute_opt_step_sgd
 * (src/backends/cpu/trc_cpu_ops.cpp:1540-1573), OP_OPT_STEP_SGD. */
int trc_cuda_opt_step_sgd(float* param, const float* grad, float* momentum, int64_t n, const float* params6,
                          void* stream);

/* acc[0] += (float) sum of (double) a[i]^2 over n contiguous floats. Replaces compute_sum_sqr_acc
 * (src/backends/cpu/trc_cpu_ops.cpp:1578-1591), OP_SUM_SQR_ACC. The double sum is taken in a parallel
 * order: it equals the reference's sequential one after rounding to float except when the two
 * double sums round to different floats (then they differ by one float ulp). workspace: device
 * memory of at least trc_cuda_sum_sqr_workspace_bytes(n) bytes. */
size_t trc_cuda_sum_sqr_workspace_bytes(int64_t n);
int    trc_cuda_sum_sqr_acc(float* acc, const float* a, int64_t n, void* workspace, size_t workspace_bytes,
                            void* stream);

/* a[i] *= min(1, max_norm / (sqrt(norm[0]) + eps)) over n contiguous floats, norm read on the device.
 * Replaces compute_clip_scale_inplace (src/backends/cpu/trc_cpu_ops.cpp:1594-1611),
 * OP_CLIP_SCALE_INPLACE. */
int trc_cuda_clip_scale_inplace(float* a, int64_t n, const float* norm, float max_norm, float eps, void* stream);

/* ------------------------------------------------------------------ measurement support
 * The dequant kernel's memory traffic without its arithmetic, to measure what HBM delivers for that
 * mix: reads n_in16 16-byte units from `in` and writes ratio * n_in16 units to `out` (each warp:
 * 512 contiguous bytes read, ratio x 512 contiguous bytes written, streaming stores). n_in16 must
 * be a multiple of 32, ratio 1..8, both pointers 16-byte aligned, `out` >= ratio * n_in16 * 16
 * bytes. bench.py reports the dequant's bandwidth as a fraction of this ceiling next to the copy
 * peak. */
int trc_cuda_stream_probe(const void* in, void* out, int64_t n_in16, int ratio, void* stream);

/* trc_cuda_stream_probe with the dequant kernel's store path: the copies are staged in shared memory
 * and written by bulk copies (cp.async.bulk), 3 CTAs per SM. Same output layout; n_in16 must be a
 * multiple of 256. */
int trc_cuda_stream_probe_bulk(const void* in, void* out, int64_t n_in16, int ratio, void* stream);

/* The tcgen05 kind::tf32 ceiling: one CTA per SM (cta_group = 1, 128 x 256 x 8 MMAs) or one CTA pair
 * per two SMs (cta_group = 2, 256 x 256 x 8 MMAs) issues `iters` K=16 steps of the 3xTF32 GEMM's
 * main loop -- three MMAs per K=8 from shared-memory operands into an fp32 TMEM accumulator -- with
 * no loads, operand split or epilogue. FLOPs per launch (each MMA counted):
 * iters x 6 x 2 x 128 x 256 x 8 x (number of CTAs). bench.py times it with CUDA events to state
 * every GEMM as a fraction of what the tensor pipe delivers here. iters in 1 .. 2^22. */
int trc_cuda_tf32_mma_probe(int cta_group, int iters, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TRC_CUDA_H */
