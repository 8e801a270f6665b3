// trc_internal.h -- host-side helpers shared by the .cu files of libtrc_cuda (not part of the ABI).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/trc_cuda.h"

namespace trc {

// A ggml view as the kernels take it (by value).
struct View4 {
    char*   data;
    int64_t ne[4];
    int64_t nb[4];
};

inline View4 to_view4(const trc_cuda_view& v) {
    View4 r;
    r.data = static_cast<char*>(v.data);
    for (int i = 0; i < 4; ++i) {
        r.ne[i] = v.ne[i];
        r.nb[i] = v.nb[i];
    }
    return r;
}

inline int64_t nelements(const trc_cuda_view& v) { return v.ne[0] * v.ne[1] * v.ne[2] * v.ne[3]; }

inline bool view_ok(const trc_cuda_view* v) {
    if (v == nullptr) return false;
    for (int i = 0; i < 4; ++i) {
        if (v->ne[i] < 0 || v->nb[i] < 0) return false;
    }
    return v->data != nullptr || nelements(*v) == 0;
}

inline bool view_contiguous(const trc_cuda_view& v) {
    int64_t expect = 4;
    for (int i = 0; i < 4; ++i) {
        if (v.ne[i] != 1 && v.nb[i] != expect) return false;
        expect *= v.ne[i];
    }
    return true;
}

// Launch bookkeeping: every kernel launch of the library goes through note_launch().
void note_launch(int n = 1);

// Records a failed CUDA call for trc_cuda_last_cuda_error() and returns TRC_CUDA_ECUDA.
int cuda_fail(cudaError_t e);

// Returns TRC_CUDA_OK, or records and maps the pending launch error.
int check_launch();

int sm_count_current();

// Keeps memory freed to the device's default pool (cudaFreeAsync) in the pool for reuse.
void retain_pool_once();

// trc_cuda_load_quant's single-copy path (arguments already checked): one host-to-device copy into
// `staging` and one dequant, both on stream s; creates no stream, event or allocation.
int load_quant_direct(int type, const void* host_blocks, int64_t n_blocks, void* staging, float* out,
                      cudaStream_t s);

// Per-library entry points implemented in the individual .cu files.
int dequant_jobs(const trc_cuda_dequant_job* jobs, int n_jobs, cudaStream_t stream);
int dequant_jobs_peers(const trc_cuda_dequant_job* jobs, int n_jobs, const void* local_base, void* const* peer_bases,
                       int n_peers, cudaStream_t stream);
int mul_mat_simt(const trc_cuda_view& a, const trc_cuda_view& b, const trc_cuda_view& d, bool accumulate,
                 cudaStream_t stream);
// Returns TRC_CUDA_EUNSUPPORTED when the layout cannot be fed by TMA (caller then uses SIMT).
// flags: TRC_CUDA_MM_ACCUMULATE, TRC_CUDA_MM_ONE_CTA (no CTA pairs), TRC_CUDA_MM_NO_PRETAIL.
int mul_mat_tc(const trc_cuda_view& a, const trc_cuda_view& b, const trc_cuda_view& d, uint32_t flags,
               cudaStream_t stream);
// True when mul_mat_tc can address these views with TMA (no launch).
bool mul_mat_tc_eligible(const trc_cuda_view& a, const trc_cuda_view& b, const trc_cuda_view& d);
// True when the fused kernel runs on CTA pairs with the packed bytes staged by TMA (16-byte aligned
// packed rows): the fastest implementation of trc_cuda_mul_mat_q for those weights.
bool mul_mat_q_tma_staged(int type, const void* w_blocks, int64_t w_ne0, int64_t w_ne1, int a_transposed, uint32_t flags);
int mul_mat_q_tc(int type, const void* w_blocks, int64_t w_ne0, int64_t w_ne1, int a_transposed,
                 const trc_cuda_view& b, const trc_cuda_view& d, uint32_t flags, cudaStream_t stream);

}  // namespace trc
