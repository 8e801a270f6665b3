// probe_tc.cu -- measurement support: the tcgen05 kind::tf32 ceiling of this GPU.
//
// The mul_mat kernels are judged against a 3xTF32 roofline: three kind::tf32 MMAs per K-step
// (tA*hB, hA*tB, hA*hB), F32 FLOPs counted once. NVIDIA publishes no TF32 figure that this pool's
// B200s reach under their power cap, and half the measured bf16 rate is only a guess, so this probe
// measures it: every CTA (or CTA pair) keeps its tensor core busy with exactly the MMA stream of
// the GEMM's main loop -- the same instruction shapes (128 x 256 x 8 per CTA, or 256 x 256 x 8 on a
// CTA pair with cta_group::2), K-major 64-byte-swizzled operands in shared memory, three MMAs per
// K=8 step into one fp32 TMEM accumulator -- with no loads, no operand split and no epilogue. Its
// rate is the most the GEMM's tensor pipe can deliver; bench.py reports every GEMM as a fraction of
// it next to the bf16-derived figure.
#include <cuda_runtime.h>

#include <cstdint>

#include "trc_internal.h"
#include "trc_ptx.cuh"

namespace trc {
namespace {

constexpr int PROBE_THREADS = 128;
constexpr int PROBE_BM = 128, PROBE_BN = 256, PROBE_BK = 16;

template <int CG>
struct ProbeGeo {
    static constexpr int A_BYTES = PROBE_BM * PROBE_BK * 4;             // 8 KiB per tile
    static constexpr int B_BYTES = (PROBE_BN / CG) * PROBE_BK * 4;      // 16 / 8 KiB per tile
    static constexpr int OFF_A_RAW = 0, OFF_A_TAIL = A_BYTES, OFF_B_RAW = 2 * A_BYTES;
    static constexpr int OFF_B_TAIL = 2 * A_BYTES + B_BYTES;
    static constexpr int TILE_BYTES = 2 * (A_BYTES + B_BYTES);
    // sized so that one CTA occupies an SM, as the GEMM's does
    static constexpr int SMEM_BYTES = 160 * 1024;
};

__device__ __forceinline__ uint64_t probe_desc(uint32_t tile, int kk) {
    return make_smem_desc(tile + kk * 32, 16, 512, 4);  // K-major, 64-byte swizzle, 32 B per K=8
}

template <int CG>
__global__ void __launch_bounds__(PROBE_THREADS, 1) tf32_mma_probe_kernel(int iters) {
    using G = ProbeGeo<CG>;
    constexpr bool PAIR = CG == 2;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* mma_done = reinterpret_cast<uint64_t*>(smem + G::TILE_BYTES);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + G::TILE_BYTES + 8);
    const int warp = threadIdx.x >> 5;
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;

    // operands: finite pseudo-random fp32 values of magnitude ~1 (no zeros, so the datapath toggles
    // as it does on real data)
    for (int i = threadIdx.x; i < G::TILE_BYTES / 4; i += PROBE_THREADS) {
        uint32_t h = (static_cast<uint32_t>(i) + 0x9E3779B9u * (blockIdx.x + 1u)) * 2654435761u;
        h ^= h >> 15;
        reinterpret_cast<uint32_t*>(smem)[i] = 0x3F800000u | (h & 0x007FFFFFu);  // [1, 2)
    }
    if (threadIdx.x == 0) {
        mbar_init(mma_done, 1);
        fence_barrier_init();
    }
    fence_proxy_async_smem();
    if (warp == 0) {
        tmem_alloc<CG>(tmem_slot, 256);
        tmem_relinquish<CG>();
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) cluster_sync();
    tc_fence_after();
    const uint32_t d_tmem = *tmem_slot;
    const uint32_t base = smem_u32(smem);
    const uint32_t idesc = make_idesc_tf32(PROBE_BM * CG, PROBE_BN, 0, 0);

    if (threadIdx.x == 0 && rank == 0) {
        for (int it = 0; it < iters; ++it) {
#pragma unroll
            for (int kk = 0; kk < PROBE_BK / 8; ++kk) {
                const uint64_t a_raw = probe_desc(base + G::OFF_A_RAW, kk), a_tail = probe_desc(base + G::OFF_A_TAIL, kk);
                const uint64_t b_raw = probe_desc(base + G::OFF_B_RAW, kk), b_tail = probe_desc(base + G::OFF_B_TAIL, kk);
                umma_tf32<CG>(d_tmem, a_tail, b_raw, idesc, (it != 0 || kk != 0) ? 1u : 0u);
                umma_tf32<CG>(d_tmem, a_raw, b_tail, idesc, 1u);
                umma_tf32<CG>(d_tmem, a_raw, b_raw, idesc, 1u);
            }
        }
        if constexpr (PAIR) umma_commit_pair_both(mma_done, 0x3);
        else umma_commit(mma_done);
    }
    // every thread waits (bounded) for the MMAs to complete before TMEM is released
    mbar_wait_scoped<PAIR>(mma_done, 0, TRC_DEVERR_WAIT_ACCUM);
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) cluster_sync();
    tc_fence_after();
    if (warp == 0) tmem_dealloc<CG>(d_tmem, 256);
}

}  // namespace
}  // namespace trc

extern "C" int trc_cuda_tf32_mma_probe(int cta_group, int iters, void* stream) {
    using namespace trc;
    if ((cta_group != 1 && cta_group != 2) || iters <= 0 || iters > (1 << 22)) return TRC_CUDA_EINVAL;
    const int sms = sm_count_current();
    if (sms <= 0) return TRC_CUDA_ECUDA;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    if (cta_group == 1) {
        constexpr int smem = ProbeGeo<1>::SMEM_BYTES;
        e = cudaFuncSetAttribute(tf32_mma_probe_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_fail(e);
        tf32_mma_probe_kernel<1><<<static_cast<unsigned>(sms), PROBE_THREADS, smem, s>>>(iters);
    } else {
        constexpr int smem = ProbeGeo<2>::SMEM_BYTES;
        e = cudaFuncSetAttribute(tf32_mma_probe_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_fail(e);
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(2 * static_cast<unsigned>(sms / 2));
        cfg.blockDim = dim3(PROBE_THREADS);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = s;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, tf32_mma_probe_kernel<2>, iters);
        if (e != cudaSuccess) return cuda_fail(e);
    }
    note_launch();
    return check_launch();
}
