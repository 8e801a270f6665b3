// dequant.cu -- GGUF legacy-block dequantization (Q4_0/Q4_1/Q5_0/Q5_1/Q8_0 -> F32) for sm_100a.
//
// Replaces the host loop of gguf_tensor_to_f32 -> dequantize_q* (src/io/trc_gguf.cpp:966-1049,
// 320-417 of train.cpp). HBM-bound: per 32 weights it reads 18..34 packed bytes and writes 128.
//
// Layout and schedule
//   * A "run" is 256 consecutive blocks of one tensor (4.5-8.5 KiB packed, 32 KiB of F32 out).
//   * Persistent CTAs of 256 threads (two per SM) walk the runs of all jobs of a launch (one launch
//     can cover a whole model shard). Each CTA double-buffers its runs in shared memory: while it
//     decodes run r it already has the bulk copy (cp.async.bulk, TMA engine) of its next run in
//     flight.
//   * Decode: warp w owns blocks 32w..32w+31 of the run. In each of 8 steps a lane decodes 4
//     weights (a quad) of one of 4 blocks, and the warp writes 4 x 128 B = 512 contiguous bytes.
//   * Output: the decoded run goes to one of two F32 buffers in shared memory, and one bulk copy
//     (cp.async.bulk global <- shared) writes it to HBM while the CTA decodes the next run. On
//     B200 this writes the dequant's 1:5.4 read:write mix at 6.20-6.23 TB/s of algorithmic traffic
//     (five 4096 x 11008 tensors of all formats in one launch), 95 % of the 6.55 TB/s copy peak,
//     against 5.55 TB/s with 16-byte streaming st.global stores from registers.
//   * The peer variant (all-gather fused into the dequant) keeps the register stores and runs of
//     128 blocks: it writes every quad to the local buffer and to each peer's buffer over NVLink.
//   * A run whose packed bytes are not 16-byte aligned / sized (a tensor's ragged tail, or an
//     unaligned tensor) is staged by ordinary loads instead of the bulk copy, and a run whose output
//     is not 16-byte aligned is written from shared memory with ordinary stores.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <cstdint>

#include "trc_internal.h"
#include "trc_ptx.cuh"
#include "trc_quant.cuh"

namespace trc {

namespace {

constexpr int kThreads   = 256;
// Blocks per run: 256 for the bulk-store kernel (one 32 KiB bulk store of F32 per run), 128 for the
// peer-store kernel.
template <bool PEERS>
constexpr int kRunOf = PEERS ? 128 : 256;
constexpr int kMaxBlk    = 34;        // largest block (Q8_0)
constexpr int kMaxJobs   = 256;       // jobs per launch (kernel parameter of ~10 KiB)
template <bool PEERS>
constexpr int kBufBytesOf = kRunOf<PEERS> * kMaxBlk;
// Dynamic shared memory of dequant_kernel<PEERS>: two input slots, two output buffers (bulk-store
// kernel), two mbarriers.
template <bool PEERS>
constexpr int kSmemOf = 2 * kBufBytesOf<PEERS> + (PEERS ? 0 : 2 * kRunOf<PEERS> * 32 * 4) + 16;
constexpr int kMaxPeers  = 8;         // copies of each output written to other GPUs' buffers
// CTAs per SM of the bulk-store kernel. Measured on B200, five-tensor step (TB/s): runs of 256
// blocks at 2 CTAs per SM 6.20-6.23; runs of 128 at 3 per SM 5.97-6.00 (4 per SM 5.77, 5 per SM
// 5.57); 192 at 3 per SM 5.78; 320 at 2 per SM 5.84; 512 at 1 per SM 5.67. A third input buffer
// (packed bytes two runs ahead instead of one) measured 5.71 against 5.97, and a warp-asynchronous
// output path (each warp bulk-storing its own 2 KiB slice, input slots released through an
// mbarrier, no CTA-wide barrier per run) 5.38 against 5.99: few large bulk stores win.
constexpr int kBulkCtasPerSm = 2;

struct DqJob {
    const uint8_t* src;
    float*         out;
    int64_t        n_blocks;
    int64_t        run_begin;  // first global run index of this job
    int32_t        type;
    int32_t        block_bytes;
};

struct DqBatch {
    DqJob   job[kMaxJobs];
    int32_t n_jobs;
    int32_t n_peers;                // PEERS kernels: copies written besides `out`
    int64_t total_runs;
    int64_t peer_delta[kMaxPeers];  // byte distance from a job's out to its copy in peer p's buffer
};

template <int RUN>
__device__ __forceinline__ bool run_bulk_ok(const DqJob& J, int64_t local_run) {
    const int64_t b0    = local_run * RUN;
    const int64_t nblk  = min(static_cast<int64_t>(RUN), J.n_blocks - b0);
    const uint64_t addr = reinterpret_cast<uint64_t>(J.src) + static_cast<uint64_t>(b0) * J.block_bytes;
    const int64_t bytes = nblk * J.block_bytes;
    return (addr & 15u) == 0 && (bytes & 15) == 0;
}

// PEERS: every quad is also stored at the same offset of each peer GPU's buffer (peer-mapped
// addresses, plain stores over NVLink), which fuses the all-gather of a sharded tensor into its
// dequantization.
// Decodes a staged run into the CTA's output buffer in shared memory (F32, the run's layout), from
// where one bulk copy writes it to HBM. Warp w owns blocks (RUN/8)w .. (RUN/8)(w+1)-1; in each step a
// lane decodes 4 weights of one of 4 blocks, so a warp writes 512 contiguous bytes (no bank
// conflicts).
template <int TYPE, int RUN>
__device__ __forceinline__ void decode_run_smem(const uint8_t* buf, float* obuf, int nblk) {
    constexpr int kBB = QuantTraits<TYPE>::kBytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = lane & 7;
#pragma unroll 2
    for (int step = 0; step < RUN / 32; ++step) {
        const int lb = warp * (RUN / 8) + step * 4 + (lane >> 3);
        if (lb < nblk) {
            float w[4];
            QuadWords r;
            load_quad_words<TYPE>(buf + lb * kBB, 4 * c, r);
            decode_quad_words<TYPE>(r, 4 * c, w);
            *reinterpret_cast<float4*>(obuf + lb * 32 + 4 * c) = make_float4(w[0], w[1], w[2], w[3]);
        }
    }
}

template <int TYPE, bool PEERS>
__device__ __forceinline__ void decode_run(const uint8_t* buf, const DqJob& J, int64_t b0, int nblk,
                                           const DqBatch& batch) {
    constexpr int kBB = QuantTraits<TYPE>::kBytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int c = lane & 7;
    const bool vec_ok = (reinterpret_cast<uint64_t>(J.out) & 15u) == 0;
    constexpr int RUN = kRunOf<PEERS>;
#pragma unroll 2
    for (int step = 0; step < RUN / 32; ++step) {
        const int lb = warp * (RUN / 8) + step * 4 + (lane >> 3);
        if (lb < nblk) {
            float w[4];
            QuadWords r;
            load_quad_words<TYPE>(buf + lb * kBB, 4 * c, r);
            decode_quad_words<TYPE>(r, 4 * c, w);
            float* o = J.out + (b0 + lb) * 32 + 4 * c;
            const float4 v = make_float4(w[0], w[1], w[2], w[3]);
            if (vec_ok) {
                // streaming store: the output is written once and read by a later kernel
                __stcs(reinterpret_cast<float4*>(o), v);
            } else {
                o[0] = w[0]; o[1] = w[1]; o[2] = w[2]; o[3] = w[3];
            }
            if constexpr (PEERS) {
                for (int p = 0; p < batch.n_peers; ++p) {
                    float* q = reinterpret_cast<float*>(reinterpret_cast<char*>(o) + batch.peer_delta[p]);
                    if (vec_ok) {
                        *reinterpret_cast<float4*>(q) = v;  // deltas are multiples of 16
                    } else {
                        q[0] = w[0]; q[1] = w[1]; q[2] = w[2]; q[3] = w[3];
                    }
                }
            }
        }
    }
}

// The persistent grid is sized from the occupancy the compiled kernel really has (a grid of more
// CTAs than can be resident would run a ragged second wave).
template <bool PEERS>
__global__ void __launch_bounds__(kThreads) dequant_kernel(const __grid_constant__ DqBatch batch) {
    constexpr int RUN = kRunOf<PEERS>, BUF = kBufBytesOf<PEERS>;
    // (dynamic) two input slots; the bulk-store kernel's decoded runs, written to HBM by bulk copies
    // (two, so one can drain while the next fills); two mbarriers
    extern __shared__ __align__(128) uint8_t dq_smem[];
    uint8_t (*buf)[BUF] = reinterpret_cast<uint8_t (*)[BUF]>(dq_smem);
    float (*obuf)[RUN * 32] = reinterpret_cast<float (*)[RUN * 32]>(dq_smem + 2 * BUF);
    uint64_t* bar = reinterpret_cast<uint64_t*>(dq_smem + 2 * BUF + (PEERS ? 0 : 2 * RUN * 32 * 4));

    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_barrier_init();
    }
    __syncthreads();

    // Per slot s, bit s: the mbarrier phase to wait for, and whether a bulk copy is in flight
    // (bit masks, so that the per-slot state stays in registers).
    uint32_t phase_bits = 0u, pending_bits = 0u;
    int      jcur       = 0;  // job cursor (runs only increase for a CTA)

    auto locate = [&](int64_t run, int& j) {
        while (j + 1 < batch.n_jobs && batch.job[j + 1].run_begin <= run) ++j;
    };
    auto issue = [&](int64_t run, int j, int slot) {
        const DqJob&  J     = batch.job[j];
        const int64_t b0    = (run - J.run_begin) * RUN;
        const int64_t nblk  = min(static_cast<int64_t>(RUN), J.n_blocks - b0);
        const uint32_t bytes = static_cast<uint32_t>(nblk * J.block_bytes);
        mbar_arrive_expect_tx(&bar[slot], bytes);
        bulk_load(smem_u32(buf[slot]), J.src + b0 * J.block_bytes, bytes, &bar[slot]);
    };

    int64_t run = blockIdx.x;
    int     it  = 0;
    bool    ok  = true;
    if (run < batch.total_runs) {
        locate(run, jcur);
        if (run_bulk_ok<RUN>(batch.job[jcur], run - batch.job[jcur].run_begin)) {
            if (threadIdx.x == 0) issue(run, jcur, 0);
            pending_bits |= 1u;
        }
    }
    for (; run < batch.total_runs && ok; run += gridDim.x, ++it) {
        const int slot = it & 1;
        locate(run, jcur);
        const DqJob&  J     = batch.job[jcur];
        const int64_t local = run - J.run_begin;
        const int64_t b0    = local * RUN;
        const int     nblk  = static_cast<int>(min(static_cast<int64_t>(RUN), J.n_blocks - b0));

        // Prefetch the next run into the other slot (its previous contents were consumed in the
        // previous iteration, which ended with __syncthreads()).
        const int64_t next = run + gridDim.x;
        if (next < batch.total_runs) {
            int jn = jcur;
            locate(next, jn);
            if (run_bulk_ok<RUN>(batch.job[jn], next - batch.job[jn].run_begin)) {
                if (threadIdx.x == 0) issue(next, jn, slot ^ 1);
                pending_bits |= 1u << (slot ^ 1);
            }
        }

        if ((pending_bits >> slot) & 1u) {
            const bool mine = mbar_wait(&bar[slot], (phase_bits >> slot) & 1u, TRC_DEVERR_WAIT_BULK);
            ok = __syncthreads_and(mine ? 1 : 0) != 0;  // every thread takes the same branch
            if (mine) {
                phase_bits ^= 1u << slot;
                pending_bits &= ~(1u << slot);
            }
            if (!ok) break;
        } else {
            const uint8_t* src   = J.src + b0 * J.block_bytes;
            const int      bytes = nblk * J.block_bytes;
            for (int i = threadIdx.x; i < bytes; i += kThreads) buf[slot][i] = src[i];
            __syncthreads();
        }

        if constexpr (PEERS) {
            switch (J.type) {
                case 2: decode_run<2, true>(buf[slot], J, b0, nblk, batch); break;
                case 3: decode_run<3, true>(buf[slot], J, b0, nblk, batch); break;
                case 6: decode_run<6, true>(buf[slot], J, b0, nblk, batch); break;
                case 7: decode_run<7, true>(buf[slot], J, b0, nblk, batch); break;
                case 8: decode_run<8, true>(buf[slot], J, b0, nblk, batch); break;
                default: break;
            }
        } else {
            // At this point at most one bulk store is still reading shared memory: the previous
            // run's, from the other buffer (each run ends by waiting for all older ones).
            float* ob = obuf[slot];
            switch (J.type) {
                case 2: decode_run_smem<2, RUN>(buf[slot], ob, nblk); break;
                case 3: decode_run_smem<3, RUN>(buf[slot], ob, nblk); break;
                case 6: decode_run_smem<6, RUN>(buf[slot], ob, nblk); break;
                case 7: decode_run_smem<7, RUN>(buf[slot], ob, nblk); break;
                case 8: decode_run_smem<8, RUN>(buf[slot], ob, nblk); break;
                default: break;
            }
            float* dst = J.out + b0 * 32;
            if ((reinterpret_cast<uint64_t>(dst) & 15u) == 0) {
                fence_proxy_async_smem();  // the generic-proxy writes become visible to the bulk copy
                __syncthreads();
                if (threadIdx.x == 0) {
                    bulk_store(dst, smem_u32(ob), static_cast<uint32_t>(nblk) * 128u);
                    bulk_commit_group();
                    bulk_wait_group_read<1>();  // the previous run's copy has read the other buffer
                }
            } else {
                __syncthreads();  // an unaligned output: plain stores
                for (int i = threadIdx.x; i < nblk * 32; i += kThreads) dst[i] = ob[i];
                // no copy was issued: let every earlier one finish reading, so that none is
                // pending when the next run fills a buffer
                if (threadIdx.x == 0) bulk_wait_group_read<0>();
            }
        }
        __syncthreads();
    }
    // Every bulk store has completed before the grid counts as complete.
    if constexpr (!PEERS) {
        if (threadIdx.x == 0) bulk_wait_group_all();
    }
    // Never leave the CTA with a bulk copy still writing into its shared memory.
    for (int s = 0; s < 2; ++s) {
        if ((pending_bits >> s) & 1u) mbar_wait_drain(&bar[s], (phase_bits >> s) & 1u);
    }
    // The peer copies are visible to every GPU before the grid counts as complete.
    if constexpr (PEERS) __threadfence_system();
}

// CTAs of dequant_kernel<PEERS> resident per SM on the current device (queried once per device).
template <bool PEERS>
int resident_ctas() {
    static std::mutex mu;
    static int cached[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    std::lock_guard<std::mutex> lock(mu);
    if (cached[dev] == 0) {
        int n = 0;
        if (cudaFuncSetAttribute(dequant_kernel<PEERS>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemOf<PEERS>) !=
                cudaSuccess ||
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, dequant_kernel<PEERS>, kThreads, kSmemOf<PEERS>) !=
                cudaSuccess)
            return 0;
        cached[dev] = n;
    }
    return cached[dev];
}

}  // namespace

int dequant_jobs(const trc_cuda_dequant_job* jobs, int n_jobs, cudaStream_t stream) {
    return dequant_jobs_peers(jobs, n_jobs, nullptr, nullptr, 0, stream);
}

int dequant_jobs_peers(const trc_cuda_dequant_job* jobs, int n_jobs, const void* local_base,
                       void* const* peer_bases, int n_peers, cudaStream_t stream) {
    static_assert(sizeof(DqBatch) < 32000, "kernel parameter limit");
    if (n_jobs < 0 || (n_jobs > 0 && jobs == nullptr)) return TRC_CUDA_EINVAL;
    if (n_peers < 0 || n_peers > kMaxPeers || (n_peers > 0 && (peer_bases == nullptr || local_base == nullptr)))
        return TRC_CUDA_EINVAL;
    int64_t deltas[kMaxPeers] = {};
    for (int p = 0; p < n_peers; ++p) {
        if (peer_bases[p] == nullptr) return TRC_CUDA_EINVAL;
        deltas[p] = static_cast<int64_t>(reinterpret_cast<uintptr_t>(peer_bases[p]) -
                                         reinterpret_cast<uintptr_t>(local_base));
        if ((deltas[p] & 15) != 0) return TRC_CUDA_EINVAL;  // copies keep the outputs' 16-byte alignment
    }
    // Validate every job before touching the device.
    bool any_work = false;
    for (int i = 0; i < n_jobs; ++i) {
        const trc_cuda_dequant_job& in = jobs[i];
        if (trc_cuda_block_bytes(in.type) == 0) return TRC_CUDA_EUNSUPPORTED;
        if (in.n_blocks < 0) return TRC_CUDA_EINVAL;
        if (in.n_blocks == 0) continue;
        if (in.blocks == nullptr || in.out == nullptr) return TRC_CUDA_EINVAL;
        if ((reinterpret_cast<uint64_t>(in.blocks) & 1u) != 0 || (reinterpret_cast<uint64_t>(in.out) & 3u) != 0)
            return TRC_CUDA_EINVAL;  // fp16 fields need 2-byte, floats 4-byte alignment
        if (n_peers > 0 && reinterpret_cast<uintptr_t>(in.out) < reinterpret_cast<uintptr_t>(local_base))
            return TRC_CUDA_EINVAL;  // outputs lie in the local buffer that the peers mirror
        any_work = true;
    }
    if (!any_work) return TRC_CUDA_OK;
    const int sms = sm_count_current();
    if (sms <= 0) return TRC_CUDA_ECUDA;
    for (int first = 0; first < n_jobs; first += kMaxJobs) {
        DqBatch batch;
        batch.n_jobs    = 0;
        batch.n_peers   = n_peers;
        for (int p = 0; p < kMaxPeers; ++p) batch.peer_delta[p] = deltas[p];
        int64_t runs    = 0;
        const int count = std::min(kMaxJobs, n_jobs - first);
        for (int i = 0; i < count; ++i) {
            const trc_cuda_dequant_job& in = jobs[first + i];
            const size_t bb = trc_cuda_block_bytes(in.type);
            if (in.n_blocks == 0) continue;
            DqJob& J      = batch.job[batch.n_jobs++];
            J.src         = static_cast<const uint8_t*>(in.blocks);
            J.out         = in.out;
            J.n_blocks    = in.n_blocks;
            J.run_begin   = runs;
            J.type        = in.type;
            J.block_bytes = static_cast<int32_t>(bb);
            const int run_blocks = n_peers > 0 ? kRunOf<true> : kRunOf<false>;
            runs += (in.n_blocks + run_blocks - 1) / run_blocks;
        }
        if (batch.n_jobs == 0) continue;
        batch.total_runs = runs;
        int per_sm = n_peers > 0 ? resident_ctas<true>() : resident_ctas<false>();
        if (n_peers == 0) per_sm = std::min(per_sm, kBulkCtasPerSm);
        if (per_sm <= 0) return TRC_CUDA_ECUDA;
        const int64_t grid = std::min<int64_t>(runs, static_cast<int64_t>(sms) * per_sm);
        if (n_peers > 0) dequant_kernel<true><<<static_cast<unsigned>(grid), kThreads, kSmemOf<true>, stream>>>(batch);
        else dequant_kernel<false><<<static_cast<unsigned>(grid), kThreads, kSmemOf<false>, stream>>>(batch);
        note_launch();
        const int st = check_launch();
        if (st != TRC_CUDA_OK) return st;
    }
    return TRC_CUDA_OK;
}

}  // namespace trc
