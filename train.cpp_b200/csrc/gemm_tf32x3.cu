// gemm_tf32x3.cu -- ggml mul_mat on the sm_100a tensor cores (tcgen05 / TMEM) at F32 accuracy.
//
// Replaces compute_mul_mat (src/backends/cpu/trc_cpu_ops.cpp:182-216 of train.cpp) for every view
// TMA can address: operands contiguous along K ("K-major": the forward product and dB) or along
// M/N ("MN-major": the transposed views of the composed backward, src/core/trc_autograd.cpp:487-503),
// with ne[2]/ne[3] modulo broadcasting of a.
//
// 3xTF32. The tensor core consumes TF32 (10 explicit mantissa bits). Each fp32 operand x is split
// into a head h = x with the low 13 mantissa bits cleared (what the tensor core reads from the raw
// fp32 word) and a tail t = x - h (exact in fp32). Per K-step the kernel issues
//     D += tA * hB,   D += hA * tB,   D += hA * hB
// into an fp32 TMEM accumulator; only tA*tB (relative size 2^-22) is dropped. Measured on B200
// against a float64 product: 2.3e-6 normwise at every K from 256 to 14336, which keeps the result
// within 1e-5 normwise of the reference CPU (itself 2.4e-6..4.4e-6 from exact at these K).
//
// fp32 promotion. The tensor core's fp32 accumulation does not round to nearest: measured on B200,
// the error of one long accumulation grows linearly with K (3.6e-5 normwise at K = 4096). So the
// K loop is cut into chunks of CHUNK_KB k-blocks (256 K); each chunk accumulates from zero in TMEM
// and the epilogue warps add it to the tile's running total with IEEE round-to-nearest fp32 adds.
// The two 256-column TMEM buffers swap roles per tile (running total T / chunk X), so the tile
// double buffering survives: tile i keeps its total in buffer i%2 and its chunks in buffer
// (i+1)%2, and tile i+1's first chunk can start while tile i's total is being stored.
//
// Schedule: persistent; each CTA (or CTA pair) walks its units (UnitCursor): whole tiles round-robin,
// the parts of a split-K plan, or a stream plan's run of k-chunks (plan_split).
//
// Structure (persistent, 18 warps per CTA):
//   warp 0      TMA producer: raw fp32 A/B tiles -> shared memory (F32 kernel: a ring of raw
//               slots; fused kernel: a ring of 5 stages that also holds the packed weight bytes)
//   warp 1      TMEM allocator + single-thread UMMA issuer (tcgen05.mma.kind::tf32)
//   warps 2-9   split warps: write the tails tA, tB of each stage (F32 kernel: into a short ring
//               of tail slots of their own; fused kernel: next to the raw tiles, after decoding
//               the packed weight tile into head + tail)
//   warps 10-17 epilogue, two teams of four (one per column half): TMEM -> registers (tcgen05.ld)
//               -> shared memory -> TMA store (or strided stores when TMA cannot address D)
// CTA pairs (default when M spans more than 128 rows): a cluster of two CTAs computes a 256 x 256
// tile with tcgen05 cta_group::2. Each CTA stages its 128 rows of A and 128 of the 256 rows of B;
// the leader's single thread issues the MMAs for both SMs, so each SM stages, splits and feeds the
// tensor core half the B bytes of a one-CTA 128 x 256 tile. One CTA per 128 x 256 tile
// (cta_group::1) is kept for M <= 128 and on request (TRC_CUDA_MM_ONE_CTA).
// Two 256-column fp32 TMEM buffers (all 512 columns). Shared-memory operand layouts: K-major tiles
// use the 64-byte swizzle (64 B rows); MN-major tiles use the 128-byte swizzle with 32-byte atoms,
// the one layout tcgen05 accepts for MN-major TF32 operands (32-element MN chunks of 16 K-rows x
// 128 B).
// Every mbarrier wait is bounded (trc_ptx.cuh); a timeout sets the device error word and the kernel
// drains its in-flight copies and MMAs, frees TMEM and returns.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <type_traits>
#include <mutex>
#include <unordered_map>

#include "trc_internal.h"
#include "trc_ptx.cuh"
#include "trc_quant.cuh"

#include <cuda_fp16.h>

namespace trc {


// Scratch buffers (B's tails, split-K workspaces, dequantized weights) come from the device's
// default memory pool; freed blocks stay in the pool (release threshold raised once per device, a
// setting of this process only) so that steady-state calls do not map memory again.
void retain_pool_once() {
    static std::mutex mu;
    static uint64_t   done = 0;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return;
    std::lock_guard<std::mutex> lock(mu);
    if (done & (uint64_t(1) << dev)) return;
    cudaMemPool_t pool;
    if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
        uint64_t threshold = UINT64_MAX;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
    }
    cudaGetLastError();
    done |= uint64_t(1) << dev;
}

namespace {

constexpr int BM = 128, BN = 256, BK = 16;   // D tile of one CTA: BM rows (TMEM lanes) x BN columns
constexpr int NUM_THREADS  = 576;
// warps 10-17: two epilogue teams of four warps (TMEM lane quarters 2,3,0,1 each); team h owns
// columns 128h .. 128h+127 of every tile
constexpr int SPLIT_WARP0 = 2, SPLIT_WARPS = 8, EPI_WARP0 = 10, EPI_WARPS = 8;
constexpr int TMEM_COLS    = 512;
constexpr int CHUNK_KB     = 16;   // k-blocks per fp32 promotion chunk (256 K)
constexpr int EPI_BUF_BYTES = BM * 32 * 4;  // one 128-row x 32-column fp32 group of D, staged for a TMA store
constexpr int EPI_BUFS      = 2;            // one staging buffer per epilogue team
constexpr int EPI_BAR_TEAM0 = 1, EPI_BAR_ALL = 3;  // named barriers: per team (1, 2), all epilogue warps (3)
constexpr int MAX_STAGES    = 12;
constexpr int BARRIER_BYTES = 512;          // shared memory reserved for struct Barriers

// The F32 kernel's separate raw and tail rings (index: CG): a slot holds 24 KiB of A+B for one CTA,
// 16 KiB per CTA of a pair. Measured on B200 against tails beside every raw stage (4 stages, the
// same 192 / 128 KiB): single CTAs (the GQA dA and dB, M = 128) 185-208 against 173-182 TFLOP/s with
// 5 raw + 3 tail slots, 178 with 6 + 2 and 171-178 with 4 + 4; CTA pairs (Linear forward / dX / dW)
// 237 / 240 / 214 against 226 / 231 / 212 with 8 + 4 slots, about 1 % less with 8 + 3 or 9 + 3,
// and dW 195 with 10 + 2 (the split warps then run out of tail slots).
constexpr int kRawStages[3]  = {0, 5, 8};
constexpr int kTailStages[3] = {0, 3, 4};

// Shared-memory geometry per CTA group. CG = 1: one CTA computes a 128 x 256 tile from a 128-row
// A tile and a 256-row B tile. CG = 2 (tcgen05 cta_group::2): a cluster of two CTAs computes a
// 256 x 256 tile; each CTA stages its own 128 rows of A and 128 of the 256 rows of B, and the
// leader's MMA reads both CTAs' shared memory, so each SM stages and splits half the B bytes.
// PQ > 0: the fused kernel's stages also hold PQ bytes of the weight's packed blocks, loaded by TMA.
// TS > 0: the raw tiles and the split warps' output live in two rings of their own -- a deep ring of
// STAGES raw slots that TMA fills, and a short ring of TS tail slots that the split warps fill just
// ahead of the MMA -- so more raw bytes can be in flight than with tails beside every stage.
//   F32 kernel (PQ = 0): raw slot [A | B], tail slot [A tail | B tail].
//   fused kernel (PQ > 0): raw slot [B | packed A], tail slot [A head | A tail | B tail].
// TS = 0: one ring of STAGES slots [A | A tail | B | B tail | packed A].
template <int CG, int PQ = 0, int TS = 0>
struct Geo {
    static constexpr int BN_CTA      = BN / CG;                     // B rows staged by one CTA
    static constexpr int A_BYTES     = BM * BK * 4;                 //  8 KiB
    static constexpr int B_BYTES     = BN_CTA * BK * 4;             // 16 KiB (CG 1) / 8 KiB (CG 2)
    static constexpr int RAW_BYTES   = A_BYTES + B_BYTES;
    static_assert(PQ % 1024 == 0 && (PQ == 0 || CG == 2), "packed slot: 1 KiB multiples, CTA pairs only");
    // raw (TS > 0) or whole (TS = 0) stage
    static constexpr int STAGE_BYTES = TS == 0 ? 2 * RAW_BYTES + PQ : (PQ ? B_BYTES + PQ : RAW_BYTES);
    static constexpr int OFF_A_RAW   = 0;                           // (PQ = 0) A; (PQ > 0, TS > 0) unused
    static constexpr int OFF_A_TAIL  = A_BYTES;                     // (TS = 0)
    static constexpr int OFF_B_RAW   = TS == 0 ? 2 * A_BYTES : (PQ ? 0 : A_BYTES);
    static constexpr int OFF_B_TAIL  = 2 * A_BYTES + B_BYTES;       // (TS = 0)
    static constexpr int OFF_PQ      = TS == 0 ? 2 * RAW_BYTES : B_BYTES;
    // tail slot (TS > 0)
    static constexpr int TAIL_BYTES  = PQ ? 2 * A_BYTES + B_BYTES : RAW_BYTES;
    static constexpr int T_A_HEAD    = 0;                           // (PQ > 0)
    static constexpr int T_A_TAIL    = PQ ? A_BYTES : 0;
    static constexpr int T_B_TAIL    = PQ ? 2 * A_BYTES : A_BYTES;
    static constexpr int RING_BUDGET = 232448 - EPI_BUFS * EPI_BUF_BYTES - 1024 - BARRIER_BYTES;
    static constexpr int fill_stages() {
        const int n = (RING_BUDGET - TS * TAIL_BYTES) / STAGE_BYTES;
        return n < MAX_STAGES ? n : MAX_STAGES;
    }
    // Stages with tails beside the raw tiles: the fused dX measured 255 TFLOP/s with 5 stages and
    // 243 with 4. With separate rings the fused kernel takes as many raw slots as fit.
    static constexpr int STAGES      = TS == 0 ? (CG == 2 ? (PQ ? 5 : 4) : 4) : (PQ ? fill_stages() : kRawStages[CG]);
    static constexpr int OFF_TAILS   = STAGES * STAGE_BYTES;        // tail slot t: OFF_TAILS + t * TAIL_BYTES
    static constexpr int RAW_TX_BYTES = A_BYTES + B_BYTES;          // bytes TMA delivers per F32 stage
    static constexpr int EPI_OFF     = OFF_TAILS + TS * TAIL_BYTES;
    static constexpr int SMEM_BYTES  = EPI_OFF + EPI_BUFS * EPI_BUF_BYTES + 1024 /*align*/ + BARRIER_BYTES;
    static constexpr int TILE_M      = CG * BM;                     // D rows per tile
    static_assert(STAGES >= 2 && STAGES <= MAX_STAGES && TS <= MAX_STAGES, "barrier arrays");
    static_assert(STAGE_BYTES % 1024 == 0 && TAIL_BYTES % 1024 == 0, "1 KiB-aligned tiles");
    static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
};

struct TcParams {
    int     M, N, K;           // M: TMEM lanes (rows of D tiles), N: columns, K: reduction
    int     m_tiles, n_tiles, k_blocks;  // m_tiles counts tiles of CG*128 rows
    int     planes2, planes3;  // output planes
    int     red2, red3;        // source planes summed into each output plane (repeat_back fused)
    int     kv_blocks;         // k-blocks per tile: k_blocks x red2 x red3
    int     a_ne2, a_ne3, b_ne2, b_ne3;
    int     a_mn, b_mn;        // 1 = operand contiguous along M (resp. N)
    int     a_tma5, b_tma5;    // MN-major operand loaded by one 5-D TMA per stage (else one per 32-row chunk)
    int     b_pretail;         // 1: B's TF32 tails were computed once before the launch and come
                               // through tmBt (same geometry as tmB); the split warps skip B
    int     accumulate;
    int64_t total_tiles;
    // split-K: each tile's kv range is cut into `splits` parts of kv_per_split k-blocks, computed by
    // different CTAs (work units) and reduce-added into D (zeroed beforehand by the host)
    int     splits, kv_per_split;
    int64_t total_units;       // units dealt round-robin to the slots: total_tiles x splits, or the
                               // whole tiles of a stream plan's first waves
    // stream plan (sk_chunks > 0): after its round-robin units, each slot (CTA or CTA pair of the
    // grid) takes an equal run of the k-chunks of tiles sk_tile0 .. total_tiles - 1, in tile order
    int     nck;               // k-chunks (CHUNK_KB k-blocks) per tile
    int64_t sk_tile0, sk_chunks;
    int64_t sk_slots;          // slots of the plan: the grid launches exactly this many
    char*   d;
    int64_t d_sm, d_sn, d_s2, d_s3;  // byte strides of D along M, N, plane2, plane3
    int     tma_store;               // 1: D is written (or reduce-added) by TMA from shared memory
    // quantized A (fused variant): packed blocks of the weight W, rows of q_row_bytes bytes
    const uint8_t* qa;
    int64_t        q_row_bytes;
    int            q_rows;           // W rows (ne1)
    int            q_blocks_per_row; // W ne0 / 32
};

struct Barriers {
    uint64_t full[MAX_STAGES];   // this CTA's TMA tiles of the stage have landed
    uint64_t split[MAX_STAGES];  // (leader) every split warp of the group has written its tails
    uint64_t empty[MAX_STAGES];  // the MMAs reading the stage have completed
    uint64_t tail_empty[MAX_STAGES];  // (separate tail ring) the MMAs reading the tail slot have completed
    uint64_t acc_full[2];
    uint64_t acc_empty[2];       // (leader) every epilogue warp of the group has drained the buffer
    uint64_t mma_done;
    uint32_t tmem_slot;
};
static_assert(sizeof(Barriers) <= BARRIER_BYTES, "barrier reservation");

__device__ __forceinline__ uint32_t tf32_tail_bits(uint32_t u) {
    const float x = __uint_as_float(u);
    const float h = __uint_as_float(u & 0xFFFFE000u);
    return __float_as_uint(isfinite(x) ? __fsub_rn(x, h) : 0.0f);
}

struct TileCoord {
    int m0, n0, p2, p3;  // m0: first row of the (CG*128-row) tile
};

// Tiles of a plane are visited in bands of GROUP_M row tiles, column by column inside a band, so
// the tiles in flight at once (one per SM or SM pair) share a few row and column panels of A and
// B, and those panels stay in L2 (a plain row-major order streams all of B once per row tile).
constexpr int GROUP_M = 8;

template <int CG>
__host__ __device__ __forceinline__ TileCoord tile_coord(const TcParams& p, int64_t tile) {
    const int64_t per_plane = static_cast<int64_t>(p.m_tiles) * p.n_tiles;
    const int64_t plane     = tile / per_plane;
    const int     r         = static_cast<int>(tile - plane * per_plane);
    const int     per_band  = GROUP_M * p.n_tiles;
    const int     band      = r / per_band;
    const int     rb        = r - band * per_band;
    const int     left      = p.m_tiles - band * GROUP_M;
    const int     band_m    = left < GROUP_M ? left : GROUP_M;           // row tiles in this band
    TileCoord c;
    c.m0 = (band * GROUP_M + rb % band_m) * Geo<CG>::TILE_M;
    c.n0 = (rb / band_m) * BN;
    c.p2 = static_cast<int>(plane % p.planes2);
    c.p3 = static_cast<int>(plane / p.planes2);
    return c;
}

struct UnitSpan {
    int64_t tile;
    int     kv0, kv1;  // the unit's virtual k-blocks [kv0, kv1)
};

__device__ __forceinline__ UnitSpan unit_span(const TcParams& p, int64_t unit) {
    UnitSpan u;
    const int64_t sp = unit / p.total_tiles;
    u.tile = unit - sp * p.total_tiles;
    u.kv0  = static_cast<int>(sp) * p.kv_per_split;
    u.kv1  = min(p.kv_blocks, u.kv0 + p.kv_per_split);
    return u;
}

// Where a unit's tile goes.
enum UnitDest { kStoreD = 0, kReduceD = 1, kReduceW = 2 };

// The units of one slot (CTA or CTA pair), in order; every warp role walks the same sequence. First
// the round-robin units slot, slot + nslots, ... below total_units; then, in a stream plan, the
// slot's run of k-chunks [slot * sk_chunks / nslots, (slot + 1) * sk_chunks / nslots) of the stream
// tiles, cut at tile boundaries into pieces. A piece that is a whole tile is stored; a tile cut into
// pieces has its first two pieces (in k order) reduce-added into D and its third and fourth into
// the workspace (the plan admits at most four), both zeroed beforehand, so the sum is
// (a + b) + (c + d) whatever order the pieces land in. The host admits a stream plan only when
// sk_chunks x nslots < 2^31, so the stream phase runs on 32-bit arithmetic.
template <int CG>
struct UnitCursor {
    int64_t  pos;  // round-robin phase: unit index; stream phase: chunk index among the stream chunks
    uint32_t end;  // stream phase: the end of this slot's run
    bool     sk;   // in the stream phase

    static __device__ __forceinline__ uint32_t slot() { return blockIdx.x / CG; }
    static __device__ __forceinline__ uint32_t nslots() { return gridDim.x / CG; }
    static __device__ __forceinline__ uint32_t sk_start(const TcParams& p, uint32_t s) {
        return s * static_cast<uint32_t>(p.sk_chunks) / nslots();
    }
    __device__ __forceinline__ void enter_stream(const TcParams& p) {
        sk  = true;
        pos = sk_start(p, slot());
        end = sk_start(p, slot() + 1);
    }
    __device__ __forceinline__ explicit UnitCursor(const TcParams& p) : pos(slot()), end(0), sk(false) {
        if (pos >= p.total_units) enter_stream(p);
    }
    __device__ __forceinline__ bool live(const TcParams& p) const {
        return sk ? static_cast<uint32_t>(pos) < end : pos < p.total_units;
    }
    __device__ __forceinline__ UnitSpan span(const TcParams& p) const {
        if (!sk) return unit_span(p, pos);
        const uint32_t c = static_cast<uint32_t>(pos), nck = static_cast<uint32_t>(p.nck);
        const uint32_t lt = c / nck, c0 = c - lt * nck, c1 = min(nck, c0 + (end - c));
        UnitSpan u;
        u.tile = p.sk_tile0 + lt;
        u.kv0  = static_cast<int>(c0) * CHUNK_KB;
        u.kv1  = min(p.kv_blocks, static_cast<int>(c1) * CHUNK_KB);
        return u;
    }
    __device__ __forceinline__ void next(const TcParams& p) {
        if (!sk) {
            pos += nslots();
            if (pos >= p.total_units) enter_stream(p);
        } else {
            const uint32_t nck = static_cast<uint32_t>(p.nck);
            pos = min(end, (static_cast<uint32_t>(pos) / nck + 1) * nck);
        }
    }
    __device__ __forceinline__ UnitDest dest(const TcParams& p, const UnitSpan& u) const {
        if (!sk) return pos >= 2 * p.total_tiles ? kReduceW : (p.accumulate || p.splits > 1 ? kReduceD : kStoreD);
        if (u.kv0 == 0) return u.kv1 == p.kv_blocks ? kStoreD : kReduceD;  // the tile's first piece
        // A piece that starts inside its tile starts this slot's run, so the previous slot holds the
        // chunks just before it: the tile's first piece (this is the second) if it also holds the
        // tile's first chunk, else a middle piece (this is the third or fourth).
        const uint32_t first = static_cast<uint32_t>(u.tile - p.sk_tile0) * static_cast<uint32_t>(p.nck);
        return sk_start(p, slot() - 1) <= first ? kReduceD : kReduceW;
    }
};

// K-major tile (rows x 16 fp32, 64 B per row, 8-row swizzle atoms of 512 B): advance 32 B per K=8.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t tile, int kk) {
    return make_smem_desc(tile + kk * 32, 16, 512, 4);
}
// MN-major tile (32-element MN chunks of 16 K-rows x 128 B = 2 KiB, 128B swizzle with 32B atoms,
// descriptor layout type 1): LBO = 2 KiB between MN chunks, SBO = 512 B between 4-row K groups,
// advance 1 KiB (8 K-rows) per K=8.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t tile, int kk) {
    return make_smem_desc(tile + kk * 1024, 2048, 512, 1);
}

// Tails of a thread's 16-byte chunks i0, i0 + i_step, ... (< i_end) of a stage's raw tiles (chunk
// index i < nA: A tile, else B tile), at most PER of them. All loads are issued before the first
// store: the compiler cannot prove the raw and tail tiles disjoint, so a load-split-store per
// chunk would keep every load behind the previous chunk's store and serialize the shared-memory
// round trips (measured: the split warps then held the F32 kernel 20-30 % below its no-split
// speed).
template <class G, int PER>
__device__ __forceinline__ void split_chunks(uint8_t* st, int i0, int i_end, int i_step, int nA) {
    uint4 v[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int i = i0 + j * i_step;
        if (i < i_end)
            v[j] = i < nA ? reinterpret_cast<const uint4*>(st + G::OFF_A_RAW)[i]
                          : reinterpret_cast<const uint4*>(st + G::OFF_B_RAW)[i - nA];
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int i = i0 + j * i_step;
        if (i < i_end) {
            uint4 u = v[j];
            u.x = tf32_tail_bits(u.x);
            u.y = tf32_tail_bits(u.y);
            u.z = tf32_tail_bits(u.z);
            u.w = tf32_tail_bits(u.w);
            if (i < nA) reinterpret_cast<uint4*>(st + G::OFF_A_TAIL)[i] = u;
            else reinterpret_cast<uint4*>(st + G::OFF_B_TAIL)[i - nA] = u;
        }
    }
}

// split_chunks for the separate raw and tail rings: chunk i of the raw slot [A | B] -> chunk i of the
// tail slot [A tail | B tail]. All loads are issued before the first store, as above.
template <int PER>
__device__ __forceinline__ void split_chunks_rings(const uint8_t* raw, uint8_t* tail, int i0, int i_end, int i_step) {
    uint4 v[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int i = i0 + j * i_step;
        if (i < i_end) v[j] = reinterpret_cast<const uint4*>(raw)[i];
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const int i = i0 + j * i_step;
        if (i < i_end) {
            uint4 u = v[j];
            u.x = tf32_tail_bits(u.x);
            u.y = tf32_tail_bits(u.y);
            u.z = tf32_tail_bits(u.z);
            u.w = tf32_tail_bits(u.w);
            reinterpret_cast<uint4*>(tail)[i] = u;
        }
    }
}

// A-tile offsets (the same in both geometries), used by the fused decode.
constexpr int OFF_A_RAW = 0, OFF_A_TAIL = BM * BK * 4;


// Fused dequant: a stage's A tile (128 rows x 16 K) is 512 quads of 4 consecutive weights. Quad q
// of the stage comes from quad_block() (nullptr: out of range, written as zeros) and goes, as head
// (TF32-truncated) and tail, to the swizzled byte offset quad_offset(q) of the A tiles. Consecutive
// quads read adjacent bytes of the packed rows, so a warp's loads touch few cache lines.
constexpr int A_QUADS = BM * BK / 4;

// TMA staging of the packed weight (CTA pairs): per stage one 2-D box of the packed rows, uint8
// elements, starting at a 16-byte-aligned column x (the TMA rule for the innermost coordinate) at or
// below the first needed byte; the needed bytes then start at an even offset o <= 14 into each box
// row (block sizes are even), and the box is wide enough for o + the needed bytes.
//   K-major (A = W): 128 W rows x the one block holding the stage's 16 weights of each row.
//   MN-major (A = transpose(W)): 16 W rows (the stage's K) x the 4 blocks of the tile's 128 columns.
// Rows or bytes outside the tensor arrive as zeros.
template <int QTYPE, int QTRANS>
struct PackedBox {
    static constexpr int kBB    = QuantTraits<QTYPE>::kBytes;
    static constexpr int kNeed  = QTRANS ? 4 * kBB : kBB;
    static constexpr int kW     = (14 + kNeed + 15) / 16 * 16;   // box width in bytes
    static constexpr int kH     = QTRANS ? BK : BM;              // box rows
    static constexpr int kBytes = kW * kH;
    static constexpr int kSlot  = (kBytes + 1023) / 1024 * 1024;
    static_assert(kW <= 256, "TMA box width");
};
template <int QTYPE, int QTRANS, int PT>
struct PackedSlot {
    static constexpr int value = 0;
};
template <int QTYPE, int QTRANS>
struct PackedSlot<QTYPE, QTRANS, 1> {
    static constexpr int value = QTYPE == 0 ? 0 : PackedBox<QTYPE == 0 ? 2 : QTYPE, QTRANS>::kSlot;
};

// Tail slots of the TMA-staged fused kernel's separate rings (its raw slots fill the rest); 0 keeps
// its tails beside the raw tiles of 5 stages. Measured on B200 (Q5_0 4096 x 14336, 2048 tokens,
// forward / dX TFLOP/s): 5 stages with tails beside 239.9 / 257.0; 4 tail slots (6 / 9 raw)
// 231.6 / 244.6; 3 tail slots the same; 2 tail slots 209.5 / 218.0. Its raw slots are small (B and
// the packed box), so a deeper raw ring buys little, while the decode groups lose tail slots.
constexpr int kPtTailStages = 0;

// The shared-memory geometry of one kernel instantiation (the kernel and its launch agree on it).
template <int QTYPE, int QTRANS, int CG, int PT>
struct KernelGeo {
    static constexpr int PQ = PackedSlot<QTYPE, QTRANS, PT>::value;
    static constexpr int TS = QTYPE == 0 ? kTailStages[CG] : (PQ ? kPtTailStages : 0);
    using type = Geo<CG, PQ, TS>;
};

// Per tile: the packed-row pointer of quad q (K-major: its W row; MN-major: its K-row offset and
// block column), nullptr when the quad's rows lie outside the matrix.
template <int QTYPE, int QTRANS>
__device__ __forceinline__ const uint8_t* quad_tile_base(const TcParams& p, int m0, int q) {
    constexpr int BB = QuantTraits<QTYPE>::kBytes;
    if constexpr (QTRANS == 0) {
        const int m = m0 + (q >> 2);
        return m < p.M ? p.qa + static_cast<int64_t>(m) * p.q_row_bytes : nullptr;
    } else {
        const int kr = q >> 5, m = m0 + 32 * ((q & 31) >> 3);
        return m < p.M ? p.qa + static_cast<int64_t>(kr) * p.q_row_bytes + static_cast<int64_t>(m >> 5) * BB : nullptr;
    }
}

// Per stage: the block holding quad q's four weights and the index j0 of the first of them
// (nullptr: out of range). K-major: block k0/32 of the row, weights (k0 mod 32) + 4 (q mod 4);
// MN-major: W row k0 + q/32, weights 4 ((q mod 32) mod 8).
template <int QTYPE, int QTRANS>
__device__ __forceinline__ const uint8_t* quad_block(const TcParams& p, const uint8_t* base, int k0, int q, int& j0) {
    constexpr int BB = QuantTraits<QTYPE>::kBytes;
    if (base == nullptr) return nullptr;
    if constexpr (QTRANS == 0) {
        j0 = (k0 & 16) + 4 * (q & 3);
        return base + (k0 >> 5) * BB;
    } else {
        j0 = (q & 7) * 4;
        return k0 + (q >> 5) < p.K ? base + static_cast<int64_t>(k0) * p.q_row_bytes : nullptr;
    }
}

template <int QTRANS>
__device__ __forceinline__ int quad_offset(int q) {
    if constexpr (QTRANS == 0) {
        const int r = q >> 2, u = q & 3;  // K-major: 64-byte rows, unit u ^ ((r >> 1) & 3)
        return r * 64 + ((u ^ ((r >> 1) & 3)) << 4);
    } else {
        const int kr = q >> 5, mq = q & 31;  // MN-major: 32-element chunk mq/8, K-row kr, 32-byte units ^ (kr & 3)
        return (mq >> 3) * 2048 + kr * 128 + ((((mq & 7) >> 1) ^ (kr & 3)) << 5) + ((mq & 1) << 4);
    }
}

// Index of the first of quad q's four weights within its block, at k-block kb (the j0 that
// quad_block returns).
template <int QTRANS>
__device__ __forceinline__ int quad_j0(int kb, int q) {
    if constexpr (QTRANS == 0) return ((kb * BK) & 16) + 4 * (q & 3);
    else return (q & 7) * 4;
}

// Decoded weights are finite for finite scales, so the tail needs no special-value handling
// (a non-finite scale makes the product NaN either way).
__device__ __forceinline__ void store_quad_head_tail(uint8_t* st, int off, const float (&w)[4]) {
    uint4 h, l;
    uint32_t* hp = &h.x;
    uint32_t* lp = &l.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const uint32_t bits = __float_as_uint(w[e]);
        hp[e] = bits & 0xFFFFE000u;
        lp[e] = __float_as_uint(__fsub_rn(w[e], __uint_as_float(hp[e])));
    }
    *reinterpret_cast<uint4*>(st + OFF_A_RAW + off)  = h;
    *reinterpret_cast<uint4*>(st + OFF_A_TAIL + off) = l;
}

// QTYPE = 0: A is an F32 view loaded by TMA. QTYPE = ggml Q-type: A is decoded from packed blocks by
// the split warps (QTRANS = 0: A = W, K-major; QTRANS = 1: A = transpose(W), MN-major).
// CG = 1: one CTA per tile. CG = 2: a cluster of two CTAs per tile (tcgen05 cta_group::2); CTA rank
// r of the pair owns rows m0 + 128 r of D and B rows n0 + 128 r of the tile. Each CTA's TMA lands on
// its own `full` barrier; its split warps then arrive on the leader's `split` barrier, the leader's
// single thread issues the pair's MMAs and commits them to both CTAs' `empty` / `acc_full`
// barriers, and both CTAs' epilogue warps arrive on the leader's `acc_empty`.
// PT = 1 (fused kernel on CTA pairs): the producer also stages each stage's packed weight bytes by
// TMA through tmA (a uint8 map of the packed rows), and the split warps decode from shared memory;
// PT = 0: the split warps load the packed words from global memory themselves.
// The TMA-staged fused decode splits its warps into kPtGroups groups that take alternate stages,
// so one group's waits, fence and arrival overlap the other group's decode.
constexpr int kPtGroups = 2;

template <int QTYPE, int QTRANS, int CG, int PT = 0>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    tf32x3_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       const __grid_constant__ CUtensorMap tmBt, const __grid_constant__ CUtensorMap tmD,
                       const __grid_constant__ CUtensorMap tmW, const __grid_constant__ TcParams p) {
    using G = typename KernelGeo<QTYPE, QTRANS, CG, PT>::type;
    constexpr int TS = KernelGeo<QTYPE, QTRANS, CG, PT>::TS;
    constexpr bool PTMA = QTYPE != 0 && PT != 0;
    constexpr int NSPLIT = TS ? TS : G::STAGES;  // slots of the split barriers
    constexpr bool PAIR = CG == 2;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Barriers* bars = reinterpret_cast<Barriers*>(smem + G::EPI_OFF + EPI_BUFS * EPI_BUF_BYTES);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = PAIR ? cluster_ctarank() : 0u;  // 0 = leader
    const int64_t tile0 = blockIdx.x / CG, tile_step = gridDim.x / CG;

    if (threadIdx.x == 0) {
        for (int s = 0; s < G::STAGES; ++s) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int s = 0; s < NSPLIT; ++s) {
            mbar_init(&bars->split[s], (SPLIT_WARPS / (PTMA ? kPtGroups : 1)) * CG);
            mbar_init(&bars->tail_empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&bars->acc_full[a], 1);
            mbar_init(&bars->acc_empty[a], EPI_WARPS * CG);
        }
        mbar_init(&bars->mma_done, 1);
        fence_barrier_init();
        if (QTYPE == 0 || PTMA) prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        if (p.b_pretail) prefetch_tmap(&tmBt);
        if (p.tma_store) prefetch_tmap(&tmD);
    }
    if (warp == 1) {
        tmem_alloc<CG>(&bars->tmem_slot, TMEM_COLS);
        tmem_relinquish<CG>();
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR) cluster_sync();  // both CTAs' barriers exist before any remote arrival
    tc_fence_after();
    const uint32_t tmem_base = bars->tmem_slot;
    const uint32_t smem_base = smem_u32(smem);

    if (warp == 0) {
        // ---------------------------------------------------------------- TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (UnitCursor<CG> cur(p); cur.live(p) && ok; cur.next(p)) {
                const UnitSpan us = cur.span(p);
                const TileCoord tc = tile_coord<CG>(p, us.tile);
                const int am0 = tc.m0 + BM * static_cast<int>(rank);              // this CTA's A rows
                const int bn0 = tc.n0 + G::BN_CTA * static_cast<int>(rank);       // this CTA's B rows
                // source-plane round and k-block of the virtual k-block vkb
                int r = us.kv0 / p.k_blocks, kb = us.kv0 - r * p.k_blocks;
                for (int vkb = us.kv0; vkb < us.kv1; ++vkb, ++it) {
                    const int sp2 = tc.p2 + p.planes2 * (r % p.red2), sp3 = tc.p3 + p.planes3 * (r / p.red2);
                    const int a2 = sp2 % p.a_ne2, a3 = sp3 % p.a_ne3;
                    const int b2 = sp2 % p.b_ne2, b3 = sp3 % p.b_ne3;
                    const int s = it % G::STAGES;
                    const uint32_t ph = (it / G::STAGES) & 1u;
                    if (!mbar_wait_scoped<PAIR>(&bars->empty[s], ph ^ 1u, TRC_DEVERR_WAIT_EMPTY)) { ok = false; break; }
                    const uint32_t st = smem_base + s * G::STAGE_BYTES;
                    constexpr int pq_tx = PTMA ? PackedBox<QTYPE, QTRANS>::kBytes : 0;
                    mbar_arrive_expect_tx(&bars->full[s], (QTYPE == 0 ? G::RAW_TX_BYTES : G::B_BYTES) +
                                                              (!TS && p.b_pretail ? G::B_BYTES : 0) + pq_tx);
                    const int k0 = kb * BK;
                    if constexpr (PTMA) {
                        // the stage's packed bytes: from the 16-byte boundary at or below the first one
                        constexpr int bbq = QuantTraits<QTYPE>::kBytes;
                        const int blk = QTRANS ? (am0 >> 5) : (k0 >> 5);
                        tma_load_4d(st + G::OFF_PQ, &tmA, &bars->full[s], (blk * bbq) & ~15, QTRANS ? k0 : am0, 0, 0);
                    }
                    if constexpr (QTYPE == 0) {
                        if (!p.a_mn) {
                            tma_load_4d(st + G::OFF_A_RAW, &tmA, &bars->full[s], k0, am0, a2, a3);
                        } else if (p.a_tma5) {
                            tma_load_5d(st + G::OFF_A_RAW, &tmA, &bars->full[s], 0, k0, am0 / 32, a2, a3);
                        } else {
#pragma unroll
                            for (int c = 0; c < BM / 32; ++c)
                                tma_load_4d(st + G::OFF_A_RAW + c * 2048, &tmA, &bars->full[s], am0 + 32 * c, k0, a2,
                                            a3);
                        }
                    }
                    // B raw, and with b_pretail B's precomputed tail through a map of the same geometry
                    for (int part = 0; part < (!TS && p.b_pretail ? 2 : 1); ++part) {
                        const CUtensorMap* mb = part == 0 ? &tmB : &tmBt;
                        const uint32_t dstb = st + (part == 0 ? G::OFF_B_RAW : G::OFF_B_TAIL);
                        if (!p.b_mn) {
                            tma_load_4d(dstb, mb, &bars->full[s], k0, bn0, b2, b3);
                        } else if (p.b_tma5) {
                            tma_load_5d(dstb, mb, &bars->full[s], 0, k0, bn0 / 32, b2, b3);
                        } else {
#pragma unroll
                            for (int c = 0; c < G::BN_CTA / 32; ++c)
                                tma_load_4d(dstb + c * 2048, mb, &bars->full[s], bn0 + 32 * c, k0, b2, b3);
                        }
                    }
                    if (++kb == p.k_blocks) {
                        kb = 0;
                        ++r;
                    }
                }
            }
            // Drain: the last load issued into each stage must have landed before the CTA exits.
            const uint32_t n_issued = it;
            for (uint32_t q = (n_issued > G::STAGES ? n_issued - G::STAGES : 0); q < n_issued; ++q)
                mbar_wait_drain(&bars->full[q % G::STAGES], (q / G::STAGES) & 1u);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- UMMA issuer (leader only)
        if (lane == 0 && rank == 0) {
            const uint32_t idesc = make_idesc_tf32(G::TILE_M, BN, p.a_mn, p.b_mn);
            // uses0/uses1: chunks committed so far into TMEM buffer 0/1 (scalars, kept in registers)
            uint32_t it = 0, tcount = 0, uses0 = 0, uses1 = 0;
            bool ok = true;
            for (UnitCursor<CG> cur(p); cur.live(p) && ok; cur.next(p), ++tcount) {
                const UnitSpan us = cur.span(p);
                const int tb = tcount & 1;  // this unit's running-total buffer; chunks >= 1 use tb ^ 1
                for (int kb0 = us.kv0; kb0 < us.kv1 && ok; kb0 += CHUNK_KB) {
                    const int b = kb0 == us.kv0 ? tb : tb ^ 1;
                    const uint32_t ub = b ? uses1 : uses0;
                    if (!mbar_wait_scoped<PAIR>(&bars->acc_empty[b], (ub & 1u) ^ 1u, TRC_DEVERR_WAIT_ACCFREE)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d_tmem = tmem_base + b * BN;
                    const int kb1 = min(us.kv1, kb0 + CHUNK_KB);
                    for (int kb = kb0; kb < kb1; ++kb, ++it) {
                        const int s = it % G::STAGES;
                        const int ts = TS ? static_cast<int>(it % NSPLIT) : s;  // tail slot / split barrier
                        if (!mbar_wait_scoped<PAIR>(&bars->split[ts], (it / NSPLIT) & 1u, TRC_DEVERR_WAIT_XFORM)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint32_t st = smem_base + s * G::STAGE_BYTES;
                        // tails: beside the raw tiles, or in tail slot ts of the separate ring (which
                        // also holds the fused kernel's decoded A head)
                        const uint32_t tsl = smem_base + G::OFF_TAILS + ts * G::TAIL_BYTES;
                        const uint32_t ah = TS && QTYPE != 0 ? tsl + G::T_A_HEAD : st + G::OFF_A_RAW;
                        const uint32_t ta = TS ? tsl + G::T_A_TAIL : st + G::OFF_A_TAIL;
                        const uint32_t tb = TS ? tsl + G::T_B_TAIL : st + G::OFF_B_TAIL;
#pragma unroll
                        for (int kk = 0; kk < BK / 8; ++kk) {
                            const uint64_t a_raw  = p.a_mn ? desc_mnmajor(ah, kk) : desc_kmajor(ah, kk);
                            const uint64_t a_tail = p.a_mn ? desc_mnmajor(ta, kk) : desc_kmajor(ta, kk);
                            const uint64_t b_raw  = p.b_mn ? desc_mnmajor(st + G::OFF_B_RAW, kk) : desc_kmajor(st + G::OFF_B_RAW, kk);
                            const uint64_t b_tail = p.b_mn ? desc_mnmajor(tb, kk) : desc_kmajor(tb, kk);
                            umma_tf32<CG>(d_tmem, a_tail, b_raw, idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
                            umma_tf32<CG>(d_tmem, a_raw, b_tail, idesc, 1u);
                            umma_tf32<CG>(d_tmem, a_raw, b_raw, idesc, 1u);
                        }
                        // frees the stage (in both CTAs) once these MMAs have read it
                        if constexpr (PAIR) {
                            umma_commit_pair_both(&bars->empty[s], 0x3);
                            if constexpr (TS != 0) umma_commit_pair_both(&bars->tail_empty[ts], 0x3);
                        } else {
                            umma_commit(&bars->empty[s]);
                            if constexpr (TS != 0) umma_commit(&bars->tail_empty[ts]);
                        }
                    }
                    if (!ok) break;
                    // this chunk is complete in TMEM buffer b
                    if constexpr (PAIR) {
                        umma_commit_pair_both(&bars->acc_full[b], 0x3);
                    } else {
                        umma_commit(&bars->acc_full[b]);
                    }
                    if (b) ++uses1; else ++uses0;
                }
            }
            // All MMAs of this thread must be complete before TMEM is released.
            if constexpr (PAIR) umma_commit_pair_local(&bars->mma_done);
            else umma_commit(&bars->mma_done);
            mbar_wait_drain(&bars->mma_done, 0);
        }
    } else if (warp < EPI_WARP0) {
        // ---------------------------------------------------------------- split warps
        const int t = threadIdx.x - SPLIT_WARP0 * 32;
        constexpr int nA = G::A_BYTES / 16, nAll = (G::A_BYTES + G::B_BYTES) / 16;
        // the leader's split barrier of stage s, as this CTA addresses it
        auto arrive_split = [&](int s) {
            if constexpr (PAIR) mbar_arrive_cluster(mapa_shared(&bars->split[s], 0));
            else mbar_arrive(&bars->split[s]);
        };
        if constexpr (PTMA) {
            // Fused kernel, packed bytes staged by TMA: once the stage has landed, each thread of the
            // stage's warp group decodes its A quads from the stage's packed box into the head + tail
            // tiles. Group g (warps g*4 .. g*4+3 of the split warps) takes the stages it with
            // it % kPtGroups == g.
            constexpr int NT = SPLIT_WARPS * 32 / kPtGroups;
            constexpr int QPT = A_QUADS / NT;
            static_assert(A_QUADS % NT == 0, "quads per thread");
            using PB = PackedBox<QTYPE, QTRANS>;
            const int group = t / NT, tg = t - group * NT;
            int qoff[QPT];
#pragma unroll
            for (int i = 0; i < QPT; ++i) qoff[i] = quad_offset<QTRANS>(tg + NT * i);
            const int row_off = BM * static_cast<int>(rank);
            uint32_t it = 0;
            bool ok = true;
            for (UnitCursor<CG> cur(p); cur.live(p) && ok; cur.next(p)) {
                const UnitSpan us = cur.span(p);
                const int am0 = tile_coord<CG>(p, us.tile).m0 + row_off;
                for (int kb = us.kv0; kb < us.kv1; ++kb, ++it) {
                    if (static_cast<int>(it % kPtGroups) != group) continue;
                    const int s = it % G::STAGES;
                    if (!mbar_wait(&bars->full[s], (it / G::STAGES) & 1u, TRC_DEVERR_WAIT_FULL)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + s * G::STAGE_BYTES;
                    // the decoded head / tail tiles go to tail slot ts once the MMAs that last read
                    // it have completed (TS = 0: beside the raw tiles)
                    const int ts = TS ? static_cast<int>(it % NSPLIT) : s;
                    uint8_t* tsl = st;
                    if constexpr (TS != 0) {
                        if (it >= static_cast<uint32_t>(NSPLIT) &&
                            !mbar_wait_scoped<PAIR>(&bars->tail_empty[ts], ((it / NSPLIT) & 1u) ^ 1u, TRC_DEVERR_WAIT_EMPTY)) {
                            ok = false;
                            break;
                        }
                        tsl = smem + G::OFF_TAILS + ts * G::TAIL_BYTES;
                    }
                    const int k0 = kb * BK;
                    const int blk = QTRANS ? (am0 >> 5) : (k0 >> 5);
                    const uint32_t box = smem_u32(st + G::OFF_PQ) + ((blk * PB::kBB) & 15);
#pragma unroll
                    for (int i = 0; i < QPT; ++i) {
                        const int q = tg + NT * i;
                        float w[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                        // rows outside the matrix are zero-filled by TMA; they are written as +0 here
                        // exactly as the F32 operand's zero fill reads
                        uint32_t bp;
                        int j0;
                        bool valid;
                        if constexpr (QTRANS == 0) {
                            bp = box + (q >> 2) * PB::kW;
                            j0 = (k0 & 16) + 4 * (q & 3);
                            valid = am0 + (q >> 2) < p.M;
                        } else {
                            bp = box + (q >> 5) * PB::kW + ((q & 31) >> 3) * PB::kBB;
                            j0 = (q & 7) * 4;
                            valid = k0 + (q >> 5) < p.K && am0 + 32 * ((q & 31) >> 3) < p.M;
                        }
                        if (valid) {
                            QuadWords wd;
                            load_quad_words_smem<QTYPE>(bp, j0, wd);
                            decode_quad_words<QTYPE>(wd, j0, w);
                        }
                        store_quad_head_tail(tsl, qoff[i], w);
                    }
                    if constexpr (TS != 0) {
                        split_chunks_rings<(nAll - nA + NT - 1) / NT>(st + G::OFF_B_RAW, tsl + G::T_B_TAIL, tg,
                                                                      nAll - nA, NT);
                    } else if (!p.b_pretail) {
                        split_chunks<G, (nAll - nA + NT - 1) / NT>(st, nA + tg, nAll, NT, nA);
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) arrive_split(ts);
                }
            }
        } else if constexpr (QTYPE != 0) {
            // Fused kernel: the split warps decode the stage's A quads (up to 2 per thread) from
            // the packed blocks into head + tail tiles, then split the TMA-loaded B tile. The packed
            // words are loaded two stages ahead of their decode (a stage takes about one loaded L2
            // latency), so the loads overlap two stages of decode, split and waits.
            constexpr int NT = SPLIT_WARPS * 32;
            constexpr int QPT = (A_QUADS + NT - 1) / NT;
            int qoff[QPT];
#pragma unroll
            for (int i = 0; i < QPT; ++i) qoff[i] = (t + NT * i) < A_QUADS ? quad_offset<QTRANS>(t + NT * i) : 0;
            const int row_off = BM * static_cast<int>(rank);
            // The loop is instantiated twice: with split-K (a unit is a tile's k-blocks [kv0, kv1))
            // and without (a unit is a whole tile). These warps run at the register cap, and the
            // unsplit loop keeps the unsplit kernel's lean schedule.
            auto run = [&](auto split_tag) {
                constexpr bool SPLIT = decltype(split_tag)::value;
                // look-ahead cursor: the (unit, k-block) whose packed words are loaded next
                int64_t lunit = tile0;
                int lkb = 0, lkv1 = p.k_blocks;
                const uint8_t* lbase[QPT];  // packed-row pointers of lunit's tile
                auto set_unit = [&]() {
                    const bool live = lunit < p.total_units;
                    int m0 = 0;
                    if (live) {
                        if constexpr (SPLIT) {
                            const UnitSpan us = unit_span(p, lunit);
                            lkb  = us.kv0;
                            lkv1 = us.kv1;
                            m0   = tile_coord<CG>(p, us.tile).m0 + row_off;
                        } else {
                            m0 = tile_coord<CG>(p, lunit).m0 + row_off;
                        }
                    }
#pragma unroll
                    for (int i = 0; i < QPT; ++i)
                        lbase[i] = (live && t + NT * i < A_QUADS) ? quad_tile_base<QTYPE, QTRANS>(p, m0, t + NT * i)
                                                                 : nullptr;
                };
                // loads the cursor's words into w and advances the cursor; bit i of the result: quad
                // i lies inside the matrix (else it is decoded as zeros)
                auto load_next = [&](QuadWords (&w)[QPT]) -> uint32_t {
                    uint32_t valid = 0;
                    if (lunit < p.total_units) {
#pragma unroll
                        for (int i = 0; i < QPT; ++i) {
                            int j0 = 0;
                            const uint8_t* blk = quad_block<QTYPE, QTRANS>(p, lbase[i], lkb * BK, t + NT * i, j0);
                            if (blk != nullptr) {
                                load_quad_words<QTYPE>(blk, j0, w[i]);
                                valid |= 1u << i;
                            }
                        }
                    }
                    if (++lkb == (SPLIT ? lkv1 : p.k_blocks)) {
                        if constexpr (!SPLIT) lkb = 0;
                        lunit += tile_step;
                        set_unit();
                    }
                    return valid;
                };
                set_unit();
                QuadWords w0[QPT], w1[QPT];
                uint32_t v0 = load_next(w0);
                uint32_t v1 = load_next(w1);
                int64_t unit = tile0;
                int kb = 0, kv1 = p.k_blocks;
                if constexpr (SPLIT) {
                    if (unit < p.total_units) {
                        const UnitSpan us = unit_span(p, unit);
                        kb  = us.kv0;
                        kv1 = us.kv1;
                    }
                }
                uint32_t it = 0;
                while (unit < p.total_units) {
                    QuadWords w2[QPT];
                    const uint32_t v2 = load_next(w2);
                    const int s = it % G::STAGES;
                    uint8_t* st = smem + s * G::STAGE_BYTES;
                    if (it >= G::STAGES &&
                        !mbar_wait_scoped<PAIR>(&bars->empty[s], ((it / G::STAGES) & 1u) ^ 1u, TRC_DEVERR_WAIT_EMPTY))
                        break;
#pragma unroll
                    for (int i = 0; i < QPT; ++i) {
                        if (t + NT * i >= A_QUADS) continue;
                        float w[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                        if ((v0 >> i) & 1u) decode_quad_words<QTYPE>(w0[i], quad_j0<QTRANS>(kb, t + NT * i), w);
                        store_quad_head_tail(st, qoff[i], w);
                    }
                    if (!mbar_wait(&bars->full[s], (it / G::STAGES) & 1u, TRC_DEVERR_WAIT_FULL)) break;
                    if (!p.b_pretail) split_chunks<G, (nAll - nA + NT - 1) / NT>(st, nA + t, nAll, NT, nA);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) arrive_split(s);
#pragma unroll
                    for (int i = 0; i < QPT; ++i) {
                        w0[i] = w1[i];
                        w1[i] = w2[i];
                    }
                    v0 = v1;
                    v1 = v2;
                    if (++kb == (SPLIT ? kv1 : p.k_blocks)) {
                        unit += tile_step;
                        if constexpr (SPLIT) {
                            if (unit < p.total_units) {
                                const UnitSpan us = unit_span(p, unit);
                                kb  = us.kv0;
                                kv1 = us.kv1;
                            }
                        } else {
                            kb = 0;
                        }
                    }
                    ++it;
                }
            };
            if (p.splits > 1) run(std::true_type{});
            else run(std::false_type{});
        } else {
            // F32 kernel: all split warps split the A and B tiles of each raw slot into the tail slot
            // the stage uses, once the MMAs that last read that tail slot have completed.
            const int i_step = SPLIT_WARPS * 32;
            uint32_t it = 0;
            bool ok = true;
            for (UnitCursor<CG> cur(p); cur.live(p) && ok; cur.next(p)) {
                const UnitSpan us = cur.span(p);
                for (int kb = us.kv0; kb < us.kv1; ++kb, ++it) {
                    const int s = it % G::STAGES;
                    if (!mbar_wait(&bars->full[s], (it / G::STAGES) & 1u, TRC_DEVERR_WAIT_FULL)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = smem + s * G::STAGE_BYTES;
                    if constexpr (TS != 0) {
                        const int ts = static_cast<int>(it % NSPLIT);
                        if (it >= static_cast<uint32_t>(NSPLIT) &&
                            !mbar_wait_scoped<PAIR>(&bars->tail_empty[ts], ((it / NSPLIT) & 1u) ^ 1u, TRC_DEVERR_WAIT_EMPTY)) {
                            ok = false;
                            break;
                        }
                        split_chunks_rings<(nAll + SPLIT_WARPS * 32 - 1) / (SPLIT_WARPS * 32)>(
                            st, smem + G::OFF_TAILS + ts * G::TAIL_BYTES, t, nAll, i_step);
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) arrive_split(ts);
                    } else {
                        const int i_end = p.b_pretail ? nA : nAll;  // B's tails arrive precomputed
                        split_chunks<G, (nAll + SPLIT_WARPS * 32 - 1) / (SPLIT_WARPS * 32)>(st, t, i_end, i_step, nA);
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) arrive_split(s);
                    }
                }
            }
        }
    } else {
        // ---------------------------------------------------------------- epilogue
        // Per tile: chunk 0 lands in buffer tb (the running total T), every further chunk in tb^1 (X)
        // and is added into T with round-to-nearest fp32 adds; the final sum goes to global memory.
        // Two teams of four warps split the 256 columns, so a chunk's promotion (which the MMA
        // issuer waits for before it reuses X) takes half as long.
        const int q = warp & 3;  // TMEM lane quarter this warp may access (warp id mod 4)
        const int team = (warp - EPI_WARP0) >> 2;
        const int row = q * 32 + lane;
        const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
        uint32_t tcount = 0, uses_t = 0, uses_x = 0;  // chunks consumed from this tile's T / X buffer roles
        uint32_t uses0 = 0, uses1 = 0;                // ... per physical buffer (scalars, in registers)
        uint32_t gcount = 0;                          // column groups this team staged for TMA stores
        const bool team_leader = (threadIdx.x == (EPI_WARP0 + 4 * team) * 32);
        const int team_bar = EPI_BAR_TEAM0 + team;
        uint8_t* stage_buf = smem + G::EPI_OFF + team * EPI_BUF_BYTES;
        // the leader's acc_empty barrier of buffer b, as this CTA addresses it
        auto release_acc = [&](int b) {
            if constexpr (PAIR) mbar_arrive_cluster(mapa_shared(&bars->acc_empty[b], 0));
            else mbar_arrive(&bars->acc_empty[b]);
        };
        bool ok = true;
        for (UnitCursor<CG> cur(p); cur.live(p) && ok; cur.next(p), ++tcount) {
            const UnitSpan us = cur.span(p);
            const UnitDest dest = cur.dest(p, us);
            const int tb = tcount & 1, xb = tb ^ 1;
            const TileCoord tc = tile_coord<CG>(p, us.tile);
            const int dm0 = tc.m0 + BM * static_cast<int>(rank);  // this CTA's rows of D
            const int m = dm0 + row;
            char* drow = p.d + static_cast<int64_t>(tc.p2) * p.d_s2 + static_cast<int64_t>(tc.p3) * p.d_s3 +
                         static_cast<int64_t>(m) * p.d_sm;
            const int n_valid = min(BN, p.N - tc.n0);
            // uniform across a team; none when this CTA's rows all lie past M (the second CTA of a
            // pair on the last row tile): nothing to add or store, and no store box starts outside D
            const int n_groups = dm0 < p.M ? (n_valid + 31) / 32 : 0;
            const int c_begin = 4 * team, c_end = min(n_groups, 4 * team + 4);
            // the final store goes by 16-column groups (two per 32-column group of the promotion)
            const int n_groups16 = dm0 < p.M ? (n_valid + 15) / 16 : 0;
            const int g_begin = 8 * team, g_end = min(n_groups16, 8 * team + 8);
            const uint32_t t_addr = tmem_base + lane_off + tb * BN;
            const uint32_t x_addr = tmem_base + lane_off + xb * BN;
            uses_t = tb ? uses1 : uses0;
            // every wait is followed by a vote of all epilogue warps, so that they all leave or all
            // stay (a team meets again at its named barrier of the TMA-store staging)
            if (!named_barrier_and(EPI_BAR_ALL, EPI_WARPS * 32,
                                   mbar_wait_scoped<PAIR>(&bars->acc_full[tb], uses_t & 1u, TRC_DEVERR_WAIT_ACCUM)))
                break;
            if (tb) ++uses1; else ++uses0;
            tc_fence_after();
            for (int kb0 = us.kv0 + CHUNK_KB; kb0 < us.kv1; kb0 += CHUNK_KB) {
                uses_x = xb ? uses1 : uses0;
                if (!named_barrier_and(EPI_BAR_ALL, EPI_WARPS * 32,
                                       mbar_wait_scoped<PAIR>(&bars->acc_full[xb], uses_x & 1u, TRC_DEVERR_WAIT_ACCUM))) {
                    ok = false;
                    break;
                }
                if (xb) ++uses1; else ++uses0;
                tc_fence_after();
#pragma unroll 1
                for (int c = c_begin; c < c_end; ++c) {
                    uint32_t x[32], t[32];
                    tmem_ld_32x32b_x32(x_addr + c * 32, x);
                    tmem_ld_32x32b_x32(t_addr + c * 32, t);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 32; ++e) t[e] = __float_as_uint(__fadd_rn(__uint_as_float(t[e]), __uint_as_float(x[e])));
                    tmem_st_32x32b_x32(t_addr + c * 32, t);
                }
                tmem_st_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) release_acc(xb);  // chunk buffer free for the next chunk
            }
            if (!ok) break;
#pragma unroll 1
            for (int g = g_begin; g < g_end; ++g) {
                uint32_t r[16];
                tmem_ld_32x32b_x16(t_addr + g * 16, r);
                tmem_ld_wait();
                if (p.tma_store) {
                    // Stage the 128 x 16 group column-major (each column's 128 rows contiguous, the
                    // layout of the TMA box) in one of the team's two staging halves, and let the team
                    // leader store or reduce-add it. A half is refilled once the store issued two
                    // groups earlier has read it, so one store is always in flight while the next
                    // group is staged.
                    float* sb = reinterpret_cast<float*>(stage_buf) + (gcount & 1u) * (BM * 16);
                    if (gcount >= 2) {
                        if (team_leader) bulk_wait_group_read<1>();  // the store of group gcount - 2 has read sb
                        named_barrier_sync(team_bar, 128);
                    }
#pragma unroll
                    for (int e = 0; e < 16; ++e) sb[e * BM + row] = __uint_as_float(r[e]);
                    fence_proxy_async_smem();
                    named_barrier_sync(team_bar, 128);
                    if (team_leader) {
                        const uint32_t src = smem_u32(sb);
                        if (dest == kReduceW) tma_reduce_add_4d(&tmW, src, dm0, tc.n0 + g * 16, tc.p2, tc.p3);
                        else if (dest == kReduceD) tma_reduce_add_4d(&tmD, src, dm0, tc.n0 + g * 16, tc.p2, tc.p3);
                        else tma_store_4d(&tmD, src, dm0, tc.n0 + g * 16, tc.p2, tc.p3);
                        bulk_commit_group();
                    }
                    ++gcount;
                } else if (m < p.M) {
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int n = tc.n0 + g * 16 + e;
                        if (n < p.N) {
                            float* o = reinterpret_cast<float*>(drow + static_cast<int64_t>(n) * p.d_sn);
                            const float v = __uint_as_float(r[e]);
                            *o = p.accumulate ? __fadd_rn(*o, v) : v;
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) release_acc(tb);
        }
        if (team_leader) bulk_wait_group_all();  // every TMA store has completed before the CTA exits
    }

    tc_fence_before();
    __syncthreads();
    // CG = 2: the leader's MMAs (which write both CTAs' TMEM and read both CTAs' shared memory) and
    // every remote arrival are complete before either CTA frees TMEM or exits.
    if constexpr (PAIR) cluster_sync();
    tc_fence_after();
    if (warp == 1) tmem_dealloc<CG>(tmem_base, TMEM_COLS);
}

// ------------------------------------------------------------------ host side
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

bool stride_ok(int64_t s) { return s > 0 && (s % 16) == 0 && s < (int64_t(1) << 40); }

// Builds the tensor map of one operand: a ggml view with ne0 = K, ne1 = rows (M or N).
// Returns false when TMA cannot address the view (the caller then uses the SIMT kernel).
bool encode_operand(const trc_cuda_view& v, int box_rows, bool& mn_major, CUtensorMap& map, bool* tma5 = nullptr) {
    if (tma5 != nullptr) *tma5 = false;
    if ((reinterpret_cast<uint64_t>(v.data) & 15u) != 0) return false;
    const int64_t K = v.ne[0], R = v.ne[1];
    if (K >= (int64_t(1) << 31) || R >= (int64_t(1) << 31)) return false;
    cuuint64_t dims[4];
    cuuint64_t strides[3];
    cuuint32_t box[4];
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    if (v.nb[0] == 4 && (R == 1 || stride_ok(v.nb[1]))) {
        mn_major = false;
        dims[0] = K; dims[1] = R;
        strides[0] = R == 1 ? static_cast<cuuint64_t>((K * 4 + 15) / 16 * 16) : v.nb[1];
        box[0] = BK; box[1] = box_rows;
    } else if (v.nb[1] == 4 && (K == 1 || stride_ok(v.nb[0]))) {
        mn_major = true;
        dims[0] = R; dims[1] = K;
        strides[0] = K == 1 ? static_cast<cuuint64_t>((R * 4 + 15) / 16 * 16) : v.nb[0];
        box[0] = 32; box[1] = BK;
    } else {
        return false;
    }
    dims[2] = v.ne[2];
    dims[3] = v.ne[3];
    // Planes of extent 1 get a dummy stride (never stepped) that keeps the strides monotonic.
    const cuuint64_t plane_bytes = strides[0] * dims[1];
    if (v.ne[2] > 1) {
        if (!stride_ok(v.nb[2])) return false;
        strides[1] = v.nb[2];
    } else {
        strides[1] = (plane_bytes + 15) / 16 * 16;
    }
    if (v.ne[3] > 1) {
        if (!stride_ok(v.nb[3])) return false;
        strides[2] = v.nb[3];
    } else {
        strides[2] = (strides[1] * dims[2] + 15) / 16 * 16;
    }
    if (strides[1] >= (cuuint64_t(1) << 40) || strides[2] >= (cuuint64_t(1) << 40)) return false;
    box[2] = 1;
    box[3] = 1;
    auto enc = tensor_map_encoder();
    if (enc == nullptr) return false;
    if (mn_major && tma5 != nullptr && R % 32 == 0 && R / 32 < (int64_t(1) << 31)) {
        // One box per stage: dims (32 MN elements, K, R/32 chunks of 32, planes), so the box
        // {32, 16, box_rows/32} lands chunk-major -- chunk c at c x 2 KiB -- the descriptor layout.
        const cuuint64_t dims5[5]    = {32, dims[1], static_cast<cuuint64_t>(R / 32), dims[2], dims[3]};
        const cuuint64_t strides5[4] = {strides[0], 128, strides[1], strides[2]};
        const cuuint32_t box5[5]     = {32, static_cast<cuuint32_t>(BK), static_cast<cuuint32_t>(box_rows / 32), 1, 1};
        const cuuint32_t estr5[5]    = {1, 1, 1, 1, 1};
        if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 5, v.data, dims5, strides5, box5, estr5,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS) {
            *tma5 = true;
            return true;
        }
    }
    const CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, v.data, dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE,
                           mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_64B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// Tensor map of D for the TMA-store epilogue, in the kernel's orientation: rows (TMEM lanes) M with
// byte stride sm, columns N with stride sn, then the two plane dimensions. Box: 128 rows x 32
// columns, no swizzle (the epilogue stages each group column-major). False when TMA cannot write
// D (rows not contiguous, unaligned base or strides); the epilogue then stores element by element.
bool encode_output(void* data, int64_t M, int64_t N, int64_t P2, int64_t P3, int64_t sm, int64_t sn, int64_t s2,
                   int64_t s3, CUtensorMap& map) {
    if (sm != 4 || (reinterpret_cast<uint64_t>(data) & 15u) != 0) return false;
    if (M >= (int64_t(1) << 31) || N >= (int64_t(1) << 31)) return false;
    cuuint64_t dims[4] = {static_cast<cuuint64_t>(M), static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(P2),
                          static_cast<cuuint64_t>(P3)};
    cuuint64_t strides[3];
    if (N > 1) {
        if (!stride_ok(sn)) return false;
        strides[0] = sn;
    } else {
        strides[0] = static_cast<cuuint64_t>((M * 4 + 15) / 16 * 16);
    }
    if (P2 > 1) {
        if (!stride_ok(s2)) return false;
        strides[1] = s2;
    } else {
        strides[1] = (strides[0] * dims[1] + 15) / 16 * 16;
    }
    if (P3 > 1) {
        if (!stride_ok(s3)) return false;
        strides[2] = s3;
    } else {
        strides[2] = (strides[1] * dims[2] + 15) / 16 * 16;
    }
    if (strides[1] >= (cuuint64_t(1) << 40) || strides[2] >= (cuuint64_t(1) << 40)) return false;
    const cuuint32_t box[4]  = {BM, 16, 1, 1};  // the epilogue's 128 x 16 staging group
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    auto enc = tensor_map_encoder();
    if (enc == nullptr) return false;
    return enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, data, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

// Launches one instantiation; the >48 KiB dynamic shared memory opt-in is set once per device.
// Tails of a B operand, written once before the GEMM: the same logical shape as `src`, unit stride
// along src's unit-stride dimension (ne0 when K-major, ne1 when MN-major), rows padded to 16 bytes.
__global__ void pretail_kernel(View4 src, float* dst, int mn, int64_t pitch_elems, int64_t n) {
    const int64_t nf = mn ? src.ne[1] : src.ne[0];  // fast (unit-stride) dimension
    const int64_t ns = mn ? src.ne[0] : src.ne[1];
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        const int64_t f = i % nf;
        int64_t r = i / nf;
        const int64_t sl = r % ns;
        r /= ns;
        const int64_t i2 = r % src.ne[2], i3 = r / src.ne[2];
        const int64_t i0 = mn ? sl : f, i1 = mn ? f : sl;
        const uint32_t u = *reinterpret_cast<const uint32_t*>(src.data + i0 * src.nb[0] + i1 * src.nb[1] + i2 * src.nb[2] +
                                                              i3 * src.nb[3]);
        dst[((i3 * src.ne[2] + i2) * ns + sl) * pitch_elems + f] = __uint_as_float(tf32_tail_bits(u));
    }
}

// Computes B's tails into stream-ordered scratch (freed on the stream after the GEMM) and encodes
// their tensor map. False (nothing allocated) when it does not pay or memory is short.
struct Pretail {
    void*       buf = nullptr;
    CUtensorMap map;
};


bool make_pretail(const trc_cuda_view& B, int box_rows, bool b_mn, bool b_tma5, cudaStream_t stream, Pretail& out) {
    retain_pool_once();
    const int64_t nf = b_mn ? B.ne[1] : B.ne[0], ns = b_mn ? B.ne[0] : B.ne[1];
    const int64_t pitch = (nf + 3) / 4 * 4;  // floats; 16-byte rows for TMA
    const int64_t planes = B.ne[2] * B.ne[3];
    const size_t bytes = static_cast<size_t>(pitch * ns * planes) * sizeof(float);
    if (cudaMallocAsync(&out.buf, bytes, stream) != cudaSuccess) {
        cudaGetLastError();
        out.buf = nullptr;
        return false;
    }
    trc_cuda_view tv;
    tv.data = out.buf;
    for (int i = 0; i < 4; ++i) tv.ne[i] = B.ne[i];
    const int64_t row = pitch * 4, plane = row * ns;
    tv.nb[b_mn ? 1 : 0] = 4;
    tv.nb[b_mn ? 0 : 1] = row;
    tv.nb[2] = plane;
    tv.nb[3] = plane * B.ne[2];
    bool mn = false, t5 = false;
    if (!encode_operand(tv, box_rows, mn, out.map, &t5) || mn != b_mn || t5 != b_tma5) {
        cudaFreeAsync(out.buf, stream);
        out.buf = nullptr;
        return false;
    }
    const int64_t n = nf * ns * planes;
    const int sms = std::max(1, sm_count_current());
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, int64_t(sms) * 16));
    pretail_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(to_view4(B), static_cast<float*>(out.buf),
                                                                     b_mn ? 1 : 0, pitch, n);
    note_launch();
    if (check_launch() != TRC_CUDA_OK) {
        cudaFreeAsync(out.buf, stream);
        out.buf = nullptr;
        return false;
    }
    return true;
}

// Tensor map of a packed weight for the fused kernel's TMA staging: uint8 elements, the packed
// rows (row_bytes each, `rows` of them) as a 2-D tensor, the box of PackedBox for the type and
// orientation. False when TMA cannot address it (base or row pitch not 16-byte multiples).
bool encode_packed(const void* blocks, int64_t row_bytes, int64_t rows, int type, bool transposed, CUtensorMap& map) {
    auto enc = tensor_map_encoder();
    if (enc == nullptr || (reinterpret_cast<uint64_t>(blocks) & 15u) != 0 || row_bytes % 16 != 0 || row_bytes <= 0 ||
        rows <= 0 || row_bytes * rows >= (int64_t(1) << 40))
        return false;
    int w = 0, h = 0;
    switch (type) {
#define TRC_PB(T)                                                                                                  \
    case T:                                                                                                        \
        w = transposed ? PackedBox<T, 1>::kW : PackedBox<T, 0>::kW;                                                \
        h = transposed ? PackedBox<T, 1>::kH : PackedBox<T, 0>::kH;                                                \
        break;
        TRC_PB(2)
        TRC_PB(3)
        TRC_PB(6)
        TRC_PB(7)
        TRC_PB(8)
#undef TRC_PB
        default: return false;
    }
    const cuuint64_t dims[4] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows), 1, 1};
    const cuuint64_t strides[3] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(row_bytes * rows),
                                   static_cast<cuuint64_t>(row_bytes * rows)};
    const cuuint32_t box[4] = {static_cast<cuuint32_t>(w), static_cast<cuuint32_t>(h), 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(blocks), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// True when the view's elements fill a gap-free byte range starting at d.data (a permutation of a
// contiguous tensor); `bytes` receives its size.
bool dense_extent(const trc_cuda_view& d, size_t& bytes) {
    int64_t count = 1, span = 4;
    for (int i = 0; i < 4; ++i) {
        if (d.ne[i] <= 0 || d.nb[i] <= 0) return false;
        count *= d.ne[i];
        span += (d.ne[i] - 1) * d.nb[i];
    }
    if (span != count * 4) return false;
    bytes = static_cast<size_t>(span);
    return true;
}

// Persistent launch: one CTA per SM (CG = 1) or one CTA pair per two SMs (CG = 2, a cluster of 2).
template <int QTYPE, int QTRANS, int CG, int PT = 0>
int launch_tc(const CUtensorMap& tmA, const CUtensorMap& tmB, const CUtensorMap& tmBt, const CUtensorMap& tmD,
              const CUtensorMap& tmW, const TcParams& p, cudaStream_t stream) {
    using G = typename KernelGeo<QTYPE, QTRANS, CG, PT>::type;
    static std::mutex mu;
    static uint64_t   configured = 0;  // bit per device ordinal
    static int        max_pairs[64] = {};
    auto kernel = tf32x3_gemm_kernel<QTYPE, QTRANS, CG, PT>;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e);
    const int sms = sm_count_current();
    if (sms <= 0) return TRC_CUDA_ECUDA;
    int pairs = sms / 2;
    {
        std::lock_guard<std::mutex> lock(mu);
        const uint64_t bit = dev < 64 ? (uint64_t(1) << dev) : 0;
        if (bit == 0 || (configured & bit) == 0) {
            e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, G::SMEM_BYTES);
            if (e != cudaSuccess) return cuda_fail(e);
            if constexpr (CG == 2) {
                // how many CTA pairs of this size fit on the device at once (a persistent grid larger
                // than that would only queue)
                cudaLaunchConfig_t cfg = {};
                cudaLaunchAttribute attr[1];
                attr[0].id = cudaLaunchAttributeClusterDimension;
                attr[0].val.clusterDim.x = 2;
                attr[0].val.clusterDim.y = 1;
                attr[0].val.clusterDim.z = 1;
                cfg.gridDim = dim3(2 * static_cast<unsigned>(sms / 2));
                cfg.blockDim = dim3(NUM_THREADS);
                cfg.dynamicSmemBytes = G::SMEM_BYTES;
                cfg.attrs = attr;
                cfg.numAttrs = 1;
                int n = 0;
                e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
                if (e != cudaSuccess) return cuda_fail(e);
                if (n <= 0) return TRC_CUDA_EUNSUPPORTED;
                if (dev < 64) max_pairs[dev] = n;
            }
            configured |= bit;
        }
        if (CG == 2 && dev < 64 && max_pairs[dev] > 0) pairs = std::min(pairs, max_pairs[dev]);
    }
    // a stream plan deals its chunks to exactly sk_slots slots (more than fit at once only queue; no
    // slot waits for another); the fused kernel that loads packed words itself has no stream phase
    if (p.sk_chunks > 0 && (p.sk_slots <= 0 || (QTYPE != 0 && PT == 0))) return TRC_CUDA_EINVAL;
    if constexpr (CG == 1) {
        const int64_t grid = p.sk_chunks > 0 ? p.sk_slots : std::min<int64_t>(p.total_units, sms);
        kernel<<<static_cast<unsigned>(grid), NUM_THREADS, G::SMEM_BYTES, stream>>>(tmA, tmB, tmBt, tmD, tmW, p);
    } else {
        const int64_t clusters = p.sk_chunks > 0 ? p.sk_slots : std::min<int64_t>(p.total_units, std::max(1, pairs));
        cudaLaunchConfig_t cfg = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters));
        cfg.blockDim = dim3(NUM_THREADS);
        cfg.dynamicSmemBytes = G::SMEM_BYTES;
        cfg.stream = stream;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, kernel, tmA, tmB, tmBt, tmD, tmW, p);
        if (e != cudaSuccess) return cuda_fail(e);
    }
    note_launch();
    return check_launch();
}

// D (+)= W over a dense byte range: the last step of a four-part split-K product.
__global__ void ws_add_kernel(float* __restrict__ d, const float* __restrict__ w, int64_t n) {
    const int64_t n4 = n / 4;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
        float4 a = reinterpret_cast<float4*>(d)[i];
        const float4 b = reinterpret_cast<const float4*>(w)[i];
        a.x = __fadd_rn(a.x, b.x);
        a.y = __fadd_rn(a.y, b.y);
        a.z = __fadd_rn(a.z, b.z);
        a.w = __fadd_rn(a.w, b.w);
        reinterpret_cast<float4*>(d)[i] = a;
    }
    for (int64_t i = 4 * n4 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        d[i] = __fadd_rn(d[i], w[i]);
}

// Split-K plan of one product. With four parts, parts 2 and 3 reduce into `ws`, a zeroed buffer of
// D's byte layout from the device's memory pool, through the tensor map tmW.
struct SplitPlan {
    void*       ws    = nullptr;
    size_t      bytes = 0;
    CUtensorMap tmW;
};

// The bytes of operand bands that at least two of the tiles [t0, t1) read over their whole
// reduction: an A band is a tile row's TILE_M rows of A, a B band a tile column's BN rows of B, per
// output plane. Tiles of the round-robin waves run side by side at the same point of K, so a band
// they share is read from HBM about once; the slots of a stream phase run at scattered points of
// K, so a shared band stays in L2 between its readers only if all such bands fit there at once.
template <int CG>
int64_t shared_band_bytes(const TcParams& p, int64_t t0, int64_t t1) {
    std::unordered_map<int64_t, int> a_uses, b_uses;
    const int64_t per_plane = static_cast<int64_t>(p.m_tiles) * p.n_tiles;
    for (int64_t t = t0; t < t1; ++t) {
        const TileCoord c = tile_coord<CG>(p, t);
        const int64_t plane = t / per_plane;
        ++a_uses[plane * p.m_tiles + c.m0 / Geo<CG>::TILE_M];
        ++b_uses[plane * p.n_tiles + c.n0 / BN];
    }
    const int64_t kbytes = static_cast<int64_t>(p.kv_blocks) * BK * 4;
    int64_t bytes = 0;
    for (const auto& u : a_uses)
        if (u.second >= 2) bytes += Geo<CG>::TILE_M * kbytes;
    for (const auto& u : b_uses)
        if (u.second >= 2) bytes += BN * kbytes;
    return bytes;
}

int64_t l2_bytes_current() {
    int dev = 0, l2 = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, dev) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return l2;
}

// Split K when it shortens the schedule. The persistent grid runs the units in waves of one unit
// per slot (CTA or CTA pair), and a tile count just above a multiple of the grid leaves most of the
// last wave idle: 448 tiles on 74 pairs take 7 waves for 6.05 waves of work. The plans:
//   - s parts (s in {1, 2, 4}): every tile's reduction is cut into s parts, s times the units at
//     1/s the length each;
//   - stream: all but the last (partial) wave of whole tiles run round-robin as unsplit, and the
//     remaining tiles' k-chunks are dealt to the slots in equal runs (UnitCursor), so every slot
//     ends within a chunk of the others. Only where the bands the stream tiles share fit in 80 %
//     of L2 (shared_band_bytes): measured on B200, the Linear forward's last 78 tiles (96 MB of
//     shared bands) ran 2-6 % faster as a stream phase; the Linear dX (352 MB) 4-6 % slower than
//     four parts, and the GQA dA at eight ne[3] planes (108 MB) 2 % slower than two.
// Every unit also pays a fixed cost (filling and draining the pipeline, storing or reduce-adding its
// tile, and with four parts the workspace pass). A plan is costed as the k-blocks its busiest slot
// runs plus kUnitCostKb per unit; the shortest one is taken when it is at least 1 % shorter than
// not splitting. kUnitCostKb = 12 k-blocks is fitted to timings on B200: 4 parts lengthen the GQA
// dB at one ne[3] plane (256 tiles of 128 k-blocks on 148 SMs) by a quarter although its waves
// shrink from 2 to 1.75, and shorten the Linear dX (128 tiles of 896 k-blocks on 74 pairs) by 7 %.
// The result never depends on the order in which parts land:
// - two parts reduce-add into a D zeroed here: 0 + a + b = 0 + b + a;
// - with four, parts 0 and 1 go to D and parts 2 and 3 to the workspace, and finish_split() adds
//   the two afterwards: (a + b) + (c + d);
// - a stream plan cuts a tile into at most four pieces and routes them the same way.
// No ACCUMULATE, since D + a + b would depend on the order. `allow_stream` is false for kernels whose
// loops do not walk UnitCursor (the fused kernel that loads packed words from global memory).
template <int CG>
int plan_split(const trc_cuda_view& d, bool accumulate, TcParams& p, SplitPlan& sp, cudaStream_t stream,
               bool allow_stream = true) {
    p.splits = 1;
    p.kv_per_split = p.kv_blocks;
    p.total_units = p.total_tiles;
    p.nck = 0;
    p.sk_tile0 = 0;
    p.sk_chunks = 0;
    const int sms = sm_count_current();
    const int64_t slots = CG == 2 ? sms / 2 : sms;
    size_t dense_bytes = 0;
    if (accumulate || !p.tma_store || slots <= 0 || p.kv_blocks < 2 * CHUNK_KB || !dense_extent(d, dense_bytes))
        return TRC_CUDA_OK;
    // each part's k-blocks (no part may be empty), and the schedule's length in k-blocks
    constexpr int kUnitCostKb = 12;
    auto per_part = [&](int s) { return ((p.kv_blocks + s - 1) / s + CHUNK_KB - 1) / CHUNK_KB * CHUNK_KB; };
    auto length = [&](int s) {
        return double((s * p.total_tiles + slots - 1) / slots) * double((s == 1 ? p.kv_blocks : per_part(s)) + kUnitCostKb);
    };
    const double unsplit = length(1);
    int parts = 1;
    double best = unsplit;
    if (length(2) <= 0.99 * unsplit) {
        parts = 2;
        best = length(2);
    }
    if (p.kv_blocks >= 4 * CHUNK_KB && 3 * per_part(4) < p.kv_blocks && length(4) <= 0.99 * unsplit &&
        length(4) < best) {
        parts = 4;
        best = length(4);
    }
    // stream plan: F round-robin waves of whole tiles, then the rest in equal chunk runs
    const int nck = (p.kv_blocks + CHUNK_KB - 1) / CHUNK_KB;
    const int64_t F = std::max<int64_t>(0, p.total_tiles / slots - 1);
    const int64_t sk_tiles = p.total_tiles - F * slots;
    const int64_t sk_chunks = sk_tiles * nck;
    const int64_t run_min = sk_chunks / slots, run_max = (sk_chunks + slots - 1) / slots;
    int max_pieces = 0;  // most pieces any stream tile is cut into
    if (allow_stream && run_min >= 1 && sk_chunks * (slots + 1) < (int64_t(1) << 31) &&
        shared_band_bytes<CG>(p, F * slots, p.total_tiles) * 5 <= l2_bytes_current() * 4) {
        max_pieces = static_cast<int>((nck - 1) / run_min + 2);
        const double len = double(F) * (p.kv_blocks + kUnitCostKb) + double(sk_tiles) * p.kv_blocks / slots +
                           double((run_max - 1) / nck + 2) * kUnitCostKb;
        if (max_pieces <= 4 && len <= 0.99 * unsplit && len < best) {
            parts = 0;  // stream
            best = len;
        }
    }
    const bool need_ws = parts == 4 || (parts == 0 && max_pieces > 2);
    if (need_ws) {
        retain_pool_once();
        if (cudaMallocAsync(&sp.ws, dense_bytes, stream) != cudaSuccess) {
            cudaGetLastError();
            sp.ws = nullptr;
        } else if (!encode_output(sp.ws, p.M, p.N, p.planes2, p.planes3, p.d_sm, p.d_sn, p.d_s2, p.d_s3, sp.tmW) ||
                   cudaMemsetAsync(sp.ws, 0, dense_bytes, stream) != cudaSuccess) {
            cudaGetLastError();
            cudaFreeAsync(sp.ws, stream);
            sp.ws = nullptr;
        } else {
            sp.bytes = dense_bytes;
        }
        if (sp.ws == nullptr) parts = length(2) <= 0.99 * unsplit ? 2 : 1;  // no workspace: at most two parts
    }
    if (parts == 1) return TRC_CUDA_OK;
    if (parts == 0) {
        p.total_units = F * slots;
        p.nck = nck;
        p.sk_tile0 = F * slots;
        p.sk_chunks = sk_chunks;
        p.sk_slots = slots;
    } else {
        p.splits = parts;
        p.kv_per_split = per_part(parts);
        p.total_units = p.total_tiles * parts;
    }
    const cudaError_t e = cudaMemsetAsync(d.data, 0, dense_bytes, stream);
    return e == cudaSuccess ? TRC_CUDA_OK : cuda_fail(e);
}

// After the GEMM of a four-part plan: D += workspace, then the workspace goes back to the pool.
// Runs (and frees) also when the GEMM failed, with `run_add` false.
int finish_split(SplitPlan& sp, void* d, bool run_add, cudaStream_t stream) {
    if (sp.ws == nullptr) return TRC_CUDA_OK;
    int st = TRC_CUDA_OK;
    if (run_add) {
        const int64_t n = static_cast<int64_t>(sp.bytes / sizeof(float));
        const int sms = std::max(1, sm_count_current());
        const int64_t grid = std::max<int64_t>(1, std::min<int64_t>((n / 4 + 255) / 256, int64_t(sms) * 8));
        ws_add_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(static_cast<float*>(d),
                                                                       static_cast<const float*>(sp.ws), n);
        note_launch();
        st = check_launch();
    }
    cudaFreeAsync(sp.ws, stream);
    sp.ws = nullptr;
    return st;
}

// CTA pairs when the tile grid has more than one 128-row tile (a single row tile would leave the
// second CTA of every pair without rows).
bool use_pair(int64_t M, bool allow_pair) { return allow_pair && M > BM; }

}  // namespace

bool mul_mat_tc_eligible(const trc_cuda_view& a_in, const trc_cuda_view& b_in, const trc_cuda_view& d) {
    const bool swap = d.nb[0] != 4 && d.nb[1] == 4;
    const trc_cuda_view& A = swap ? b_in : a_in;
    const trc_cuda_view& B = swap ? a_in : b_in;
    const int64_t M = A.ne[1], N = B.ne[1], K = a_in.ne[0];
    if (M <= 0 || N <= 0 || K <= 0 || M >= (1 << 30) || N >= (1 << 30) || K >= (1 << 30)) return false;
    if (b_in.ne[2] >= (1 << 30) || b_in.ne[3] >= (1 << 30)) return false;
    if (d.ne[2] <= 0 || d.ne[3] <= 0 || b_in.ne[2] % d.ne[2] != 0 || b_in.ne[3] % d.ne[3] != 0) return false;
    CUtensorMap tm;
    bool mn = false;
    return encode_operand(A, BM, mn, tm) && encode_operand(B, BN, mn, tm);
}

namespace {

// The fused kernel whose split warps load the packed words from global memory takes B's tails
// precomputed (one extra pass over B) when B is reused by at least two row tiles and the caller did
// not opt out: its split warps then only decode A. Measured on B200 (Q5_0 4096 x 14336, 2048
// tokens) for that kernel: forward +27 %, dX +16 %. The TMA-staged fused kernel (CTA pairs) and the
// F32 kernel split B in the loop instead: there the tails' extra TMA traffic and the pass over B
// cost more than the split work they save (TMA-staged fused: forward 228 vs 196-200 TFLOP/s, dX
// 235-249 vs 180-198; F32 4096^3: -14 %).
bool want_pretail(uint32_t flags, int m_tiles) { return (flags & TRC_CUDA_MM_NO_PRETAIL) == 0 && m_tiles >= 2; }

template <int CG>
int mul_mat_tc_impl(const trc_cuda_view& a_in, const trc_cuda_view& b_in, const trc_cuda_view& d, uint32_t flags,
                    cudaStream_t stream) {
    using G = Geo<CG>;
    const bool accumulate = (flags & TRC_CUDA_MM_ACCUMULATE) != 0;
    // Put D's unit-stride dimension on the TMEM lanes so that epilogue stores coalesce: if D is
    // contiguous along ggml's j (ne1) rather than i (ne0), compute D^T = b^T a with roles swapped.
    const bool swap = d.nb[0] != 4 && d.nb[1] == 4;
    const trc_cuda_view& A = swap ? b_in : a_in;  // MMA-A: rows = M
    const trc_cuda_view& B = swap ? a_in : b_in;  // MMA-B: rows = N
    const int64_t M = A.ne[1], N = B.ne[1], K = a_in.ne[0];
    // Output planes; when d has fewer planes than b, the source planes p with p % d.ne == q are
    // summed into output plane q (repeat_back fused into the K loop).
    const int64_t planes2 = d.ne[2], planes3 = d.ne[3];
    const int64_t red2 = b_in.ne[2] / planes2, red3 = b_in.ne[3] / planes3;

    CUtensorMap tmA, tmB;
    bool a_mn = false, b_mn = false, a5 = false, b5 = false;
    if (!encode_operand(A, BM, a_mn, tmA, &a5)) return TRC_CUDA_EUNSUPPORTED;
    if (!encode_operand(B, G::BN_CTA, b_mn, tmB, &b5)) return TRC_CUDA_EUNSUPPORTED;

    TcParams p;
    std::memset(&p, 0, sizeof(p));
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.m_tiles  = static_cast<int>((M + G::TILE_M - 1) / G::TILE_M);
    p.n_tiles  = static_cast<int>((N + BN - 1) / BN);
    p.k_blocks = static_cast<int>((K + BK - 1) / BK);
    if (static_cast<int64_t>(p.m_tiles) * p.n_tiles * GROUP_M >= (int64_t(1) << 31)) return TRC_CUDA_EUNSUPPORTED;
    p.planes2 = static_cast<int>(planes2);
    p.planes3 = static_cast<int>(planes3);
    p.red2 = static_cast<int>(red2);
    p.red3 = static_cast<int>(red3);
    p.kv_blocks = p.k_blocks * p.red2 * p.red3;
    p.a_ne2 = static_cast<int>(A.ne[2]);
    p.a_ne3 = static_cast<int>(A.ne[3]);
    p.b_ne2 = static_cast<int>(B.ne[2]);
    p.b_ne3 = static_cast<int>(B.ne[3]);
    p.a_mn = a_mn ? 1 : 0;
    p.b_mn = b_mn ? 1 : 0;
    p.a_tma5 = a5 ? 1 : 0;
    p.b_tma5 = b5 ? 1 : 0;
    p.accumulate = accumulate ? 1 : 0;
    p.total_tiles = static_cast<int64_t>(p.m_tiles) * p.n_tiles * planes2 * planes3;
    p.d    = static_cast<char*>(d.data);
    p.d_sm = swap ? d.nb[1] : d.nb[0];
    p.d_sn = swap ? d.nb[0] : d.nb[1];
    p.d_s2 = d.nb[2];
    p.d_s3 = d.nb[3];

    CUtensorMap tmD;
    std::memset(&tmD, 0, sizeof(tmD));
    p.tma_store = encode_output(d.data, M, N, planes2, planes3, p.d_sm, p.d_sn, p.d_s2, p.d_s3, tmD) ? 1 : 0;

    SplitPlan sp;
    int st = plan_split<CG>(d, accumulate, p, sp, stream);
    if (st == TRC_CUDA_OK) st = launch_tc<0, 0, CG>(tmA, tmB, tmB, tmD, sp.ws ? sp.tmW : tmD, p, stream);
    const int fin = finish_split(sp, d.data, st == TRC_CUDA_OK, stream);
    return st != TRC_CUDA_OK ? st : fin;
}

template <int CG>
int mul_mat_q_tc_impl(int type, const void* w_blocks, int64_t w_ne0, int64_t w_ne1, int a_transposed,
                      const trc_cuda_view& b, const trc_cuda_view& d, uint32_t flags, cudaStream_t stream) {
    using G = Geo<CG>;
    const bool accumulate = (flags & TRC_CUDA_MM_ACCUMULATE) != 0;
    const int64_t M = a_transposed ? w_ne0 : w_ne1;
    const int64_t K = a_transposed ? w_ne1 : w_ne0;
    const int64_t N = b.ne[1];
    CUtensorMap tmA, tmB;
    std::memset(&tmA, 0, sizeof(tmA));
    bool b_mn = false, b5 = false;
    if (!encode_operand(b, G::BN_CTA, b_mn, tmB, &b5)) return TRC_CUDA_EUNSUPPORTED;
    const size_t bb = trc_cuda_block_bytes(type);

    TcParams p;
    std::memset(&p, 0, sizeof(p));
    p.M = static_cast<int>(M);
    p.N = static_cast<int>(N);
    p.K = static_cast<int>(K);
    p.m_tiles  = static_cast<int>((M + G::TILE_M - 1) / G::TILE_M);
    p.n_tiles  = static_cast<int>((N + BN - 1) / BN);
    p.k_blocks = static_cast<int>((K + BK - 1) / BK);
    if (static_cast<int64_t>(p.m_tiles) * p.n_tiles * GROUP_M >= (int64_t(1) << 31)) return TRC_CUDA_EUNSUPPORTED;
    p.planes2 = static_cast<int>(b.ne[2]);
    p.planes3 = static_cast<int>(b.ne[3]);
    p.red2 = 1;
    p.red3 = 1;
    p.kv_blocks = p.k_blocks;
    p.a_ne2 = 1;
    p.a_ne3 = 1;
    p.b_ne2 = static_cast<int>(b.ne[2]);
    p.b_ne3 = static_cast<int>(b.ne[3]);
    p.a_mn = a_transposed ? 1 : 0;
    p.b_mn = b_mn ? 1 : 0;
    p.b_tma5 = b5 ? 1 : 0;
    p.accumulate = accumulate ? 1 : 0;
    p.total_tiles = static_cast<int64_t>(p.m_tiles) * p.n_tiles * b.ne[2] * b.ne[3];
    p.d    = static_cast<char*>(d.data);
    p.d_sm = d.nb[0];
    p.d_sn = d.nb[1];
    p.d_s2 = d.nb[2];
    p.d_s3 = d.nb[3];
    p.qa = static_cast<const uint8_t*>(w_blocks);
    p.q_blocks_per_row = static_cast<int>(w_ne0 / 32);
    p.q_row_bytes = static_cast<int64_t>(w_ne0 / 32) * static_cast<int64_t>(bb);
    p.q_rows = static_cast<int>(w_ne1);
    CUtensorMap tmD;
    std::memset(&tmD, 0, sizeof(tmD));
    p.tma_store = encode_output(d.data, M, N, b.ne[2], b.ne[3], p.d_sm, p.d_sn, p.d_s2, p.d_s3, tmD) ? 1 : 0;
    // CTA pairs stage the packed bytes by TMA where the packed rows allow a tensor map (16-byte
    // aligned base and row pitch); otherwise the split warps load them from global memory.
    const bool ptma = CG == 2 && encode_packed(w_blocks, p.q_row_bytes, w_ne1, type, a_transposed != 0, tmA);
    SplitPlan sp;
    const int sst = plan_split<CG>(d, accumulate, p, sp, stream, /*allow_stream=*/ptma);
    if (sst != TRC_CUDA_OK) {
        finish_split(sp, d.data, false, stream);
        return sst;
    }
    const CUtensorMap& tmW = sp.ws ? sp.tmW : tmD;
    Pretail pt;
    if (!ptma && want_pretail(flags, p.m_tiles) && make_pretail(b, G::BN_CTA, b_mn, b5, stream, pt)) p.b_pretail = 1;
    const CUtensorMap& tmBt = p.b_pretail ? pt.map : tmB;
    int st = TRC_CUDA_EUNSUPPORTED;
#define TRC_Q_CASE(T)                                                                                 \
    case T:                                                                                           \
        if constexpr (CG == 2) {                                                                      \
            if (ptma) {                                                                               \
                st = a_transposed ? launch_tc<T, 1, 2, 1>(tmA, tmB, tmBt, tmD, tmW, p, stream)        \
                                  : launch_tc<T, 0, 2, 1>(tmA, tmB, tmBt, tmD, tmW, p, stream);       \
                break;                                                                                \
            }                                                                                         \
        }                                                                                             \
        st = a_transposed ? launch_tc<T, 1, CG>(tmA, tmB, tmBt, tmD, tmW, p, stream)                  \
                          : launch_tc<T, 0, CG>(tmA, tmB, tmBt, tmD, tmW, p, stream);                 \
        break;
    switch (type) {
        TRC_Q_CASE(2)
        TRC_Q_CASE(3)
        TRC_Q_CASE(6)
        TRC_Q_CASE(7)
        TRC_Q_CASE(8)
        default: break;
    }
#undef TRC_Q_CASE
    if (pt.buf != nullptr) cudaFreeAsync(pt.buf, stream);
    const int fin = finish_split(sp, d.data, st == TRC_CUDA_OK, stream);
    return st != TRC_CUDA_OK ? st : fin;
}

}  // namespace

int mul_mat_tc(const trc_cuda_view& a_in, const trc_cuda_view& b_in, const trc_cuda_view& d, uint32_t flags,
               cudaStream_t stream) {
    const bool allow_pair = (flags & TRC_CUDA_MM_ONE_CTA) == 0;
    const bool swap = d.nb[0] != 4 && d.nb[1] == 4;
    const trc_cuda_view& A = swap ? b_in : a_in;
    const trc_cuda_view& B = swap ? a_in : b_in;
    const int64_t M = A.ne[1], N = B.ne[1], K = a_in.ne[0];
    const int64_t planes2 = d.ne[2], planes3 = d.ne[3];
    if (planes2 <= 0 || planes3 <= 0 || b_in.ne[2] % planes2 != 0 || b_in.ne[3] % planes3 != 0) return TRC_CUDA_EINVAL;
    const int64_t red2 = b_in.ne[2] / planes2, red3 = b_in.ne[3] / planes3;
    if (M <= 0 || N <= 0 || K <= 0 || M >= (1 << 30) || N >= (1 << 30) || K >= (1 << 30)) return TRC_CUDA_EUNSUPPORTED;
    if (planes2 >= (1 << 30) || planes3 >= (1 << 30)) return TRC_CUDA_EUNSUPPORTED;
    if ((K + BK - 1) / BK * red2 * red3 >= (int64_t(1) << 30)) return TRC_CUDA_EUNSUPPORTED;
    return use_pair(M, allow_pair) ? mul_mat_tc_impl<2>(a_in, b_in, d, flags, stream)
                                   : mul_mat_tc_impl<1>(a_in, b_in, d, flags, stream);
}

bool mul_mat_q_tma_staged(int type, const void* w_blocks, int64_t w_ne0, int64_t w_ne1, int a_transposed, uint32_t flags) {
    const int64_t M = a_transposed ? w_ne0 : w_ne1;
    const size_t bb = trc_cuda_block_bytes(type);
    if (bb == 0 || w_ne0 % 32 != 0 || !use_pair(M, (flags & TRC_CUDA_MM_ONE_CTA) == 0)) return false;
    const int64_t row_bytes = (w_ne0 / 32) * static_cast<int64_t>(bb);
    return (reinterpret_cast<uint64_t>(w_blocks) & 15u) == 0 && row_bytes % 16 == 0;
}

int mul_mat_q_tc(int type, const void* w_blocks, int64_t w_ne0, int64_t w_ne1, int a_transposed,
                 const trc_cuda_view& b, const trc_cuda_view& d, uint32_t flags, cudaStream_t stream) {
    const bool allow_pair = (flags & TRC_CUDA_MM_ONE_CTA) == 0;
    const int64_t M = a_transposed ? w_ne0 : w_ne1;
    const int64_t K = a_transposed ? w_ne1 : w_ne0;
    const int64_t N = b.ne[1];
    if (M >= (1 << 30) || N >= (1 << 30) || K >= (1 << 30) || N <= 0) return TRC_CUDA_EUNSUPPORTED;
    if ((reinterpret_cast<uint64_t>(w_blocks) & 1u) != 0) return TRC_CUDA_EINVAL;
    return use_pair(M, allow_pair)
               ? mul_mat_q_tc_impl<2>(type, w_blocks, w_ne0, w_ne1, a_transposed, b, d, flags, stream)
               : mul_mat_q_tc_impl<1>(type, w_blocks, w_ne0, w_ne1, a_transposed, b, d, flags, stream);
}

}  // namespace trc
