// zs_lmhead.cuh -- the lm_head of Model::eval (src/model.cpp:401-403) on the
// tensor cores, with the sampler's shortlist selection as the GEMM epilogue.
//
//   xn     = rmsnorm(hidden, output_norm)          zs_lm_rmsnorm_kernel, bf16 out
//   logits = xn . W^T   (W = output.weight [V][E])  zs_lmhead_kernel
//
// zs_lmhead_kernel is a persistent tcgen05 GEMM: D[128 rows][128 vocab] tiles per
// CTA, or D[256][256] per CTA pair (cta_group::2, LmGeom), accumulate in tensor
// memory (all 512 columns: four or two accumulators, so the MMAs run ahead of the
// epilogue, whose time per tile varies); operands arrive by TMA (2-D tiles, 128-byte
// swizzle, no multicast) through a shared-memory ring of 3 to 5 stages (deeper when
// the batch leaves candidate buffers unused).  Work units are (row tile, vocabulary
// slice); a CTA walks its units' tiles in column order.  Warp 0 issues the copies,
// one thread of warp 1 issues the MMAs, warps 2-9 are the epilogue: two warps per
// TMEM lane quarter, 16 rows (lanes) each, a row's 32-column chunk split over a lane
// pair (16x64b TMEM loads), so each scheduler has two epilogue warps to switch
// between.  The epilogue keeps, per row, a buffer of candidate keys (value desc, id
// asc is the sampler's key order) above a threshold: about the keff-th best key of
// the row's unit so far, as of the buffer's last compaction.  Columns come in id
// order, so a column passes exactly when its value order beats the threshold's.
// When a row's passing columns would overflow its buffer, the warp cuts that row
// back to (about) its keff best keys together (warp_topk_keep), which raises the
// threshold.  A row's slices also share a lower bound through global memory
// (lm_shared_bound / lm_adopt).  At the end of a unit each row writes its exact top
// keff as one partial block, (row, slice), in the layout zs_merge_kernel and
// zs_warp_merge_kernel read, so the merge, f64 softmax, nucleus and draw are the
// sampler's own.  Optionally the epilogue also writes the f32 logits.
//
// Every wait is bounded (kWaitLimitNs); a wait that runs out sets the handle's
// status to ZS_ERR_DEVICE_TIMEOUT and the kernel unwinds: the copy issuer waits
// for its copies in flight, the MMA issuer for its MMAs, then TMEM is freed.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "zs_device.cuh"
#include "zs_kernels.cuh"

namespace zs {

constexpr int kLmM = 128;       // batch rows per tile: the TMEM lanes
constexpr int kLmN = 128;       // vocabulary columns per tile
constexpr int kLmBK = 64;       // K per stage: one 128-byte swizzle row of bf16
constexpr int kLmStages = 3;      // ring stages when all 128 rows hold candidates
constexpr int kLmStagesMax = 5;   // with only 32 rows' buffers the ring takes the rest
constexpr int kLmCap = 120;     // candidate keys buffered per row
constexpr int kLmKeffMax = kLmCap - 32;  // a compaction leaves room for a whole chunk
constexpr int kLmRowStride = kLmCap + 1; // odd, so rows spread over the banks
constexpr int kLmThreads = 320; // warp 0 copies, warp 1 MMAs, warps 2-9 epilogue
constexpr int kLmEpiWarps = 8;  // two per TMEM lane quarter, 16 rows (lanes) each
// Lanes of an epilogue warp that own a row (the other lane of each pair, lane ^ 2,
// holds the row's other 16 columns of a chunk): lanes whose bit 1 is clear.
constexpr unsigned kLmOwnerLanes = 0x33333333u;
constexpr int kLmAccs = 4;  // accumulators in tensor memory (all 512 columns)
constexpr int kLmTmemCols = kLmAccs * kLmN;
constexpr uint32_t kLmTileABytes = kLmM * kLmBK * 2;
constexpr uint32_t kLmTileBBytes = kLmN * kLmBK * 2;
constexpr int64_t kLmPartStride = kPartialHeaderBytes + 8 * kLmKeffMax;
static_assert(kLmPartStride % 16 == 0, "block headers are read as uint4");
constexpr uint32_t kLmStageBytes = kLmTileABytes + kLmTileBBytes;
constexpr uint32_t kLmRowBytes = kLmRowStride * 8;  // one row's candidate buffer
// ns stages of A tiles, ns of B tiles, then the candidate buffers of the rows in use
constexpr uint32_t kLmRingBytes = kLmStages * kLmStageBytes + kLmM * kLmRowBytes;
static_assert(kLmStagesMax * kLmStageBytes + 32 * kLmRowBytes <= kLmRingBytes,
              "the deepest ring leaves room for one warp's buffers");

struct LmSmem {  // placed at a 1024-byte boundary: the swizzled tiles need it
    uint8_t ring[kLmRingBytes];  // tiles (1024-byte aligned), then per row: keys, unordered
    uint64_t full[kLmStagesMax];
    uint64_t empty[kLmStagesMax];
    uint64_t acc_full[kLmAccs];
    uint64_t acc_empty[kLmAccs];
    uint64_t drain;
    uint32_t tmem_base;
    int abort;
};
constexpr size_t kLmSmemBytes = sizeof(LmSmem) + 1024;

struct LmArgs {
    int32_t B, E, V, V_total;
    int32_t mt, nt, S, n_units;  // row tiles, column tiles, slices per row, units
    int32_t select;              // 1: partial blocks per (row, slice); 0: logits only
    Params shared;
    const Params* row_params;
    uint8_t* part;               // [B][S] blocks of kLmPartStride bytes
    float* out_logits;           // optional [B][logits_ld]
    int64_t logits_ld;
    int32_t tma_out;             // logits only: staged in shared memory, stored by TMA
    int32_t ns;                  // ring stages: kLmStages, or more when few rows hold keys
    int32_t prefetch;            // weight boxes each CTA prefetches into L2 while rmsnorm runs
    uint32_t* tau;               // optional [B] value orders shared by a row's slices
    int* status;
    int32_t pair;                // 2: zs_lmhead_kernel<2> (CTA pairs), else <1>; host only
};

// ---- PTX wrappers: TMA tiles and the 5th-generation tensor cores ----
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// Shared -> global tile store (no multicast); completion tracked by bulk groups.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int32_t x,
                                             int32_t y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(smem_addr(src))
                 : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most one committed store is still reading shared memory.
__device__ __forceinline__ void bulk_wait_read_1() {
    asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
// Waits until every committed store has completed.
__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// One box of a tensor into L2 only (no shared memory, no barrier).
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int32_t x, int32_t y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y)
                 : "memory");
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tc_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrives once on `bar` when every tcgen05 operation this thread issued before
// has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}
// D[tmem] (+)= A[smem] . B[smem]^T, bf16 inputs, f32 accumulators.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// 32 consecutive f32 columns of this thread's TMEM lane.  tc_ld_wait names the
// destination registers as read and written, so no use of them can be scheduled
// before the data has arrived.
__device__ __forceinline__ void tc_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tc_ld_wait(uint32_t (&r)[32]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

// 32 columns of 16 TMEM lanes (shape 16x64b, 16 repeats): lane t of the warp gets
// lane 8 (t & 1) + (t >> 2) of the 16, columns ((t >> 1) & 1) + 2 j, j = 0..15.
__device__ __forceinline__ void tc_ld16_issue(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.16x64b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void tc_ld16_wait(uint32_t (&r)[16]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}
__device__ __forceinline__ int lm_dp(int lane) { return 8 * (lane & 1) + (lane >> 2); }
__device__ __forceinline__ int lm_par(int lane) { return (lane >> 1) & 1; }

// Shared-memory matrix descriptor of a K-major tile written by TMA with 128-byte
// swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte offset),
// leading byte offset unused for this layout (1), descriptor version 1, layout
// type 2 (128-byte swizzle).  The tile starts at a 1024-byte boundary, so the
// base offset is 0; a K step of 16 elements (32 bytes) adds 2 to the start field.
__device__ __forceinline__ uint64_t sw128_desc(const void* tile) {
    const uint32_t a = smem_addr(tile);
    return (uint64_t)((a & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor, kind::f16: D f32 (bits 4-5 = 1), A and B bf16 (bits 7-9,
// 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t lm_idesc(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Tile geometry of zs_lmhead_kernel<P>.  P = 1: one CTA computes 128 rows x 128
// vocabulary columns per tile.  P = 2: a CTA pair (a cluster of two) computes 256 x
// 256 with tcgen05.mma.cta_group::2: each CTA stages its own 128 rows of xn and its
// own 128 of the tile's 256 weight rows, and holds its 128 rows x all 256 columns in
// its tensor memory.  Per MMA an SM then reads 8 KB of operands from shared memory
// for 128 x 256 x 16 products, where the one-CTA tile reads 8 KB for 128 x 128 x 16:
// half the shared-memory and L2 traffic per product.
template <int P>
struct LmGeom {
    static_assert(P == 1 || P == 2, "one CTA or a CTA pair");
    static constexpr int kRows = kLmM * P;        // batch rows per tile (the pair's)
    static constexpr int kCols = kLmN * P;        // vocabulary columns per tile
    static constexpr int kAccs = 512 / kCols;     // accumulators: all 512 TMEM columns
    static constexpr uint32_t kIdesc = lm_idesc(kRows, kCols);
    // epilogue arrivals that free an accumulator: one lane per epilogue warp (P = 1),
    // of both CTAs on the leader's barrier (P = 2)
    static constexpr uint32_t kAccEmptyCount = P * kLmEpiWarps;
};
static_assert(LmGeom<1>::kAccs <= kLmAccs && LmGeom<2>::kAccs <= kLmAccs, "barrier arrays");

// ---- CTA-pair (cluster of two) primitives ----
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The shared::cluster address of `local` (this CTA's shared memory) in CTA `rank`.
__device__ __forceinline__ uint32_t smem_in_cta(const void* local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(local)), "r"(rank));
    return r;
}
// Every thread of both CTAs: orders this CTA's earlier shared-memory writes (barrier
// initialisation included) before the other CTA's later accesses.
__device__ __forceinline__ void cluster_sync_all() {
    __syncwarp();  // the .aligned forms want the whole warp at the same instruction
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}
// Arrives on a barrier of either CTA of the pair (default release at CTA scope: the
// accumulator it frees is ordered by tcgen05.wait::ld and the before_thread_sync
// fence, not by memory ordering).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
// A 2-D tile into this CTA's shared memory whose bytes count on the barrier of the
// pair's leader (bar_cluster: a shared::cluster address), no multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int32_t x,
                                                 int32_t y, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}
__device__ __forceinline__ void tc_alloc_pair(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
// D (both CTAs' tensor memory) (+)= A (both CTAs' rows) . B (both CTAs' halves)^T;
// the descriptors and the TMEM address name the leader's copies, the peer's are at
// the same offsets.
__device__ __forceinline__ void tc_mma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives once on `bar` (same offset) in every CTA of `mask` when this thread's
// earlier tcgen05 operations of the pair have completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 "
        "[%0], %1;" ::"r"(smem_addr(bar)),
        "h"(mask)
        : "memory");
}

// Bounded wait that also gives up when another role has aborted.
__device__ __forceinline__ bool lm_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 15u) == 0u) {
            if (*abort) return false;
            if (global_ns() - t0 > kWaitLimitNs) {
                *abort = 1;
                return false;
            }
        }
    }
}

// Units [u_begin, u_end) of this CTA (of this CTA pair for P = 2, whose CTAs are
// consecutive blocks): a contiguous share, so consecutive units of one row tile
// (adjacent slices) meet in one CTA and share its candidate buffers.
template <int P>
__device__ __forceinline__ void lm_range(const LmArgs& a, int& u_begin, int& u_end) {
    const int64_t c = blockIdx.x / P, n = gridDim.x / P;
    u_begin = (int)((c * a.n_units) / n);
    u_end = (int)(((c + 1) * a.n_units) / n);
}

__device__ __forceinline__ void lm_unit(const LmArgs& a, int u, int& m, int& s, int& t0, int& t1) {
    m = u / a.S;
    s = u - m * a.S;
    t0 = (int)(((int64_t)s * a.nt) / a.S);
    t1 = (int)(((int64_t)(s + 1) * a.nt) / a.S);
}

// ---- rmsnorm (src/model.cpp:31-38), rounded to bf16 ----
// One warp per row: the lanes stage the row in shared memory (coalesced), lane 0
// sums the squares in order in double like the reference (each term is a product
// of two floats, exact in double; 1/sqrt and the division are correctly rounded, so
// xn equals the reference's float before the bf16 rounding), then every lane writes
// its share.  Dynamic shared memory: E floats per warp.
__global__ void zs_lm_rmsnorm_kernel(const float* hidden, int64_t hld, const float* norm_w,
                                     float eps, int32_t B, int32_t E, __nv_bfloat16* xn,
                                     uint32_t* tau) {
    extern __shared__ float lm_stage[];
    grid_dep_trigger();  // zs_lmhead_kernel may start its weight prefetch now
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    float* xs = lm_stage + (int64_t)warp * E;
    for (int r = blockIdx.x * nw + warp; r < B; r += gridDim.x * nw) {
        const float* x = hidden + (int64_t)r * hld;
        for (int i = lane; i < E; i += 32) xs[i] = x[i];
        __syncwarp();
        double scale = 0.0;
        if (lane == 0) {
            double sum = 0.0;
#pragma unroll 8
            for (int i = 0; i < E; ++i) {
                const double v = (double)xs[i];
                sum = __dadd_rn(sum, __dmul_rn(v, v));
            }
            scale = 1.0 / sqrt(sum / (double)E + (double)eps);
        }
        scale = __shfl_sync(kFull, scale, 0);
        if (tau && lane == 0) tau[r] = 0u;  // no shared bound yet for this row
        __nv_bfloat16* o = xn + (int64_t)r * E;
        for (int i = lane; i < E; i += 32) {
            const float v = __double2float_rn(__dmul_rn(__dmul_rn((double)xs[i], scale), (double)norm_w[i]));
            o[i] = __float2bfloat16_rn(v);
        }
        __syncwarp();
    }
}

// ---- the lm_head in f32, in the reference's own summation order (small batches) ----
// zs_lm_exact_kernel computes the logits as the reference does by default
// (src/model.cpp:401-403 with src/kernels.cpp:52-78 dot_f32_avx2): xn in f32
// (rmsnorm as above, without the bf16 rounding), and per logit 32 f32 accumulators,
// accumulator l taking w[i] * xn[i] for i = l, l + 32, ... by fused multiply-add in
// order (lane l of a warp holds accumulator l), then the AVX2 code's reduction tree
// (lanes e, 8 + e, 16 + e, 24 + e as (a0 + a1) + (a2 + a3), then + 4, + 2, + 1 apart)
// by shuffles, the terms past the last multiple of 32 in double, one float rounding:
// bit-exact with the reference's logits.  No tensor cores: up to kExMaxRows rows the
// lm_head is a stream of the weights, which the copy warp moves through a ring of
// bulk copies (and, while the rows' f64 sums of squares run, prefetches into L2).
constexpr int kExMaxRows = 8;
constexpr int kExMaxE = 2048;
constexpr int kExMaxElems = 8192;  // rows x hidden size: xn in shared memory, 32 KB
constexpr int kExWarps = 8;                      // consumer warps
constexpr int kExThreads = 32 * (kExWarps + 1);  // + the copy warp
constexpr int kExStages = 3;
constexpr uint32_t kExStageBytes = 58u << 10;  // 32 padded rows of 896
constexpr int kExMaxStageRows = 64;
constexpr int kExRowsPerWarp = 4;  // a warp's rows at once: 8 lanes per row
// Weight rows sit in the ring padded by 64 bytes: with 8 lanes per row each reading 8
// bytes, the 4 rows of a warp then fall on two bank halves (two wavefronts).
__host__ __device__ constexpr uint32_t ex_row_stride(int E) { return (uint32_t)E * 2u + 64u; }

struct ExArgs {
    const float* hidden;
    int64_t hld;
    const float* norm_w;
    float eps;
    int32_t B, E, V;
    const uint16_t* w;  // bf16 bits [V][E]
    float* out;         // [B][lld]
    int64_t lld;
    int32_t rows_per_stage;
    int64_t prefetch_bytes;  // per CTA, after the ring's first stages
    int* status;
};

// ring, xn [B][E], the B scales, 2 x kExStages barriers, the abort flag
__host__ __device__ constexpr size_t ex_smem_bytes(int B, int E) {
    return (size_t)kExStages * kExStageBytes + (size_t)B * E * 4 + (size_t)kExMaxRows * 8 +
           (size_t)2 * kExStages * 8 + 16;
}

__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__global__ void __launch_bounds__(kExThreads, 1) zs_lm_exact_kernel(const ExArgs a) {
    extern __shared__ __align__(128) uint8_t ex_raw[];
    uint8_t* ring = ex_raw;
    float* xn = reinterpret_cast<float*>(ring + (size_t)kExStages * kExStageBytes);
    double* scale_s = reinterpret_cast<double*>(xn + (size_t)a.B * a.E);  // E % 8 == 0
    uint64_t* full = reinterpret_cast<uint64_t*>(scale_s + kExMaxRows);
    uint64_t* empty = full + kExStages;
    volatile int* abort = reinterpret_cast<volatile int*>(empty + kExStages);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kExStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kExWarps);
        }
        *abort = 0;
        mbar_fence_init();
    }
    __syncthreads();
    const int64_t v_lo = (int64_t)blockIdx.x * a.V / gridDim.x;
    const int64_t v_hi = (int64_t)(blockIdx.x + 1) * a.V / gridDim.x;
    const int R = a.rows_per_stage;
    const int nst = (int)((v_hi - v_lo + R - 1) / R);
    if (warp == 0) {
        // ---- copy issuer ----
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            bool ok = true;
            int issued = 0;
            for (int st = 0; st < nst; ++st) {
                const int slot = st % kExStages;
                if (!lm_wait(&empty[slot], (uint32_t)((st / kExStages) & 1) ^ 1u, abort)) {
                    ok = false;
                    break;
                }
                const int64_t v0 = v_lo + (int64_t)st * R;
                const int nrow = (int)min((int64_t)R, v_hi - v0);
                const uint32_t rb = (uint32_t)a.E * 2u;
                mbar_arrive_expect_tx(&full[slot], (uint32_t)nrow * rb);
                for (int r = 0; r < nrow; ++r)  // one copy per row, into its padded slot
                    bulk_load(ring + (size_t)slot * kExStageBytes + (size_t)r * ex_row_stride(a.E),
                              a.w + (v0 + r) * a.E, rb, &full[slot], pol);
                ++issued;
                if (st == kExStages - 1 || (st == nst - 1 && nst < kExStages)) {
                    // the rest of this CTA's weights (up to prefetch_bytes) into L2
                    // while the consumers' row sums run
                    const uint8_t* p0 = reinterpret_cast<const uint8_t*>(a.w + (v0 + R) * a.E);
                    const uint8_t* pend = reinterpret_cast<const uint8_t*>(a.w + v_hi * a.E);
                    int64_t left = min((int64_t)a.prefetch_bytes, pend - p0);
                    for (const uint8_t* p = p0; left > 0; p += 65536, left -= 65536)
                        prefetch_l2_bulk(p, (uint32_t)min((int64_t)65536, left));
                }
            }
            if (!ok) set_status(a.status, kStatusTimeout);
            for (int i = issued - kExStages; i < issued; ++i)  // copies landed before exit
                if (i >= 0) mbar_wait_bounded(&full[i % kExStages], (uint32_t)((i / kExStages) & 1));
        }
        __syncwarp();
        return;
    }
    // ---- consumers: rmsnorm (src/model.cpp:31-38) to f32, then the dot products ----
    const int cw = warp - 1;
    // the rows, staged in xn's place (coalesced), then row lane's sum of squares in
    // order in double, then xn over them in place
    for (int idx = threadIdx.x - 32; idx < a.B * a.E; idx += kExWarps * 32) {
        const int b = idx / a.E, i = idx - b * a.E;
        xn[idx] = a.hidden[(int64_t)b * a.hld + i];
    }
    consumer_sync<kExWarps * 32>();
    if (cw == 0 && lane < a.B) {
        const float* x = xn + lane * a.E;
        double sum = 0.0;
#pragma unroll 8
        for (int i = 0; i < a.E; ++i) {
            const double v = (double)x[i];
            sum = __fma_rn(v, v, sum);  // v * v is exact in double
        }
        scale_s[lane] = 1.0 / sqrt(sum / (double)a.E + (double)a.eps);
    }
    consumer_sync<kExWarps * 32>();
    for (int idx = threadIdx.x - 32; idx < a.B * a.E; idx += kExWarps * 32) {
        const int b = idx / a.E, i = idx - b * a.E;
        xn[idx] = __double2float_rn(__dmul_rn(__dmul_rn((double)xn[idx], scale_s[b]),
                                              (double)a.norm_w[i]));
    }
    consumer_sync<kExWarps * 32>();
    const int n32 = a.E & ~31;
    bool ok = true;
    for (int st = 0; st < nst && ok; ++st) {
        const int slot = st % kExStages;
        const bool got = lm_wait(&full[slot], (uint32_t)((st / kExStages) & 1), abort);
        if (!__all_sync(kFull, got)) {
            ok = false;
            break;
        }
        const int64_t v0 = v_lo + (int64_t)st * R;
        const int rows = (int)min((int64_t)R, v_hi - v0);
        const uint16_t* wt = reinterpret_cast<const uint16_t*>(ring + (size_t)slot * kExStageBytes);
        // A warp takes kExRowsPerWarp rows at once, 8 lanes per row: lane p of a row
        // holds accumulators 4p .. 4p + 3 (the reference's accumulator l takes the
        // columns l, l + 32, ...), so its four chains are independent and each
        // 32-column block is one 8-byte load of weights per lane.
        const int rq = lane >> 3, p = lane & 7;
        const uint32_t rs = ex_row_stride(a.E);
        for (int r0 = cw * kExRowsPerWarp; r0 < rows; r0 += kExWarps * kExRowsPerWarp) {
            const int r = r0 + rq;
            const bool live = r < rows;
            const uint8_t* wrow = ring + (size_t)slot * kExStageBytes + (size_t)(live ? r : 0) * rs;
            float acc[kExMaxRows][4];
#pragma unroll
            for (int b = 0; b < kExMaxRows; ++b)
#pragma unroll
                for (int c = 0; c < 4; ++c) acc[b][c] = 0.0f;
#pragma unroll 4
            for (int blk = 0; blk < n32; blk += 32) {
                const uint2 wq = *reinterpret_cast<const uint2*>(wrow + (size_t)(blk + 4 * p) * 2);
                const float w0 = __uint_as_float(wq.x << 16), w1 = __uint_as_float(wq.x & 0xffff0000u);
                const float w2 = __uint_as_float(wq.y << 16), w3 = __uint_as_float(wq.y & 0xffff0000u);
#pragma unroll
                for (int b = 0; b < kExMaxRows; ++b) {
                    if (b < a.B) {
                        const float4 x = *reinterpret_cast<const float4*>(xn + b * a.E + blk + 4 * p);
                        acc[b][0] = __fmaf_rn(w0, x.x, acc[b][0]);
                        acc[b][1] = __fmaf_rn(w1, x.y, acc[b][1]);
                        acc[b][2] = __fmaf_rn(w2, x.z, acc[b][2]);
                        acc[b][3] = __fmaf_rn(w3, x.w, acc[b][3]);
                    }
                }
            }
#pragma unroll
            for (int b = 0; b < kExMaxRows; ++b) {
                if (b >= a.B) break;
                // The AVX2 reduction.  Accumulator l = 8 k + e is vector k's lane e;
                // lane p holds l = 4p .. 4p + 3, so vector k sits on lanes 2k, 2k + 1.
                // (a0 + a1) + (a2 + a3) per vector lane e: lanes 0, 1 and 4, 5 add the
                // lanes two above them, then lanes 0, 1 add lanes 4, 5: lane 0 holds
                // s[0..3], lane 1 s[4..7]; then s[m] + s[m + 4], [0] + [2], [1] + [3],
                // and those two.
                float v[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    v[c] = __fadd_rn(acc[b][c], __shfl_down_sync(kFull, acc[b][c], 2));
                    v[c] = __fadd_rn(v[c], __shfl_down_sync(kFull, v[c], 4));
                    v[c] = __fadd_rn(v[c], __shfl_down_sync(kFull, v[c], 1));
                }
                const float t20 = __fadd_rn(v[0], v[2]), t21 = __fadd_rn(v[1], v[3]);
                const float t3 = __fadd_rn(t20, t21);
                if (p == 0 && live) {
                    double total = (double)t3;
                    const uint16_t* wr = reinterpret_cast<const uint16_t*>(wrow);
                    for (int i = n32; i < a.E; ++i)
                        total = __fma_rn((double)__uint_as_float((uint32_t)wr[i] << 16),
                                         (double)xn[b * a.E + i], total);
                    a.out[(int64_t)b * a.lld + v0 + r] = __double2float_rn(total);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (!ok) set_status(a.status, kStatusTimeout);
}

__device__ __forceinline__ uint64_t lm_keep(uint64_t* buf, uint32_t n, uint32_t kk, int lane,
                                            uint32_t slack, uint32_t* kept) {
    return warp_topk_keep<(kLmCap + 31) / 32>(buf, n, kk, lane, slack, kept);
}

// Keys an intermediate compaction may keep beyond keff: the radix walk stops once
// its bucket is within this many keys of keff (a quarter of keff), which saves most
// of its bits, while the kept keys still leave room for a whole 32-column chunk.
__device__ __forceinline__ uint32_t lm_slack(uint32_t keff) {
    const uint32_t room = keff < (uint32_t)kLmKeffMax ? (uint32_t)kLmKeffMax - keff : 0u;
    return min(keff / 4u, room);
}

// Cuts one row's buffer (row lm_dp(L) of this warp's 16, L an owner lane) back to
// its keff best keys (exact) or to the radix walk's bucket of at most keff +
// lm_slack(keff) keys; lanes L and L ^ 2 take the new count and threshold (the
// higher of the new one and one they hold already), and L publishes its value order
// for the row's other slices.
__device__ __forceinline__ void lm_compact_row(uint64_t* rows, int L, uint32_t& count,
                                               uint32_t& tau_ord, float& tau_f, bool& open,
                                               uint32_t keff, uint32_t* gtau, int lane,
                                               bool exact) {
    const uint32_t n = __shfl_sync(kFull, count, L);
    const uint32_t kk = __shfl_sync(kFull, keff, L);
    uint32_t kept = kk;
    const uint64_t T = lm_keep(rows + (int64_t)lm_dp(L) * kLmRowStride, n, kk, lane,
                               exact ? 0u : lm_slack(kk), &kept);
    if ((lane & ~2) == L) {
        count = kept;  // keff keys, or (not exact) the bucket of at most keff + slack
        uint32_t t = (uint32_t)(T >> 32);
        if (gtau && lane == L) atomicMax(gtau, t);
        if (!open && tau_ord > t) t = tau_ord;
        tau_ord = t;
        tau_f = value_of_ord(t);
        open = false;
    }
}

// A row's slices share a bound: a slice whose buffer held more than keff keys
// publishes the value order g of its keff-th best, so the row has at least keff keys
// of value >= value(g), and no key of a smaller value is among its keff best.  Other
// slices hold ids below or above this slice's, so an equal value may still rank in;
// they take the bound as "value >= value(g)", that is order g - 1 under the strict
// test of lm_pass_mask.  Orders at or below -FLT_MAX (and NaN's 0) are not taken;
// for g = +-0, g - 1 is -0, which zeros would not pass, so -denorm_min stands in.
__device__ __forceinline__ uint32_t lm_shared_bound(const uint32_t* gtau) {
    uint32_t g;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(g) : "l"(gtau));
    return g;
}
__device__ __forceinline__ void lm_adopt(uint32_t g, uint32_t& tau_ord, float& tau_f, bool& open) {
    if (g <= 0x00800000u) return;
    uint32_t c = g - 1u;
    if (c == 0x7fffffffu) c = 0x7ffffffeu;
    if (open || c > tau_ord) {
        tau_ord = c;
        tau_f = value_of_ord(c);
        open = false;
    }
}

// Bit j set when this lane's column col0 + par + 2 j (< V) passes: every column
// while the buffer is open (no threshold yet), else a value order above tau_ord.
// With tau_f the threshold's value that is v > tau_f (orders are monotone in the
// value, -0 and +0 share one), or for a NaN threshold (order 0) any non-NaN value.
__device__ __forceinline__ uint32_t lm_pass_mask(const float (&v)[16], int col0, int par, int V,
                                                 uint32_t tau_ord, float tau_f, bool open) {
    const int lim = V - col0 - par;  // column j of this lane lies in the row while 2 j < lim
    const uint32_t inside = lim >= 32 ? 0xffffu : (lim <= 0 ? 0u : (1u << ((lim + 1) >> 1)) - 1u);
    if (open) return inside;
    // an OR tree (depth 3) over all 16 tests: nothing hides a dependent chain's
    // latency, and some row of the warp passes in most chunks, so there is no early
    // test of the chunk's maximum
    uint32_t b[8];
    if (tau_ord != 0u) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
            b[j] = (v[j] > tau_f ? 1u << j : 0u) | (v[j + 8] > tau_f ? 1u << (j + 8) : 0u);
    } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
            b[j] = (v[j] == v[j] ? 1u << j : 0u) | (v[j + 8] == v[j + 8] ? 1u << (j + 8) : 0u);
    }
#pragma unroll
    for (int w = 4; w >= 1; w >>= 1)
#pragma unroll
        for (int j = 0; j < w; ++j) b[j] |= b[j + w];
    return b[0] & inside;
}

// v[j] for a j known only at run time, by four levels of selects (the array stays
// in registers; an indexed load would put it in local memory).
__device__ __forceinline__ float lm_pick(const float (&v)[16], int j) {
    float x8[8], x4[4], x2[2];
#pragma unroll
    for (int i = 0; i < 8; ++i) x8[i] = (j & 8) ? v[i + 8] : v[i];
#pragma unroll
    for (int i = 0; i < 4; ++i) x4[i] = (j & 4) ? x8[i + 4] : x8[i];
#pragma unroll
    for (int i = 0; i < 2; ++i) x2[i] = (j & 2) ? x4[i + 2] : x4[i];
    return (j & 1) ? x2[1] : x2[0];
}

__device__ __forceinline__ uint64_t lm_key(float x, int col) {
    return ((uint64_t)ord_of(x) << 32) | (uint64_t)(~(uint32_t)col);
}

// One 32-column chunk of a tile for this warp's 16 rows, each row split over a lane
// pair (L, L ^ 2: 16 columns each, interleaved).  Rows whose passing columns would
// overflow their buffers are compacted first (the whole warp, one row at a time),
// then both lanes of every row append their passing keys, the lane with the odd
// columns behind the other's; both keep the row's count.
__device__ __forceinline__ void lm_chunk(const uint32_t (&r)[16], int col0, int par, int V,
                                         bool sel, float* lrow, bool& x0nan, bool select,
                                         uint64_t* rows, uint64_t* mine, uint32_t& count,
                                         uint32_t& tau_ord, float& tau_f, bool& open,
                                         uint32_t keff, uint32_t* gtau, int lane) {
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
    if (col0 == 0 && par == 0) x0nan = (v[0] != v[0]);
    if (lrow) {
#pragma unroll
        for (int j = 0; j < 16; ++j)
            if (col0 + par + 2 * j < V) lrow[col0 + par + 2 * j] = v[j];
    }
    if (!select) return;
    uint32_t pm = sel ? lm_pass_mask(v, col0, par, V, tau_ord, tau_f, open) : 0u;
    {
        const uint32_t pc = __popc(pm);
        const uint32_t tot = pc + __shfl_xor_sync(kFull, pc, 2);
        unsigned over = __ballot_sync(kFull, count + tot > (uint32_t)kLmCap) & kLmOwnerLanes;
        while (over) {
            const int L = __ffs(over) - 1;
            over &= over - 1;
            lm_compact_row(rows, L, count, tau_ord, tau_f, open, keff, gtau, lane, false);
            if ((lane & ~2) == L) pm = lm_pass_mask(v, col0, par, V, tau_ord, tau_f, open);
        }
    }
    const uint32_t pc = __popc(pm);
    const uint32_t pp = __shfl_xor_sync(kFull, pc, 2);
    uint32_t at = count + (par ? pp : 0u);
    count += pc + pp;
    const int cb = col0 + par;  // column of v[j]: cb + 2 j
    // Appends: while any lane passes many columns (a buffer still open) one
    // predicated step per column; otherwise a loop over each lane's passing columns,
    // two per step (the two picks are independent, so their latencies overlap).
    if (__any_sync(kFull, pc > 8u)) {
        if (pm) {
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if ((pm >> j) & 1u) mine[at++] = lm_key(v[j], cb + 2 * j);
        }
    } else {
        while (pm) {
            const int j1 = __ffs(pm) - 1;
            pm &= pm - 1u;
            const bool two = pm != 0u;
            const int j2 = two ? __ffs(pm) - 1 : j1;
            pm &= pm - 1u;
            const float x1 = lm_pick(v, j1), x2 = lm_pick(v, j2);
            mine[at] = lm_key(x1, cb + 2 * j1);
            if (two) mine[at + 1] = lm_key(x2, cb + 2 * j2);
            at += two ? 2u : 1u;
        }
    }
}

// P = 1: one CTA per tile.  P = 2: launched in clusters of two CTAs, each pair one
// 256 x 256 tile at a time (LmGeom); the leader (cluster rank 0) issues the MMAs for
// both, the copies of both CTAs count on the leader's barriers, the MMA commits
// arrive on both CTAs' barriers, and both epilogues free an accumulator on the
// leader's barrier.
template <int P>
__global__ void __launch_bounds__(kLmThreads, 1)
    zs_lmhead_kernel(const __grid_constant__ CUtensorMap tm_a,
                     const __grid_constant__ CUtensorMap tm_b,
                     const __grid_constant__ CUtensorMap tm_c, const LmArgs a) {
    using G = LmGeom<P>;
    extern __shared__ uint8_t lm_raw[];
    const uint32_t pad = (1024u - (smem_addr(lm_raw) & 1023u)) & 1023u;
    LmSmem& sm = *reinterpret_cast<LmSmem*>(lm_raw + pad);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nk = (a.E + kLmBK - 1) / kLmBK;
    volatile int* abort = &sm.abort;
    const uint32_t rank = P == 2 ? cluster_rank() : 0u;  // this CTA's half of the pair
    const bool leader = rank == 0u;

    const int ns = a.ns;
    uint8_t* const tiles_a = sm.ring;
    uint8_t* const tiles_b = sm.ring + (size_t)ns * kLmTileABytes;
    uint64_t* const cand = reinterpret_cast<uint64_t*>(sm.ring + (size_t)ns * kLmStageBytes);

    if (threadIdx.x == 0) {
        for (int s = 0; s < ns; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        for (int i = 0; i < G::kAccs; ++i) {
            mbar_init(&sm.acc_full[i], 1);
            mbar_init(&sm.acc_empty[i], G::kAccEmptyCount);
        }
        mbar_init(&sm.drain, 1);
        sm.abort = 0;
        mbar_fence_init();
        tma_prefetch_map(&tm_a);
        tma_prefetch_map(&tm_b);
    }
    if (warp == 1) {
        if (P == 1) {
            tc_alloc(&sm.tmem_base, kLmTmemCols);
            tc_relinquish();
        } else {
            tc_alloc_pair(&sm.tmem_base, kLmTmemCols);
            tc_relinquish_pair();
        }
    }
    tc_fence_before();
    if (P == 1)
        __syncthreads();
    else
        cluster_sync_all();  // both CTAs' barriers exist before either signals the other's
    tc_fence_after();
    const uint32_t tmem = sm.tmem_base;
    int u_begin, u_end;
    lm_range<P>(a, u_begin, u_end);

    // Launched behind zs_lm_rmsnorm_kernel as a programmatic dependent: the copy
    // issuer first pulls its first weight boxes into L2 (they do not depend on the
    // rmsnorm), then every thread waits for that grid before reading xn or the
    // shared bounds the rmsnorm clears.
    if (warp == 0 && lane == 0 && a.prefetch > 0) {
        int left = a.prefetch;
        for (int u = u_begin; left > 0 && u < u_end; ++u) {
            int m, s, t0, t1;
            lm_unit(a, u, m, s, t0, t1);
            for (int t = t0; left > 0 && t < t1; ++t)
                for (int kb = 0; left > 0 && kb < nk; ++kb, --left)
                    tma_prefetch_l2_2d(&tm_b, kb * kLmBK, t * G::kCols + (int)rank * kLmN);
        }
    }
    grid_dep_wait();

    if (warp == 0) {
        // ---- copy issuer ----
        if (lane == 0) {
            uint32_t stage = 0, phase = 0;
            int64_t issued = 0;
            bool ok = true;
            for (int u = u_begin; ok && u < u_end; ++u) {
                int m, s, t0, t1;
                lm_unit(a, u, m, s, t0, t1);
                for (int t = t0; ok && t < t1; ++t) {
                    for (int kb = 0; kb < nk; ++kb) {
                        if (!lm_wait(&sm.empty[stage], phase ^ 1u, abort)) {
                            ok = false;
                            break;
                        }
                        if (P == 1) {
                            mbar_arrive_expect_tx(&sm.full[stage], kLmTileABytes + kLmTileBBytes);
                            tma_load_2d(tiles_a + stage * kLmTileABytes, &tm_a, kb * kLmBK,
                                        m * kLmM, &sm.full[stage]);
                            tma_load_2d(tiles_b + stage * kLmTileBBytes, &tm_b, kb * kLmBK,
                                        t * kLmN, &sm.full[stage]);
                        } else {
                            // both CTAs' bytes count on the leader's barrier, which the
                            // leader alone arms; the peer's copies may land first
                            if (leader)
                                mbar_arrive_expect_tx(&sm.full[stage],
                                                      2u * (kLmTileABytes + kLmTileBBytes));
                            const uint32_t bar = smem_in_cta(&sm.full[stage], 0u);
                            tma_load_2d_pair(tiles_a + stage * kLmTileABytes, &tm_a, kb * kLmBK,
                                             m * G::kRows + (int)rank * kLmM, bar);
                            tma_load_2d_pair(tiles_b + stage * kLmTileBBytes, &tm_b, kb * kLmBK,
                                             t * G::kCols + (int)rank * kLmN, bar);
                        }
                        ++issued;
                        if (++stage == (uint32_t)ns) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                }
            }
            if (!ok) set_status(a.status, kStatusTimeout);
            // Every copy issued has landed before the CTA may exit (the MMA issuer
            // has waited for all of them already unless a wait ran out).  The peer
            // of a pair cannot see its copies complete (they count on the leader's
            // barriers, which the leader waits for): after a wait ran out it gives
            // them time to land instead.
            if (P == 1 || leader) {
                for (int64_t i = issued - ns; i < issued; ++i)
                    if (i >= 0) mbar_wait_bounded(&sm.full[i % ns], (uint32_t)((i / ns) & 1));
            } else if (!ok) {
                for (int i = 0; i < 100; ++i) __nanosleep(1000);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- MMA issuer (the leader's, for a pair) ----
        if (lane == 0 && (P == 1 || leader)) {
            uint32_t stage = 0, phase = 0, acc = 0, acc_phase = 0;
            bool ok = true;
            for (int u = u_begin; ok && u < u_end; ++u) {
                int m, s, t0, t1;
                lm_unit(a, u, m, s, t0, t1);
                for (int t = t0; ok && t < t1; ++t) {
                    if (!lm_wait(&sm.acc_empty[acc], acc_phase ^ 1u, abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem + acc * (uint32_t)G::kCols;
                    for (int kb = 0; kb < nk; ++kb) {
                        if (!lm_wait(&sm.full[stage], phase, abort)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        const uint64_t ad = sw128_desc(tiles_a + stage * kLmTileABytes);
                        const uint64_t bd = sw128_desc(tiles_b + stage * kLmTileBBytes);
#pragma unroll
                        for (int k = 0; k < kLmBK / 16; ++k) {
                            if (P == 1)
                                tc_mma_bf16(d, ad + 2ull * k, bd + 2ull * k, G::kIdesc,
                                            (kb | k) != 0 ? 1u : 0u);
                            else
                                tc_mma_bf16_pair(d, ad + 2ull * k, bd + 2ull * k, G::kIdesc,
                                                 (kb | k) != 0 ? 1u : 0u);
                        }
                        if (P == 1)
                            tc_commit(&sm.empty[stage]);
                        else
                            tc_commit_pair(&sm.empty[stage], (uint16_t)3u);  // both CTAs' stage
                        if (++stage == (uint32_t)ns) {
                            stage = 0;
                            phase ^= 1u;
                        }
                    }
                    if (!ok) break;
                    if (P == 1)
                        tc_commit(&sm.acc_full[acc]);
                    else
                        tc_commit_pair(&sm.acc_full[acc], (uint16_t)3u);
                    if (++acc == G::kAccs) {
                        acc = 0;
                        acc_phase ^= 1u;
                    }
                }
            }
            if (!ok) set_status(a.status, kStatusTimeout);
            // Every MMA issued has completed before the tensor memory is freed.
            if (P == 1)
                tc_commit(&sm.drain);
            else
                tc_commit_pair(&sm.drain, (uint16_t)1u);  // the leader's own barrier
            mbar_wait_bounded(&sm.drain, 0u);
        }
        __syncwarp();
    } else {
        // ---- epilogue: 8 warps, two per TMEM lane quarter, each 16 rows of the
        // tile (TMEM lanes); a row's 32-column chunk is split over a lane pair ----
        const int ew = warp - 2;
        const int g16 = (warp & 3) * 32 + (ew >> 2) * 16;  // first row (lane) of this warp
        const int dp = lm_dp(lane), par = lm_par(lane);
        const bool owner = par == 0;
        const int r_in = g16 + dp;
        // rows at or beyond the batch never touch their buffers (the host sized
        // the ring so that the buffers of the rows in use fit behind it)
        uint64_t* rows = cand + (int64_t)g16 * kLmRowStride;
        uint64_t* mine = rows + (int64_t)dp * kLmRowStride;
        const uint32_t lane_addr = tmem + ((uint32_t)g16 << 16);
        uint32_t acc = 0, acc_phase = 0;
        bool ok = true;
        uint32_t count = 0;    // keys in the row's buffer (both lanes of the pair)
        uint32_t tau_ord = 0;  // threshold's value order (after the first compaction)
        float tau_f = 0.0f;    // its value
        bool open = true;      // no threshold yet: every column enters
        bool x0nan = false, has0 = false;
        int stg_buf = 0;  // logits-only staging buffer of this warp (two, alternating)
        for (int u = u_begin; ok && u < u_end; ++u) {
            int m, s, t0, t1;
            lm_unit(a, u, m, s, t0, t1);
            const int row = m * G::kRows + (int)rank * kLmM + r_in;
            const bool valid = row < a.B;
            uint32_t keff = 1;
            if (valid) {
                const RowPlan rp = plan_row(load_params(a.row_params, a.shared, row), a.V_total,
                                            nullptr, nullptr, 0, row);
                keff = (uint32_t)rp.ksel;
            }
            if (u == u_begin || s == 0) {  // a new run of this row tile's slices
                count = 0;
                tau_ord = 0;
                open = true;
                x0nan = false;
                has0 = false;
            }
            has0 = has0 || t0 == 0;
            const bool sel = a.select && valid;
            uint32_t* gtau = (sel && a.tau) ? a.tau + row : nullptr;
            float* lrow = (a.out_logits && valid) ? a.out_logits + (int64_t)row * a.logits_ld : nullptr;
            for (int t = t0; t < t1; ++t) {
                const bool got = lm_wait(&sm.acc_full[acc], acc_phase, abort);
                if (!__all_sync(kFull, got)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const int tcol = t * G::kCols;
                const uint32_t base = lane_addr + acc * (uint32_t)G::kCols;
                // the other slices' bound, read now and taken after this tile (the
                // owner's reading, so both lanes of a row keep one threshold)
                uint32_t g_seen = (gtau && owner) ? lm_shared_bound(gtau) : 0u;
                g_seen = __shfl_sync(kFull, g_seen, lane & ~2);
                // The next chunk's TMEM load is in flight while this chunk is
                // processed (rb is written asynchronously between its issue and the
                // wait; nothing reads it there).
                uint32_t rb[16];
                __syncwarp();
                tc_ld16_issue(base, rb);
#pragma unroll 1
                for (int c = 0; c < G::kCols / 32; ++c) {
                    uint32_t ra[16];
                    tc_ld16_wait(rb);
#pragma unroll
                    for (int j = 0; j < 16; ++j) ra[j] = rb[j];
                    __syncwarp();
                    if (c + 1 < G::kCols / 32) tc_ld16_issue(base + (uint32_t)((c + 1) * 32), rb);
                    if (a.tma_out) {
                        // logits only: this warp's 16 rows x 32 columns go to a staging
                        // buffer in the (here unused) candidate area, in the 128-byte
                        // swizzled layout of the output tensor map (rows of 128 bytes,
                        // 16-byte unit u of row i at u ^ (i & 7)), then one TMA store
                        uint8_t* stg = reinterpret_cast<uint8_t*>(cand) + (ew * 2 + stg_buf) * 2048;
                        if (lane == 0) bulk_wait_read_1();  // the store two chunks ago read it
                        __syncwarp();
                        uint8_t* my = stg + dp * 128;
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int col = par + 2 * j;
                            *reinterpret_cast<uint32_t*>(my + ((((col >> 2) ^ (dp & 7)) << 4) |
                                                               ((col & 3) << 2))) = ra[j];
                        }
                        fence_proxy_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            tma_store_2d(&tm_c, stg, tcol + c * 32,
                                         m * G::kRows + (int)rank * kLmM + g16);
                            bulk_commit_group();
                        }
                        stg_buf ^= 1;
                        continue;
                    }
                    lm_chunk(ra, tcol + c * 32, par, a.V, sel, lrow, x0nan, a.select, rows, mine,
                             count, tau_ord, tau_f, open, keff, gtau, lane);
                }
                if (gtau) lm_adopt(g_seen, tau_ord, tau_f, open);
                tc_fence_before();
                __syncwarp();  // the warp's TMEM loads have all completed
                if (lane == 0) {
                    if (P == 1)
                        mbar_arrive(&sm.acc_empty[acc]);
                    else
                        mbar_arrive_cluster(smem_in_cta(&sm.acc_empty[acc], 0u));
                }
                if (++acc == G::kAccs) {
                    acc = 0;
                    acc_phase ^= 1u;
                }
            }
            if (!ok) break;
            if (!a.select) continue;
            // The run goes on into the next slice of this row tile: this slice's
            // block stays empty and the buffer carries over.
            const bool run_on = (u + 1 < u_end) && (s + 1 < a.S);
            if (run_on) {
                if (sel && owner)
                    *reinterpret_cast<uint4*>(a.part + ((int64_t)row * a.S + s) * kLmPartStride) =
                        make_uint4(0u, 0u, __float_as_uint(-INFINITY), 0u);
                continue;
            }
            unsigned over = __ballot_sync(kFull, sel && count > keff) & kLmOwnerLanes;
            while (over) {
                const int L = __ffs(over) - 1;
                over &= over - 1;
                lm_compact_row(rows, L, count, tau_ord, tau_f, open, keff, gtau, lane, true);
            }
            if (sel && owner) {  // the owner lane holds column 0's NaN flag
                uint8_t* blk = a.part + ((int64_t)row * a.S + s) * kLmPartStride;
                const uint32_t flags = has0 ? (kPartHasId0 | (x0nan ? kPartX0Nan : 0u)) : 0u;
                *reinterpret_cast<uint4*>(blk) = make_uint4(count, flags, __float_as_uint(-INFINITY), 0u);
                uint64_t* keys = reinterpret_cast<uint64_t*>(blk + kPartialHeaderBytes);
                for (uint32_t i = 0; i < count; ++i) keys[i] = mine[i];
            }
        }
        if (!ok) set_status(a.status, kStatusTimeout);
        if (a.tma_out && lane == 0) bulk_wait_all();  // stores done before the CTA exits
        __syncwarp();
    }

    tc_fence_before();
    if (P == 1)
        __syncthreads();
    else
        cluster_sync_all();  // the leader's MMAs (into both CTAs) have drained
    if (warp == 1) {
        tc_fence_after();
        if (P == 1)
            tc_dealloc(tmem, kLmTmemCols);
        else
            tc_dealloc_pair(tmem, kLmTmemCols);
    }
}

}  // namespace zs
