// zs_sampler.cu -- host side of the C ABI in include/zs_sampler.h.
//
// Plans a batch (which path each row can take, where the candidate blocks go),
// owns the per-device scratch, and launches:
//   zs_wselect_kernel  rows whose shortlist + penalty window is at most 320 (every
//                      default of the reference)
//   zs_select_kernel   rows with longer shortlists up to 2048
//   zs_warp_merge_kernel / zs_merge_kernel  per row: merge the blocks, sort, draw
//                      (also the vocab-sharded merge after the all-gather)
//   zs_large_kernel    the remaining rows (top_k > 2048, long penalty windows)
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <cudaTypedefs.h>
#include <nvtx3/nvToolsExt.h>

#include "zs_kernels.cuh"
#include "zs_lmhead.cuh"
#include "zs_sampler.h"
#include "zs_stats.cuh"

// Named NVTX ranges around the entry points that launch work, so a timeline
// (Nsight Systems, or any NVTX client) shows each call with its kernels.  Without
// a tool attached a push/pop is a check of one function pointer.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};

static_assert(sizeof(zs_params) == sizeof(zs::Params), "zs_params layout");
static_assert(sizeof(zs_row_info) == sizeof(zs::RowInfo), "zs_row_info layout");
static_assert(sizeof(zs_row_info) == 48, "zs_row_info size");

namespace {

thread_local std::string g_last_error;

zs_status fail(zs_status s, const std::string& msg) {
    g_last_error = msg;
    return s;
}

zs_status cuda_fail(cudaError_t e, const char* what) {
    g_last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return e == cudaErrorMemoryAllocation ? ZS_ERR_OUT_OF_MEMORY : ZS_ERR_CUDA;
}

#define ZS_CUDA(call)                                        \
    do {                                                     \
        cudaError_t e_ = (call);                             \
        if (e_ != cudaSuccess) return cuda_fail(e_, #call);  \
    } while (0)

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    bool ok = false;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) == cudaSuccess && cudaSetDevice(dev) == cudaSuccess) ok = true;
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

// Fixed layouts of the vocab-sharded mode, so every rank derives the same blocks.
constexpr int kShardLayoutCtas = 296;
constexpr int kShardLayoutWarps[2] = {148 * zs::WCfgS::kWarps, 148 * zs::WCfgL::kWarps};

// Where the partial blocks of one call go, and which kernels run.  The block
// areas depend only on the batch, the columns and the params (never on whether a
// history is passed), so the ranks of a vocab shard agree on them.
struct Plan {
    int max_ksel = 1;
    bool any_large = false;
    bool any_penal = false;
    int max_win = 0;  // longest penalty window a row of this call may have
    // zs_select_kernel rows: [B][S] blocks at offset 0
    bool cta_area = false;    // the layout holds them
    bool launch_cta = false;  // some row of this call needs the kernel
    int S = 1;
    int slice = 0;
    int64_t part_stride = 0;
    // zs_wselect_kernel rows, one layout per warp configuration (index = class):
    // warp-piece blocks at w[c].off
    struct Warp {
        bool any = false;     // the layout holds blocks of this class
        bool launch = false;  // some row of this call may be of this class
        int max_ksel = 1;
        int64_t E = 0;
        int32_t NW = 1;
        int32_t P = 1;
        int32_t Vn = 1;
        int64_t stride = 0;
        int64_t off = 0;
        int64_t bytes() const { return any ? (int64_t)NW * P * stride : 0; }
    } w[2];
    int64_t bytes = 0;  // all blocks of one rank
};

int ksel_of(const zs_params& p, int V_total) {
    if (p.temp <= 0.0f) return 1;
    if (p.top_k > 0) return std::min(p.top_k, V_total);
    return std::min(zs::kShortlistDefault, V_total);
}

int win_bound_of(const zs_params& p) {
    if (!(p.repeat_penalty != 1.0f)) return 0;
    return std::max(0, p.repeat_last_n);
}

// Keys one zs_select_kernel block can hold for a row: the unit epilogue keeps the
// top keff = ksel + window plus the compaction's slack, then appends up to
// `window` penalised values.
int64_t partial_keys_for(int ksel, int wb) {
    const uint32_t keff = (uint32_t)std::min<int64_t>((int64_t)ksel + wb, zs::kKeffFastMax);
    const uint32_t slack = zs::slack_for(keff);
    const uint32_t extra = keff <= zs::kGroupMaxK ? 2 * slack + 256u : slack;
    return (int64_t)keff + extra + std::min(wb, zs::kWinFastMax);
}

int choose_slices(int B, int V, int ctas) {
    if (B <= 0 || V <= 0) return 1;
    const int smax = std::max(1, V / (2 * zs::kTileElems));
    const long want = (8L * ctas + B - 1) / B;
    return (int)std::max(1L, std::min((long)smax, want));
}

int64_t round_up(int64_t v, int64_t m) { return (v + m - 1) / m * m; }

// Cuts the [B][V_cols] batch among `layout_warps` warps (each at least
// kWMinElems columns) and sizes the warp-piece blocks for shortlists <= max_ksel.
// Few rows are spread over fewer warps than that when needed, so that the blocks
// of one row, from all n_ranks ranks, hold at most kCandCap - kCandMargin keys:
// the merge then gathers a row in one pass.  With at least as many warps as rows
// the warp count is a multiple of B, which puts every share inside one row
// (warp w's share starts at w E / NW = (w / q) Vn for q = NW / B): no warp ramps
// up two pieces, and the slowest warp, which sets the kernel's time, is no longer
// one that straddles a row boundary (measured on B200: 256 rows of top-k 40
// 72.5 -> 63.9 µs, 1024 rows of the 256 shortlist 262 -> 234 µs, 512 rows of
// top-k 1024 407 -> 287 µs).
void plan_warp_layout(Plan::Warp& pl, int B, int V_cols, int layout_warps, int max_ksel,
                      int n_ranks) {
    pl.Vn = std::max(1, V_cols);
    pl.E = (int64_t)B * pl.Vn;
    const int64_t by_size = std::max<int64_t>(1, pl.E / zs::kWMinElems);
    const int64_t blocks_per_row =
        std::max<int64_t>(1, (zs::kCandCap - zs::kCandMargin) / ((int64_t)std::max(1, max_ksel) *
                                                                 std::max(1, n_ranks)));
    // a row spanning w warps' shares owns at most NW / B + 2 of them
    const int64_t by_merge = (int64_t)B * std::max<int64_t>(1, blocks_per_row - 2);
    pl.NW = (int32_t)std::max<int64_t>(
        1, std::min<int64_t>({(int64_t)layout_warps, by_size, by_merge}));
    if (pl.NW >= B) pl.NW = (pl.NW / B) * B;
    const int64_t share = (pl.E + pl.NW - 1) / pl.NW;
    pl.P = (int32_t)((share + pl.Vn - 1) / pl.Vn + 1);
    pl.stride = round_up(zs::kPartialHeaderBytes + 8LL * std::max(1, max_ksel), 16);
}

// Places the block areas: [B][S] CTA blocks, then each warp configuration's.
void place_areas(Plan& pl, int B) {
    const int64_t cta_bytes = pl.cta_area ? (int64_t)B * pl.S * pl.part_stride : 0;
    pl.w[0].off = round_up(cta_bytes, 256);
    pl.w[1].off = round_up(pl.w[0].off + pl.w[0].bytes(), 256);
    pl.bytes = pl.w[1].off + pl.w[1].bytes();
}

Plan make_plan(int B, int V_cols, int V_total, const zs_params* params, int per_row, int ctas,
               const int* layout_warps, bool have_history, int n_ranks = 1) {
    Plan pl;
    const int np = per_row ? B : 1;
    int64_t max_keys = 1;
    for (int i = 0; i < np; ++i) {
        const zs_params& p = params[i];
        const int ks = ksel_of(p, V_total);
        const int wb = win_bound_of(p);
        pl.max_ksel = std::max(pl.max_ksel, ks);
        if (have_history && wb > 0) {
            pl.any_penal = true;
            pl.max_win = std::max(pl.max_win, wb);
        }
        // The device puts a row in the first class whose limits ksel + its
        // actual window (empty without a history) and the window fit: the short
        // warp configuration, the long one, the CTA path; the rest on the large
        // path.  Any class a row may take gets a block area (whatever the
        // history), and a launch when this call can put a row there.
        using S = zs::WCfgS;
        using Lc = zs::WCfgL;
        if (ks <= S::kKeffMax) {
            pl.w[0].any = pl.w[0].launch = true;
            pl.w[0].max_ksel = std::max(pl.w[0].max_ksel, ks);
        }
        const bool long_s = wb > 0 && (ks + wb > S::kKeffMax || wb > S::kWinMax);
        if (ks <= Lc::kKeffMax && (ks > S::kKeffMax || long_s)) {
            pl.w[1].any = true;
            pl.w[1].max_ksel = std::max(pl.w[1].max_ksel, ks);
            if (ks > S::kKeffMax || have_history) pl.w[1].launch = true;
        }
        const bool long_l = wb > 0 && (ks + wb > Lc::kKeffMax || wb > Lc::kWinMax);
        if (ks <= zs::kKeffFastMax && (ks > Lc::kKeffMax || long_l)) {
            pl.cta_area = true;
            max_keys = std::max(max_keys, partial_keys_for(ks, wb));
            if (ks > Lc::kKeffMax || have_history) pl.launch_cta = true;
        }
        if (ks > zs::kKeffFastMax ||
            (have_history && ((long)ks + wb > zs::kKeffFastMax || wb > zs::kWinFastMax)))
            pl.any_large = true;
    }
    pl.S = choose_slices(B, V_cols, ctas);
    const int per = (V_cols + pl.S - 1) / pl.S;
    pl.slice = std::max(4, (per + 3) & ~3);
    pl.S = std::max(1, (V_cols + pl.slice - 1) / pl.slice);
    pl.part_stride = round_up(zs::kPartialHeaderBytes + 8LL * max_keys, 16);
    for (int c = 0; c < 2; ++c)
        plan_warp_layout(pl.w[c], B, V_cols, layout_warps[c], pl.w[c].max_ksel, n_ranks);
    place_areas(pl, B);
    return pl;
}

// Columns per rank the shard layout is cut for: equal slices, the last one also
// taking the remainder (the largest shard that convention gives).
int shard_cols(int V_total, int n_ranks) { return V_total / n_ranks + V_total % n_ranks; }

// Byte ranges of one rank's block area that hold every block the merge of rows
// [r0, r0 + n) reads: the rows' CTA blocks, and in each warp layout all pieces of
// the warps whose shares touch those rows (block_at's arithmetic).  At most three
// (offset, length) pairs, in area order; returns how many.
int row_spans(const Plan& pl, int B, int r0, int n, int64_t spans[3][2]) {
    int k = 0;
    if (n <= 0 || r0 < 0 || r0 + n > B) return 0;
    if (pl.cta_area) {
        spans[k][0] = (int64_t)r0 * pl.S * pl.part_stride;
        spans[k][1] = (int64_t)n * pl.S * pl.part_stride;
        ++k;
    }
    for (int c = 0; c < 2; ++c) {
        const Plan::Warp& w = pl.w[c];
        if (!w.any) continue;
        const int32_t w_lo = zs::wl_warp_of(w.E, w.NW, (int64_t)r0 * w.Vn);
        const int32_t w_hi = zs::wl_warp_of(w.E, w.NW, (int64_t)(r0 + n) * w.Vn - 1);
        spans[k][0] = w.off + (int64_t)w_lo * w.P * w.stride;
        spans[k][1] = (int64_t)(w_hi - w_lo + 1) * w.P * w.stride;
        ++k;
    }
    return k;
}

// ---- NCCL, resolved at run time from the libnccl.so.2 this process uses ----
// ncclResult_t values used here (nccl.h): ncclSuccess 0, ncclInProgress 7.
constexpr int kNcclSuccess = 0;
constexpr int kNcclInProgress = 7;
// ncclDataType_t: ncclUint8 1, ncclInt32 2, ncclUint64 5.
constexpr int kNcclUint8 = 1;
constexpr int kNcclInt32 = 2;
constexpr int kNcclUint64 = 5;

struct NcclApi {
    typedef int (*AllGatherFn)(const void*, void*, size_t, int, void*, cudaStream_t);
    typedef int (*SendFn)(const void*, size_t, int, int, void*, cudaStream_t);
    typedef int (*RecvFn)(void*, size_t, int, int, void*, cudaStream_t);
    typedef int (*VoidFn)();
    typedef int (*CommIntFn)(void*, int*);
    typedef int (*CommFn)(void*);
    typedef const char* (*ErrStrFn)(int);
    AllGatherFn all_gather = nullptr;
    SendFn send = nullptr;
    RecvFn recv = nullptr;
    VoidFn group_start = nullptr;
    VoidFn group_end = nullptr;
    CommIntFn user_rank = nullptr;
    CommIntFn count = nullptr;
    CommIntFn async_error = nullptr;  // ncclCommGetAsyncError(comm, ncclResult_t*)
    CommFn abort = nullptr;
    ErrStrFn err_str = nullptr;
    bool tried = false;
    bool ok = false;
};
NcclApi g_nccl;
std::mutex g_nccl_mu;

bool load_nccl() {
    std::lock_guard<std::mutex> lk(g_nccl_mu);
    if (g_nccl.tried) return g_nccl.ok;
    g_nccl.tried = true;
    void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) return false;
    g_nccl.all_gather = (NcclApi::AllGatherFn)dlsym(lib, "ncclAllGather");
    g_nccl.send = (NcclApi::SendFn)dlsym(lib, "ncclSend");
    g_nccl.recv = (NcclApi::RecvFn)dlsym(lib, "ncclRecv");
    g_nccl.group_start = (NcclApi::VoidFn)dlsym(lib, "ncclGroupStart");
    g_nccl.group_end = (NcclApi::VoidFn)dlsym(lib, "ncclGroupEnd");
    g_nccl.user_rank = (NcclApi::CommIntFn)dlsym(lib, "ncclCommUserRank");
    g_nccl.count = (NcclApi::CommIntFn)dlsym(lib, "ncclCommCount");
    g_nccl.async_error = (NcclApi::CommIntFn)dlsym(lib, "ncclCommGetAsyncError");
    g_nccl.abort = (NcclApi::CommFn)dlsym(lib, "ncclCommAbort");
    g_nccl.err_str = (NcclApi::ErrStrFn)dlsym(lib, "ncclGetErrorString");
    g_nccl.ok = g_nccl.all_gather && g_nccl.send && g_nccl.recv && g_nccl.group_start &&
                g_nccl.group_end && g_nccl.user_rank && g_nccl.count && g_nccl.async_error &&
                g_nccl.abort;
    return g_nccl.ok;
}

std::string nccl_msg(const char* what, int r) {
    return std::string(what) + ": " + (g_nccl.err_str ? g_nccl.err_str(r) : "error") + " (" +
           std::to_string(r) + ")";
}

// Rows the row-owner merge gives rank `rank`: [*r0, *r0 + *n), R = ceil(B / G)
// rows per rank, so the ranks' shares sit back to back in a [G][R] padded array.
void owner_rows(int B, int G, int rank, int* r0, int* n) {
    const int R = (B + G - 1) / G;
    const int lo = std::min(B, rank * R);
    *r0 = lo;
    *n = std::min(B, lo + R) - lo;
}

}  // namespace

struct zs_context {
    int device = 0;
    int num_sms = 0;
    int select_ctas_per_sm = 0;
    int select_ctas = 0;
    size_t select_smem = 0;
    size_t merge_smem = 0;
    size_t warp_merge_smem = 0;
    size_t wsel_smem[2] = {0, 0};  // per warp configuration (WCfgS, WCfgL)
    int wsel_warps[2] = {0, 0};    // warps of one full zs_wselect_kernel launch
    // scratch, grown on demand (never shrinks)
    uint8_t* part = nullptr;
    size_t part_bytes = 0;
    int* status = nullptr;
    zs::Params* params = nullptr;
    size_t params_n = 0;
    uint8_t* large = nullptr;
    size_t large_bytes = 0;
    uint8_t* spec = nullptr;  // speculative thresholds: [0] failed-row count, then the rows
    size_t spec_bytes = 0;
    uint8_t* gather = nullptr;  // zs_sample_sharded: every rank's blocks, padded ids/states
    size_t gather_bytes = 0;
    int32_t coll_timeout_ms = 30000;     // zs_set_collective_timeout
    cudaEvent_t coll_event = nullptr;    // marks the end of zs_sample_sharded's work
    unsigned* fail_count = nullptr;  // units whose speculative threshold was too high
    int32_t* fail_units = nullptr;
    size_t fail_units_n = 0;
    // optional per-kernel timing (zs_set_timing): event pairs around each launch
    struct TimedLaunch {
        int kind;  // 0 select, 1 merge, 2 large, 3 lm_head GEMM, 4 lm_head rmsnorm
        cudaEvent_t begin, end;
    };
    bool timing = false;
    int32_t lm_route = ZS_LMHEAD_ROUTE_AUTO;  // zs_set_lmhead_route
    int32_t lm_tiles = ZS_LMHEAD_TILES_AUTO;  // zs_set_lmhead_tiles
    int lm_pairs = 0;                         // resident CTA pairs of zs_lmhead_kernel<2>
    int32_t spec_mode = ZS_SPECULATION_ON;    // zs_set_speculation
    int small_clusters = 0;                   // zs_small_kernel clusters resident at once (0: none)
    int32_t small_max_rows = 8;               // zs_set_small_batch
    std::vector<TimedLaunch> timed;      // recorded since the last zs_get_timing
    std::vector<cudaEvent_t> spare;      // events free for reuse
    int64_t launches = 0;                // kernel launches since the last zs_get_timing
    // zs_logits_stats: where the draw of its top-N selection lands, chunk partials
    uint64_t* stats_rng = nullptr;
    size_t stats_rng_bytes = 0;
    int32_t* stats_ids = nullptr;
    size_t stats_ids_bytes = 0;
    uint8_t* stats_part = nullptr;
    size_t stats_part_bytes = 0;
    // zs_decode_step: the Rng states before the step's draws
    uint64_t* rng_prev = nullptr;
    size_t rng_prev_bytes = 0;
    // zs_lmhead_sample: normalised rows (bf16), logits of the two-pass route, the
    // driver's tensor-map encoder
    uint8_t* lm_xn = nullptr;
    size_t lm_xn_bytes = 0;
    uint8_t* lm_logits = nullptr;
    size_t lm_logits_bytes = 0;
    PFN_cuTensorMapEncodeTiled_v12000 encode_tiled = nullptr;
};

namespace {

zs_status grow(void** p, size_t* have, size_t want) {
    if (want <= *have) return ZS_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *have = 0;
    const size_t sz = std::max(want, (size_t)4096);
    ZS_CUDA(cudaMalloc(p, sz));
    *have = sz;
    return ZS_OK;
}

zs_status validate_common(zs_handle h, const float* logits, int64_t ld, int32_t batch,
                          int32_t n_vocab, const zs_params* params) {
    if (!h) return fail(ZS_ERR_INVALID_ARGUMENT, "null handle");
    if (batch < 0) return fail(ZS_ERR_INVALID_ARGUMENT, "batch < 0");
    if (!params) return fail(ZS_ERR_INVALID_ARGUMENT, "params is null");
    if (batch > 0 && n_vocab > 0) {
        if (!logits) return fail(ZS_ERR_INVALID_ARGUMENT, "logits is null");
        if (((uintptr_t)logits & 3u) != 0) return fail(ZS_ERR_INVALID_ARGUMENT, "logits not 4-byte aligned");
        if (ld < n_vocab) return fail(ZS_ERR_INVALID_ARGUMENT, "ld < n_vocab");
        if (batch > 1 && ld > (int64_t)1 << 40) return fail(ZS_ERR_INVALID_ARGUMENT, "ld too large");
    }
    return ZS_OK;
}

bool needs_rng(const zs_params* params, int per_row, int batch) {
    const int np = per_row ? batch : 1;
    for (int i = 0; i < np; ++i)
        if (!(params[i].temp <= 0.0f)) return true;
    return false;
}

zs_status upload_params(zs_context* h, const zs_params* params, int32_t per_row, int32_t batch,
                        cudaStream_t st, const zs::Params** dev) {
    *dev = nullptr;
    if (!per_row) return ZS_OK;
    if ((size_t)batch > h->params_n) {
        if (h->params) cudaFree(h->params);
        h->params = nullptr;
        h->params_n = 0;
        const size_t n = std::max((size_t)batch, (size_t)1024);
        ZS_CUDA(cudaMalloc((void**)&h->params, n * sizeof(zs::Params)));
        h->params_n = n;
    }
    ZS_CUDA(cudaMemcpyAsync(h->params, params, (size_t)batch * sizeof(zs::Params),
                            cudaMemcpyHostToDevice, st));
    *dev = h->params;
    return ZS_OK;
}

zs::Params to_dev(const zs_params& p) {
    zs::Params d;
    std::memcpy(&d, &p, sizeof(d));
    return d;
}

// Launches the select kernel for one batch, which leaves one partial block per
// (row, slice); zs_merge_kernel then merges each row's blocks, sorts the
// shortlist and draws.  Rows needing the large shortlist path follow in
// zs_large_kernel.
// Brackets one kernel launch with events when timing is on; counts launches.
struct LaunchScope {
    zs_context* h;
    int kind;
    cudaStream_t st;
    cudaEvent_t b = nullptr, e = nullptr;
    LaunchScope(zs_context* h_, int kind_, cudaStream_t st_) : h(h_), kind(kind_), st(st_) {
        h->launches += 1;
        if (!h->timing) return;
        b = take();
        e = take();
        if (b && e) cudaEventRecord(b, st);
    }
    ~LaunchScope() {
        if (!h->timing || !b || !e) return;
        cudaEventRecord(e, st);
        h->timed.push_back({kind, b, e});
    }
    cudaEvent_t take() {
        cudaEvent_t ev = nullptr;
        if (!h->spare.empty()) {
            ev = h->spare.back();
            h->spare.pop_back();
        } else if (cudaEventCreate(&ev) != cudaSuccess) {
            ev = nullptr;
        }
        return ev;
    }
};

// Merge launch: one warp per row when every shortlist fits a warp slot and the
// batch has at least two rows per SM; otherwise one CTA per row (a small batch
// has many blocks per row and too few rows to fill the GPU by warps; measured on
// B200, the two break even between 256 and 591 rows).
zs_status launch_merge(zs_context* h, const zs::MergeArgs& m, int max_ksel, bool want_lse,
                       cudaStream_t st) {
    const int rows = m.row1 - m.row0;
    if (rows <= 0) return ZS_OK;
    LaunchScope scope(h, 1, st);
    // Programmatic dependent launch: the merge may be scheduled while the kernel
    // before it finishes; it waits (grid_dep_wait) before reading any block.
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.blockDim = dim3(zs::kNC);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if ((uint32_t)max_ksel <= zs::kWarpMergeMaxK && rows >= 2 * h->num_sms) {
        // at least one CTA per SM: rows are dealt to CTAs first, then to their warps
        const int rows_per_cta = zs::kConsumerWarps;
        const int by_rows = (rows + rows_per_cta - 1) / rows_per_cta;
        cfg.gridDim = dim3(std::max(1, std::min(std::max(by_rows, std::min(rows, h->num_sms)),
                                                8 * h->num_sms)));
        cfg.dynamicSmemBytes = h->warp_merge_smem;
        e = want_lse ? cudaLaunchKernelEx(&cfg, zs::zs_warp_merge_kernel<true>, m)
                     : cudaLaunchKernelEx(&cfg, zs::zs_warp_merge_kernel<false>, m);
    } else {
        cfg.gridDim = dim3(std::max(1, std::min(rows, 4 * h->num_sms)));
        cfg.dynamicSmemBytes = h->merge_smem;
        e = want_lse ? cudaLaunchKernelEx(&cfg, zs::zs_merge_kernel<true>, m)
                     : cudaLaunchKernelEx(&cfg, zs::zs_merge_kernel<false>, m);
    }
    if (e != cudaSuccess) return cuda_fail(e, "merge launch");
    ZS_CUDA(cudaGetLastError());
    return ZS_OK;
}

zs::MergeArgs merge_args_for(const zs::Args& a, const Plan& pl, const uint8_t* gathered, int G,
                             int64_t rank_stride) {
    zs::MergeArgs m;
    std::memset(&m, 0, sizeof(m));
    m.gathered = gathered;
    m.rank_stride = rank_stride;
    m.G = G;
    m.S = pl.S;
    m.part_stride = pl.part_stride;
    m.B = a.B;
    m.row0 = 0;
    m.row1 = a.B;
    m.V_total = a.V_total;
    m.shared = a.shared;
    m.row_params = a.row_params;
    m.hist_len = a.hist_len;
    m.hist_ld = a.hist_ld;
    m.hist = a.hist;
    m.rng = a.rng;
    m.out_ids = a.out_ids;
    m.info = a.info;
    m.cand_ids = a.cand_ids;
    m.cand_probs = a.cand_probs;
    m.cand_ld = a.cand_ld;
    m.status = a.status;
    for (int c = 0; c < 2; ++c) {
        m.wl[c].off = pl.w[c].off;
        m.wl[c].E = pl.w[c].E;
        m.wl[c].stride = pl.w[c].stride;
        m.wl[c].NW = pl.w[c].NW;
        m.wl[c].P = pl.w[c].P;
        m.wl[c].Vn = pl.w[c].Vn;
    }
    return m;
}

// Sets a warp configuration's kernel attributes; its warps per full launch.
template <class C>
zs_status setup_wselect(size_t* smem, int* warps, int num_sms) {
    *smem = sizeof(zs::WSelSmem<C>);
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(zs::zs_wselect_kernel<C, true, false>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)*smem)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(zs::zs_wselect_kernel<C, false, false>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)*smem)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(zs::zs_wselect_kernel<C, false, true>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)*smem)) != cudaSuccess)
        return cuda_fail(e, "cudaFuncSetAttribute zs_wselect_kernel");
    int per_sm = 0;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, zs::zs_wselect_kernel<C, false, false>,
                                                           C::kWarps * 32, *smem)) != cudaSuccess)
        return cuda_fail(e, "occupancy query");
    if (per_sm < 1) return fail(ZS_ERR_NO_DEVICE, "zs_wselect_kernel does not fit an SM");
    *warps = per_sm * num_sms * C::kWarps;
    return ZS_OK;
}

// One warp configuration's launch over its layout in `blocks`.
template <class C>
zs_status launch_wselect(zs_context* h, zs::Args a, const Plan& pl, uint8_t* blocks, bool want_lse,
                         cudaStream_t st) {
    const Plan::Warp& L = pl.w[C::kClass];
    a.wpart = blocks + L.off;
    a.wl_E = L.E;
    a.wl_stride = L.stride;
    a.wl_NW = L.NW;
    a.wl_P = L.P;
    a.wl_Vn = L.Vn;
    a.wl_class = C::kClass;
    // At least one CTA per SM (up to one per warp): the kernel deals warp slots across
    // CTAs, so a row-aligned layout of, say, 1024 warps runs on all SMs rather than on
    // 86 full CTAs.
    const int grid = std::max((L.NW + C::kWarps - 1) / C::kWarps, std::min(L.NW, h->num_sms));
    const size_t smem = h->wsel_smem[C::kClass];
    LaunchScope scope(h, 0, st);
    if (want_lse)
        zs::zs_wselect_kernel<C, true, false><<<grid, C::kWarps * 32, smem, st>>>(a);
    else if (a.spec && L.max_ksel >= (int)zs::kSpecMinKeff)
        zs::zs_wselect_kernel<C, false, true><<<grid, C::kWarps * 32, smem, st>>>(a);
    else
        zs::zs_wselect_kernel<C, false, false><<<grid, C::kWarps * 32, smem, st>>>(a);
    ZS_CUDA(cudaGetLastError());
    return ZS_OK;
}

// Launches the select kernels that write one rank's partial blocks: the warp
// kernel's two configurations for their rows, the CTA kernel (and its exact
// redo) for the rest of the rows up to kKeffFastMax.  `blocks` is the rank's block area; a.status,
// a.fail_count and a.fail_units (>= B * S entries) are set by the caller.
zs_status launch_partials(zs_context* h, zs::Args a, const Plan& pl, uint8_t* blocks,
                          bool want_lse, cudaStream_t st) {
    a.S = pl.S;
    a.slice = pl.slice;
    a.n_units = (int32_t)std::min<int64_t>((int64_t)a.B * pl.S, INT32_MAX);
    a.part_stride = pl.part_stride;
    a.part = blocks;
    zs_status s = ZS_OK;
    if (pl.w[0].launch && (s = launch_wselect<zs::WCfgS>(h, a, pl, blocks, want_lse, st)) != ZS_OK)
        return s;
    if (pl.w[1].launch && (s = launch_wselect<zs::WCfgL>(h, a, pl, blocks, want_lse, st)) != ZS_OK)
        return s;
    if (pl.launch_cta) {
        a.redo = 0;
        ZS_CUDA(cudaMemsetAsync(a.fail_count, 0, sizeof(unsigned), st));
        const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(a.n_units, h->select_ctas));
        for (int pass = 0; pass < 2; ++pass) {
            a.redo = pass;  // pass 1 redoes the units listed by pass 0 (usually none)
            LaunchScope scope(h, 0, st);
            if (want_lse)
                zs::zs_select_kernel<true><<<grid, zs::kThreads, h->select_smem, st>>>(a);
            else
                zs::zs_select_kernel<false><<<grid, zs::kThreads, h->select_smem, st>>>(a);
            ZS_CUDA(cudaGetLastError());
        }
    }
    return ZS_OK;
}

zs_status ensure_fail_units(zs_context* h, int64_t units) {
    if ((size_t)units <= h->fail_units_n) return ZS_OK;
    if (h->fail_units) cudaFree(h->fail_units);
    h->fail_units = nullptr;
    h->fail_units_n = 0;
    const size_t n = std::max((size_t)units, (size_t)4096);
    ZS_CUDA(cudaMalloc((void**)&h->fail_units, n * sizeof(int32_t)));
    h->fail_units_n = n;
    return ZS_OK;
}

// zs_sample's launches: partial blocks in the handle's scratch, the merge (which
// sorts and draws every row of the two fast paths), then the large path.
// Blocks per CTA of the exact redo of rows whose speculative thresholds their
// merge could not certify (zs_large_kernel over a device list; normally empty).
constexpr int kSpecRedoCtas = 8;

zs_status launch_large(zs_context* h, zs::Args a, int grid, bool want_lse, cudaStream_t st) {
    const int64_t per_cta = ((int64_t)a.V * 24 + 255) & ~255LL;
    zs_status s = grow((void**)&h->large, &h->large_bytes, (size_t)per_cta * grid);
    if (s != ZS_OK) return s;
    a.large_ws = h->large;
    a.large_ws_per_cta = per_cta;
    LaunchScope scope(h, 2, st);
    if (want_lse)
        zs::zs_large_kernel<true><<<grid, zs::kNC, h->merge_smem, st>>>(a);
    else
        zs::zs_large_kernel<false><<<grid, zs::kNC, h->merge_smem, st>>>(a);
    ZS_CUDA(cudaGetLastError());
    return ZS_OK;
}

// One launch for a small batch: a cluster of zs::kSmallCl CTAs per row
// (zs_small_kernel), when every row fits that kernel's limits.
bool small_path_ok(const zs_context* h, const zs::Args& a, const Plan& pl, bool want_lse) {
    return !want_lse && a.mode == 0 && a.B >= 1 && a.B <= h->small_max_rows &&
           a.B <= h->small_clusters && !pl.any_large && pl.max_win <= zs::kSmallWinMax &&
           pl.max_ksel <= (int)zs::kGroupMaxK && a.V >= zs::kSmallMinCols &&
           a.V <= zs::kSmallMaxCols && ((uintptr_t)a.logits & 15u) == 0 && (a.ld & 3) == 0;
}

zs_status launch_small(zs_context* h, const zs::Args& a, cudaStream_t st) {
    LaunchScope scope(h, 0, st);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = zs::kSmallCl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(a.B * zs::kSmallCl);
    cfg.blockDim = dim3(zs::kNC);
    cfg.dynamicSmemBytes = sizeof(zs::SmallSmem);
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, zs::zs_small_kernel, a);
    if (e != cudaSuccess) return cuda_fail(e, "small-batch launch");
    ZS_CUDA(cudaGetLastError());
    return ZS_OK;
}

zs_status launch_select(zs_context* h, const zs::Args& base, const Plan& pl, bool want_lse,
                        cudaStream_t st) {
    zs::Args a = base;
    a.status = h->status;
    if (small_path_ok(h, a, pl, want_lse)) return launch_small(h, a, st);
    zs_status s = grow((void**)&h->part, &h->part_bytes, (size_t)std::max<int64_t>(pl.bytes, 16));
    if (s != ZS_OK) return s;
    if (pl.launch_cta) {
        s = ensure_fail_units(h, (int64_t)a.B * pl.S);
        if (s != ZS_OK) return s;
    }
    a.fail_count = h->fail_count;
    a.fail_units = h->fail_units;
    // Speculative opening thresholds for the warp paths' long shortlists: the
    // merge lists the rows it cannot certify and zs_large_kernel redoes them.
    const bool spec = h->spec_mode != ZS_SPECULATION_OFF && !want_lse && a.mode == 0 &&
                      a.V >= zs::kSpecMinCols &&
                      ((pl.w[0].launch && pl.w[0].max_ksel >= (int)zs::kSpecMinKeff) ||
                       (pl.w[1].launch && pl.w[1].max_ksel >= (int)zs::kSpecMinKeff));
    unsigned* spec_count = nullptr;
    int32_t* spec_rows = nullptr;
    if (spec) {
        s = grow((void**)&h->spec, &h->spec_bytes, 256 + (size_t)a.B * sizeof(int32_t));
        if (s != ZS_OK) return s;
        spec_count = reinterpret_cast<unsigned*>(h->spec);
        spec_rows = reinterpret_cast<int32_t*>(h->spec + 256);
        ZS_CUDA(cudaMemsetAsync(spec_count, 0, sizeof(unsigned), st));
        a.spec = 1;
    }
    s = launch_partials(h, a, pl, h->part, want_lse, st);
    if (s != ZS_OK) return s;
    if (pl.w[0].any || pl.w[1].any || pl.cta_area) {
        zs::MergeArgs m = merge_args_for(a, pl, h->part, 1, 0);
        m.spec_count = spec_count;
        m.spec_rows = spec_rows;
        m.spec_redo_all = h->spec_mode == ZS_SPECULATION_REDO_ALL ? 1 : 0;
        s = launch_merge(h, m, pl.max_ksel, want_lse, st);
        if (s != ZS_OK) return s;
    }
    if (pl.any_large) {
        s = launch_large(h, a, std::max(1, std::min(a.B, h->num_sms)), want_lse, st);
        if (s != ZS_OK) return s;
    }
    if (spec) {
        zs::Args r = a;
        r.spec_count = spec_count;
        r.spec_rows = spec_rows;
        s = launch_large(h, r, std::max(1, std::min(a.B, kSpecRedoCtas)), want_lse, st);
        if (s != ZS_OK) return s;
    }
    return ZS_OK;
}

}  // namespace

namespace {

using Clock = std::chrono::steady_clock;

// A NCCL call's result on a communicator that may be non-blocking: ncclInProgress
// is polled through ncclCommGetAsyncError until it resolves or the deadline passes.
int nccl_settle(int r, void* comm, Clock::time_point deadline) {
    while (r == kNcclInProgress) {
        if (Clock::now() > deadline) return kNcclInProgress;
        std::this_thread::sleep_for(std::chrono::microseconds(20));
        int ae = kNcclInProgress;
        if (g_nccl.async_error(comm, &ae) != kNcclSuccess) return kNcclInProgress;
        r = ae;
    }
    return r;
}

// Waits (bounded by the handle's collective timeout) until every operation this
// call queued on `st` has finished, watching the communicator's asynchronous
// error.  A peer that stopped taking part leaves the NCCL kernels waiting; at
// the deadline the communicator is aborted (ncclCommAbort ends its kernels) and
// ZS_ERR_NCCL returned, so the caller never blocks for good.
zs_status wait_collectives(zs_context* h, void* comm, cudaStream_t st, Clock::time_point t0) {
    if (h->coll_timeout_ms <= 0) return ZS_OK;
    if (!h->coll_event) ZS_CUDA(cudaEventCreateWithFlags(&h->coll_event, cudaEventDisableTiming));
    ZS_CUDA(cudaEventRecord(h->coll_event, st));
    const Clock::time_point deadline = t0 + std::chrono::milliseconds(h->coll_timeout_ms);
    for (;;) {
        const cudaError_t q = cudaEventQuery(h->coll_event);
        if (q == cudaSuccess) return ZS_OK;
        if (q != cudaErrorNotReady) return cuda_fail(q, "waiting for the sharded step");
        int ae = kNcclSuccess;
        const int qr = g_nccl.async_error(comm, &ae);
        const bool failed = qr != kNcclSuccess || (ae != kNcclSuccess && ae != kNcclInProgress);
        const bool late = Clock::now() > deadline;
        if (failed || late) {
            g_nccl.abort(comm);
            // the aborted kernels return; give the stream a bounded time to drain
            const Clock::time_point drain = Clock::now() + std::chrono::seconds(10);
            while (cudaEventQuery(h->coll_event) == cudaErrorNotReady && Clock::now() < drain)
                std::this_thread::sleep_for(std::chrono::microseconds(200));
            const std::string why =
                failed ? nccl_msg("NCCL reported an asynchronous error", qr != kNcclSuccess ? qr : ae)
                       : "the sharded step did not finish within " +
                             std::to_string(h->coll_timeout_ms) + " ms (a rank stopped taking part?)";
            return fail(ZS_ERR_NCCL, why + "; the communicator was aborted and must not be used again");
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

}  // namespace

extern "C" {

int zs_abi_version(void) { return ZS_ABI_VERSION; }

const char* zs_last_error(void) { return g_last_error.c_str(); }

const char* zs_status_string(zs_status s) {
    switch (s) {
        case ZS_OK: return "ok";
        case ZS_ERR_INVALID_ARGUMENT: return "invalid argument";
        case ZS_ERR_CUDA: return "CUDA error";
        case ZS_ERR_NO_DEVICE: return "no sm_100 device";
        case ZS_ERR_DEVICE_TIMEOUT: return "device wait timed out";
        case ZS_ERR_NCCL: return "NCCL error";
        case ZS_ERR_OUT_OF_MEMORY: return "out of device memory";
    }
    return "unknown status";
}

uint64_t zs_rng_seed(uint64_t seed) { return seed ? seed : 0x9E3779B97F4A7C15ull; }

zs_status zs_create(int device, zs_handle* out) {
    if (!out) return fail(ZS_ERR_INVALID_ARGUMENT, "out is null");
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0)
        return fail(ZS_ERR_NO_DEVICE, "no CUDA device visible");
    if (device < 0 || device >= n) return fail(ZS_ERR_INVALID_ARGUMENT, "device out of range");
    cudaDeviceProp prop;
    ZS_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) return fail(ZS_ERR_NO_DEVICE, std::string("not an sm_100 device: ") + prop.name);
    DeviceGuard g(device);
    if (!g.ok) return fail(ZS_ERR_CUDA, "cudaSetDevice failed");
    zs_context* h = new zs_context();
    h->device = device;
    h->num_sms = prop.multiProcessorCount;
    h->select_smem = sizeof(zs::FastSmem);
    h->merge_smem = sizeof(zs::CandState);
    h->warp_merge_smem = sizeof(zs::WarpMergeSmem);
    auto cleanup = [&](zs_status s) {
        delete h;
        return s;
    };
    cudaError_t e;
    if ((e = cudaFuncSetAttribute(zs::zs_select_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)h->select_smem)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(zs::zs_select_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)h->select_smem)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(zs::zs_merge_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)h->merge_smem)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(zs::zs_merge_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)h->merge_smem)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(zs::zs_large_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)h->merge_smem)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(zs::zs_large_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)h->merge_smem)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(zs::zs_warp_merge_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)h->warp_merge_smem)) != cudaSuccess ||
        (e = cudaFuncSetAttribute(zs::zs_warp_merge_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)h->warp_merge_smem)) != cudaSuccess)
        return cleanup(cuda_fail(e, "cudaFuncSetAttribute"));
    if ((size_t)prop.sharedMemPerBlockOptin >= zs::kLmSmemBytes &&
        ((e = cudaFuncSetAttribute(zs::zs_lmhead_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)zs::kLmSmemBytes)) != cudaSuccess ||
         (e = cudaFuncSetAttribute(zs::zs_lmhead_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)zs::kLmSmemBytes)) != cudaSuccess))
        return cleanup(cuda_fail(e, "cudaFuncSetAttribute zs_lmhead_kernel"));
    if ((size_t)prop.sharedMemPerBlockOptin >= zs::ex_smem_bytes(1, zs::kExMaxElems) &&
        (e = cudaFuncSetAttribute(zs::zs_lm_exact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)zs::ex_smem_bytes(1, zs::kExMaxElems))) != cudaSuccess)
        return cleanup(cuda_fail(e, "cudaFuncSetAttribute zs_lm_exact_kernel"));
    // CTA pairs of the lm_head kernel that can be resident at once (0: none; the
    // one-CTA tiles are used then).
    h->lm_pairs = 0;
    if ((size_t)prop.sharedMemPerBlockOptin >= zs::kLmSmemBytes) {
        cudaLaunchConfig_t cfg;
        std::memset(&cfg, 0, sizeof(cfg));
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.gridDim = dim3(2 * (h->num_sms / 2));
        cfg.blockDim = dim3(zs::kLmThreads);
        cfg.dynamicSmemBytes = zs::kLmSmemBytes;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, zs::zs_lmhead_kernel<2>, &cfg) == cudaSuccess)
            h->lm_pairs = std::min(n, h->num_sms / 2);
        (void)cudaGetLastError();
    }
    zs_status sw = setup_wselect<zs::WCfgS>(&h->wsel_smem[0], &h->wsel_warps[0], h->num_sms);
    if (sw == ZS_OK) sw = setup_wselect<zs::WCfgL>(&h->wsel_smem[1], &h->wsel_warps[1], h->num_sms);
    if (sw != ZS_OK) return cleanup(sw);
    // The one-launch small-batch path needs clusters of zs::kSmallCl CTAs (a
    // non-portable size); where they cannot be resident the path stays off.
    h->small_clusters = 0;
    if (cudaFuncSetAttribute(zs::zs_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)sizeof(zs::SmallSmem)) == cudaSuccess &&
        cudaFuncSetAttribute(zs::zs_small_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed,
                             1) == cudaSuccess) {
        cudaLaunchAttribute cattr[1];
        cattr[0].id = cudaLaunchAttributeClusterDimension;
        cattr[0].val.clusterDim.x = zs::kSmallCl;
        cattr[0].val.clusterDim.y = 1;
        cattr[0].val.clusterDim.z = 1;
        cudaLaunchConfig_t ccfg;
        std::memset(&ccfg, 0, sizeof(ccfg));
        ccfg.gridDim = dim3(zs::kSmallCl);
        ccfg.blockDim = dim3(zs::kNC);
        ccfg.dynamicSmemBytes = sizeof(zs::SmallSmem);
        ccfg.attrs = cattr;
        ccfg.numAttrs = 1;
        int nc = 0;
        if (cudaOccupancyMaxActiveClusters(&nc, zs::zs_small_kernel, &ccfg) == cudaSuccess)
            h->small_clusters = nc;
    }
    (void)cudaGetLastError();  // a refused cluster size only turns the path off
    int per_sm = 0;
    if ((e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, zs::zs_select_kernel<false>, zs::kThreads, h->select_smem)) != cudaSuccess)
        return cleanup(cuda_fail(e, "occupancy query"));
    h->select_ctas_per_sm = std::max(1, per_sm);
    h->select_ctas = h->select_ctas_per_sm * h->num_sms;
    if ((e = cudaMalloc((void**)&h->status, sizeof(int))) != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc status"));
    if ((e = cudaMemset(h->status, 0, sizeof(int))) != cudaSuccess) return cleanup(cuda_fail(e, "cudaMemset status"));
    if ((e = cudaMalloc((void**)&h->fail_count, sizeof(unsigned))) != cudaSuccess) return cleanup(cuda_fail(e, "cudaMalloc fail_count"));
    if ((e = cudaMemset(h->fail_count, 0, sizeof(unsigned))) != cudaSuccess) return cleanup(cuda_fail(e, "cudaMemset fail_count"));
    *out = h;
    return ZS_OK;
}

zs_status zs_destroy(zs_handle h) {
    if (!h) return ZS_OK;
    DeviceGuard g(h->device);
    cudaFree(h->part);
    cudaFree(h->status);
    cudaFree(h->params);
    cudaFree(h->large);
    cudaFree(h->spec);
    cudaFree(h->gather);
    cudaFree(h->fail_count);
    cudaFree(h->fail_units);
    cudaFree(h->stats_rng);
    cudaFree(h->stats_ids);
    cudaFree(h->stats_part);
    cudaFree(h->rng_prev);
    cudaFree(h->lm_xn);
    cudaFree(h->lm_logits);
    for (auto& t : h->timed) {
        cudaEventDestroy(t.begin);
        cudaEventDestroy(t.end);
    }
    for (cudaEvent_t ev : h->spare) cudaEventDestroy(ev);
    if (h->coll_event) cudaEventDestroy(h->coll_event);
    delete h;
    return ZS_OK;
}

zs_status zs_set_collective_timeout(zs_handle h, int32_t timeout_ms) {
    if (!h) return fail(ZS_ERR_INVALID_ARGUMENT, "null handle");
    if (timeout_ms < 0) return fail(ZS_ERR_INVALID_ARGUMENT, "timeout_ms < 0");
    h->coll_timeout_ms = timeout_ms;
    return ZS_OK;
}

zs_status zs_set_timing(zs_handle h, int32_t enable) {
    if (!h) return fail(ZS_ERR_INVALID_ARGUMENT, "null handle");
    h->timing = enable != 0;
    return ZS_OK;
}

zs_status zs_set_small_batch(zs_handle h, int32_t max_rows) {
    if (!h) return fail(ZS_ERR_INVALID_ARGUMENT, "null handle");
    if (max_rows < 0) return fail(ZS_ERR_INVALID_ARGUMENT, "max_rows < 0");
    h->small_max_rows = max_rows;
    return ZS_OK;
}

zs_status zs_set_speculation(zs_handle h, int32_t mode) {
    if (!h) return fail(ZS_ERR_INVALID_ARGUMENT, "null handle");
    if (mode != ZS_SPECULATION_OFF && mode != ZS_SPECULATION_ON && mode != ZS_SPECULATION_REDO_ALL)
        return fail(ZS_ERR_INVALID_ARGUMENT, "unknown speculation mode");
    h->spec_mode = mode;
    return ZS_OK;
}

zs_status zs_set_lmhead_route(zs_handle h, int32_t route) {
    if (!h) return fail(ZS_ERR_INVALID_ARGUMENT, "null handle");
    if (route != ZS_LMHEAD_ROUTE_AUTO && route != ZS_LMHEAD_ROUTE_FUSED &&
        route != ZS_LMHEAD_ROUTE_TWO_PASS && route != ZS_LMHEAD_ROUTE_EXACT)
        return fail(ZS_ERR_INVALID_ARGUMENT,
                    "route must be ZS_LMHEAD_ROUTE_AUTO, _FUSED, _TWO_PASS or _EXACT");
    h->lm_route = route;
    return ZS_OK;
}

zs_status zs_set_lmhead_tiles(zs_handle h, int32_t mode) {
    if (!h) return fail(ZS_ERR_INVALID_ARGUMENT, "null handle");
    if (mode != ZS_LMHEAD_TILES_AUTO && mode != ZS_LMHEAD_TILES_SINGLE &&
        mode != ZS_LMHEAD_TILES_PAIR)
        return fail(ZS_ERR_INVALID_ARGUMENT,
                    "mode must be ZS_LMHEAD_TILES_AUTO, _SINGLE or _PAIR");
    h->lm_tiles = mode;
    return ZS_OK;
}

zs_status zs_get_timing(zs_handle h, zs_timing* out) {
    if (!h || !out) return fail(ZS_ERR_INVALID_ARGUMENT, "null handle or out");
    DeviceGuard g(h->device);
    std::memset(out, 0, sizeof(*out));
    double* dst[5] = {&out->select_ms, &out->merge_ms, &out->large_ms, &out->lmhead_ms,
                      &out->lmnorm_ms};
    int64_t* cnt[5] = {&out->select_launches, &out->merge_launches, &out->large_launches,
                       &out->lmhead_launches, &out->lmnorm_launches};
    zs_status s = ZS_OK;
    for (auto& t : h->timed) {
        float ms = 0.0f;
        cudaError_t e = cudaEventSynchronize(t.end);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, t.begin, t.end);
        if (e != cudaSuccess && s == ZS_OK) s = cuda_fail(e, "timing events");
        *dst[t.kind] += ms;
        *cnt[t.kind] += 1;
        h->spare.push_back(t.begin);
        h->spare.push_back(t.end);
    }
    h->timed.clear();
    out->launches = h->launches;
    h->launches = 0;
    return s;
}

zs_status zs_sample(zs_handle h, const float* logits, int64_t ld, int32_t batch, int32_t n_vocab,
                    const zs_params* params, int32_t params_per_row, const int32_t* history,
                    int64_t history_ld, const int32_t* history_len, uint64_t* rng_state,
                    int32_t* out_ids, const zs_extras* extras, void* stream) {
    NvtxRange nvtx_range("zs_sample");
    zs_status s = validate_common(h, logits, ld, batch, n_vocab, params);
    if (s != ZS_OK) return s;
    if (batch == 0) return ZS_OK;
    if (!out_ids) return fail(ZS_ERR_INVALID_ARGUMENT, "out_ids is null");
    cudaStream_t st = (cudaStream_t)stream;
    DeviceGuard g(h->device);
    if (!g.ok) return fail(ZS_ERR_CUDA, "cudaSetDevice failed");
    if (n_vocab <= 0) {  // sample.cpp:34 -- returns 0 before touching the Rng
        ZS_CUDA(cudaMemsetAsync(out_ids, 0, (size_t)batch * sizeof(int32_t), st));
        return ZS_OK;
    }
    if (!rng_state && needs_rng(params, params_per_row, batch))
        return fail(ZS_ERR_INVALID_ARGUMENT, "rng_state is null");
    const bool have_hist = history && history_len;
    if (have_hist && history_ld < 0) return fail(ZS_ERR_INVALID_ARGUMENT, "history_ld < 0");
    const zs::Params* dparams = nullptr;
    s = upload_params(h, params, params_per_row, batch, st, &dparams);
    if (s != ZS_OK) return s;
    const Plan pl = make_plan(batch, n_vocab, n_vocab, params, params_per_row, h->select_ctas,
                              h->wsel_warps, have_hist);
    zs::Args a;
    std::memset(&a, 0, sizeof(a));
    a.logits = logits;
    a.ld = ld;
    a.B = batch;
    a.V = n_vocab;
    a.id_offset = 0;
    a.V_total = n_vocab;
    a.shared = to_dev(params[0]);
    a.row_params = dparams;
    a.hist = have_hist ? history : nullptr;
    a.hist_ld = history_ld;
    a.hist_len = have_hist ? history_len : nullptr;
    a.rng = rng_state;
    a.out_ids = out_ids;
    bool want_lse = false;
    if (extras) {
        a.info = reinterpret_cast<zs::RowInfo*>(extras->row_info);
        a.cand_ids = extras->cand_ids;
        a.cand_probs = extras->cand_probs;
        a.cand_ld = (extras->cand_ids || extras->cand_probs) ? extras->cand_ld : 0;
        if (a.cand_ld < 0) return fail(ZS_ERR_INVALID_ARGUMENT, "cand_ld < 0");
        want_lse = extras->want_log_z && extras->row_info;
    }
    a.mode = 0;
    return launch_select(h, a, pl, want_lse, st);
}

zs_status zs_decode_step(zs_handle h, const float* logits, int64_t ld, int32_t batch,
                         int32_t n_vocab, const zs_params* params, int32_t params_per_row,
                         int32_t* history, int64_t history_ld, int32_t* history_len,
                         uint64_t* rng_state, int32_t* done, int32_t eos_id, int32_t* out_ids,
                         int32_t* tokens, int64_t tokens_ld, int64_t step, void* stream) {
    NvtxRange nvtx_range("zs_decode_step");
    zs_status s = validate_common(h, logits, ld, batch, n_vocab, params);
    if (s != ZS_OK) return s;
    if (batch == 0) return ZS_OK;
    if (!done || !out_ids) return fail(ZS_ERR_INVALID_ARGUMENT, "done and out_ids are required");
    if (!rng_state) return fail(ZS_ERR_INVALID_ARGUMENT, "rng_state is required");
    if ((history == nullptr) != (history_len == nullptr))
        return fail(ZS_ERR_INVALID_ARGUMENT, "history and history_len go together");
    if (history) {
        if (history_ld < 1) return fail(ZS_ERR_INVALID_ARGUMENT, "history_ld < 1");
        const int32_t np = params_per_row ? batch : 1;
        for (int32_t i = 0; i < np; ++i)  // a full history keeps the penalty window
            if (params[i].repeat_penalty != 1.0f && params[i].repeat_last_n >= history_ld)
                return fail(ZS_ERR_INVALID_ARGUMENT,
                            "history_ld must exceed repeat_last_n of every penalised row");
    }
    if (tokens && (step < 0 || step >= tokens_ld))
        return fail(ZS_ERR_INVALID_ARGUMENT, "step outside [0, tokens_ld)");
    cudaStream_t st = (cudaStream_t)stream;
    DeviceGuard g(h->device);
    if (!g.ok) return fail(ZS_ERR_CUDA, "cudaSetDevice failed");
    s = grow((void**)&h->rng_prev, &h->rng_prev_bytes, (size_t)batch * sizeof(uint64_t));
    if (s != ZS_OK) return s;
    ZS_CUDA(cudaMemcpyAsync(h->rng_prev, rng_state, (size_t)batch * sizeof(uint64_t),
                            cudaMemcpyDeviceToDevice, st));
    s = zs_sample(h, logits, ld, batch, n_vocab, params, params_per_row, history, history_ld,
                  history_len, rng_state, out_ids, nullptr, stream);
    if (s != ZS_OK) return s;
    zs::DecodeArgs a;
    std::memset(&a, 0, sizeof(a));
    a.B = batch;
    a.eos = eos_id;
    a.rng_prev = h->rng_prev;
    a.rng = rng_state;
    a.done = done;
    a.out_ids = out_ids;
    a.hist = history;
    a.hist_ld = history_ld;
    a.hist_len = history_len;
    a.row_params = params_per_row ? h->params : nullptr;  // uploaded by zs_sample
    a.shared = to_dev(params[0]);
    a.tokens = tokens;
    a.tokens_ld = tokens_ld;
    a.step = step;
    zs::zs_decode_append_kernel<<<(batch + 127) / 128, 128, 0, st>>>(a);
    ZS_CUDA(cudaGetLastError());
    h->launches += 1;
    return ZS_OK;
}

namespace {

// A 2-D tensor map over rows x cols (row-major, cols contiguous, rows `ld` elements
// apart) with 128-byte swizzle: bf16 boxes of 128 rows x 64 columns, as
// zs_lmhead_kernel reads its operands, or (f32) boxes of 32 x 32, as it stores logits.
zs_status lm_tensor_map(zs_context* h, CUtensorMap* map, const void* base, int64_t rows,
                        int64_t cols, bool f32 = false, int64_t ld = 0) {
    if (!h->encode_tiled) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                                         cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
            return fail(ZS_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
        h->encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    const int64_t esize = f32 ? 4 : 2;
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(ld > 0 ? ld : cols) * esize};
    const cuuint32_t box[2] = {f32 ? 32u : (cuuint32_t)zs::kLmBK, f32 ? 16u : (cuuint32_t)zs::kLmM};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = h->encode_tiled(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                                       2, const_cast<void*>(base),
                                       dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                       CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return fail(ZS_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
    return ZS_OK;
}

// Slices per row for mt row tiles x nt column tiles on `ctas` CTAs: the fewest
// slices (at most `cap`) whose busiest CTA has at most 2% more tiles than the best
// split.
// Tiles of one CTA (128 rows x 128 columns) or of a CTA pair (256 x 256): pairs
// halve the operand traffic per product, so they are the default from 512 rows up
// (measured on B200, fused route, 151,936 x 896: 289 against 292 us at 512 rows,
// 226 against 208 us at 256, where one pair tile holds all rows and the epilogue
// sets the pace); zs_set_lmhead_tiles overrides.
int lm_pair_for(const zs_context* h, int batch) {
    if (h->lm_pairs <= 0 || h->lm_tiles == ZS_LMHEAD_TILES_SINGLE) return 1;
    if (h->lm_tiles == ZS_LMHEAD_TILES_PAIR) return 2;
    return batch >= 4 * zs::kLmM ? 2 : 1;
}

int lm_slices(int mt, int nt, int ctas, int cap);

// Sets a.pair, the row and column tile counts, the slices per row tile (at most
// `cap`) and the units of a batch.
void lm_geometry(const zs_context* h, zs::LmArgs& a, int batch, int n_vocab, int cap) {
    a.pair = lm_pair_for(h, batch);
    const int rows = zs::kLmM * a.pair, cols = zs::kLmN * a.pair;
    a.mt = (batch + rows - 1) / rows;
    a.nt = (n_vocab + cols - 1) / cols;
    a.S = lm_slices(a.mt, a.nt, a.pair == 2 ? h->lm_pairs : h->num_sms, cap);
    a.n_units = a.mt * a.S;
}

int lm_slices(int mt, int nt, int ctas, int cap) {
    auto span = [&](int S) {
        const int64_t units = (int64_t)mt * S;
        return ((units + ctas - 1) / ctas) * (int64_t)((nt + S - 1) / S);
    };
    const int smax = std::max(1, std::min(std::min(nt, 1024), cap));
    int64_t best = span(1);
    for (int S = 2; S <= smax; ++S) best = std::min(best, span(S));
    for (int S = 1; S <= smax; ++S)
        if (span(S) * 100 <= best * 102) return S;
    return 1;
}

}  // namespace

namespace {

constexpr int32_t kLmTwoPassMaxRows = 1023;

// Checks shared by the lm_head entry points.
zs_status lm_validate(zs_handle h, const float* hidden, int64_t hidden_ld, const float* norm_w,
                      const void* weight, int32_t n_embd, int32_t n_vocab, const float* out_logits,
                      int64_t logits_ld) {
    if (!hidden || !norm_w || !weight)
        return fail(ZS_ERR_INVALID_ARGUMENT, "hidden, norm_w and weight are required");
    if (n_vocab < 1) return fail(ZS_ERR_INVALID_ARGUMENT, "n_vocab < 1");
    if (n_embd < zs::kLmBK || n_embd % 8 != 0 || n_embd > 12288)
        return fail(ZS_ERR_INVALID_ARGUMENT, "n_embd must be a multiple of 8 from 64 to 12288");
    if (hidden_ld < n_embd) return fail(ZS_ERR_INVALID_ARGUMENT, "hidden_ld < n_embd");
    if (((uintptr_t)weight & 15u) != 0) return fail(ZS_ERR_INVALID_ARGUMENT, "weight not 16-byte aligned");
    if (((uintptr_t)hidden & 3u) != 0 || ((uintptr_t)norm_w & 3u) != 0)
        return fail(ZS_ERR_INVALID_ARGUMENT, "hidden or norm_w not 4-byte aligned");
    if (out_logits && (logits_ld < n_vocab || ((uintptr_t)out_logits & 15u) != 0 || logits_ld % 4 != 0))
        return fail(ZS_ERR_INVALID_ARGUMENT,
                    "out_logits needs logits_ld >= n_vocab, a multiple of 4, 16-byte alignment");
    if (zs::kLmSmemBytes > 232448) return fail(ZS_ERR_NO_DEVICE, "lm_head tiles do not fit");
    return ZS_OK;
}

// rmsnorm into the handle's bf16 rows, then zs_lmhead_kernel over `a` (whose B, E,
// V, S, select, parameters and outputs the caller has set).
zs_status lm_run(zs_context* h, const float* hidden, int64_t hidden_ld, const float* norm_w,
                 float eps, const void* weight, zs::LmArgs& a, cudaStream_t st) {
    zs_status s = grow((void**)&h->lm_xn, &h->lm_xn_bytes, (size_t)a.B * a.E * 2);
    if (s != ZS_OK) return s;
    CUtensorMap tm_a, tm_b, tm_c;
    s = lm_tensor_map(h, &tm_a, h->lm_xn, a.B, a.E);
    if (s == ZS_OK) s = lm_tensor_map(h, &tm_b, weight, a.V, a.E);
    if (s != ZS_OK) return s;
    // logits only: the epilogue stores 32 x 32 tiles by TMA (its candidate buffers
    // are free); below 64 rows most of each tile is outside the batch and direct
    // stores of the live rows are cheaper.  Otherwise tm_c is not used.
    a.tma_out = (!a.select && a.out_logits && a.B >= 64) ? 1 : 0;
    if (a.tma_out) {
        s = lm_tensor_map(h, &tm_c, a.out_logits, a.B, a.V, true, a.logits_ld);
        if (s != ZS_OK) return s;
    } else {
        tm_c = tm_a;
    }
    // Ring depth: the candidate buffers (or the logits staging) of the rows in use
    // sit behind the ring, so a batch within one warp's 32 rows (or logits stored
    // directly) leaves room for more weight tiles in flight.
    {
        const int64_t rows_in_use =
            (a.select || a.tma_out)
                ? (a.mt > 1 || a.tma_out ? zs::kLmM
                                         : std::min<int64_t>(zs::kLmM, ((int64_t)a.B + 31) / 32 * 32))
                : 0;
        a.ns = zs::kLmStages;
        for (int n = zs::kLmStagesMax; n > zs::kLmStages; --n)
            if ((int64_t)n * zs::kLmStageBytes + rows_in_use * zs::kLmRowBytes <= (int64_t)zs::kLmRingBytes) {
                a.ns = n;
                break;
            }
    }
    a.status = h->status;
    {
        LaunchScope scope(h, 4, st);
        // warps per CTA: as many rows as fit 48 KB of staged floats, at most 8
        const int nw = (int)std::max<int64_t>(1, std::min<int64_t>(8, (48 << 10) / ((int64_t)a.E * 4)));
        const size_t smem = (size_t)nw * a.E * sizeof(float);
        const int grid = (int)std::min<int64_t>((a.B + nw - 1) / nw, (int64_t)h->num_sms * 16);
        zs::zs_lm_rmsnorm_kernel<<<grid, nw * 32, smem, st>>>(
            hidden, hidden_ld, norm_w, eps, a.B, a.E, reinterpret_cast<__nv_bfloat16*>(h->lm_xn),
            a.tau);
        ZS_CUDA(cudaGetLastError());
    }
    {
        LaunchScope scope(h, 3, st);
        // one CTA per SM, or one CTA pair per two SMs (clusters of two)
        const int grid = a.pair == 2 ? 2 * std::min(a.n_units, h->lm_pairs)
                                     : std::min(a.n_units, h->num_sms);
        // One row tile streams the weights once: while the rmsnorm runs, each CTA
        // prefetches its first weight boxes, about 80 MB in all (within the L2).
        a.prefetch = a.mt == 1 ? (int)((80ll << 20) / zs::kLmTileBBytes / grid) : 0;
        cudaLaunchAttribute attr[2];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = 2;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        cudaLaunchConfig_t cfg;
        std::memset(&cfg, 0, sizeof(cfg));
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(zs::kLmThreads);
        cfg.dynamicSmemBytes = zs::kLmSmemBytes;
        cfg.stream = st;
        cfg.attrs = attr;
        cfg.numAttrs = a.pair == 2 ? 2 : 1;
        if (a.pair == 2)
            ZS_CUDA(cudaLaunchKernelEx(&cfg, zs::zs_lmhead_kernel<2>, tm_a, tm_b, tm_c, a));
        else
            ZS_CUDA(cudaLaunchKernelEx(&cfg, zs::zs_lmhead_kernel<1>, tm_a, tm_b, tm_c, a));
    }
    return ZS_OK;
}

// The exact route: zs_lm_exact_kernel writes f32 logits [batch][lld] computed in the
// reference's own summation order; one CTA per SM streams its share of the vocabulary.
bool lm_exact_fits(int batch, int n_embd) {
    return batch <= zs::kExMaxRows && n_embd <= zs::kExMaxE &&
           (int64_t)batch * n_embd <= zs::kExMaxElems;
}

bool lm_take_exact(const zs_context* h, int batch, int n_embd) {
    return h->lm_route == ZS_LMHEAD_ROUTE_EXACT ||
           (h->lm_route == ZS_LMHEAD_ROUTE_AUTO && lm_exact_fits(batch, n_embd));
}

zs_status lm_exact_run(zs_context* h, const float* hidden, int64_t hidden_ld, const float* norm_w,
                       float eps, const void* weight, int batch, int n_embd, int n_vocab,
                       float* logits, int64_t lld, cudaStream_t st) {
    if (!lm_exact_fits(batch, n_embd))
        return fail(ZS_ERR_INVALID_ARGUMENT,
                    "the exact lm_head route holds up to 8 rows, hidden sizes up to 2048 and "
                    "rows x hidden size up to 8192");
    zs::ExArgs a;
    std::memset(&a, 0, sizeof(a));
    a.hidden = hidden;
    a.hld = hidden_ld;
    a.norm_w = norm_w;
    a.eps = eps;
    a.B = batch;
    a.E = n_embd;
    a.V = n_vocab;
    a.w = reinterpret_cast<const uint16_t*>(weight);
    a.out = logits;
    a.lld = lld;
    a.rows_per_stage = std::max(1, std::min<int>(zs::kExMaxStageRows,
                                                 (int)(zs::kExStageBytes / zs::ex_row_stride(n_embd))));
    // about 96 MB of the weights (within the L2) prefetched while the rows' sums run
    a.prefetch_bytes = (96ll << 20) / h->num_sms;
    a.status = h->status;
    LaunchScope scope(h, 3, st);
    zs::zs_lm_exact_kernel<<<h->num_sms, zs::kExThreads, zs::ex_smem_bytes(batch, n_embd), st>>>(a);
    ZS_CUDA(cudaGetLastError());
    return ZS_OK;
}

}  // namespace

zs_status zs_lmhead_logits(zs_handle h, const float* hidden, int64_t hidden_ld,
                           const float* norm_w, float eps, const void* weight, int32_t batch,
                           int32_t n_embd, int32_t n_vocab, float* out_logits, int64_t logits_ld,
                           void* stream) {
    NvtxRange nvtx_range("zs_lmhead_logits");
    if (!h) return fail(ZS_ERR_INVALID_ARGUMENT, "null handle");
    if (batch < 0) return fail(ZS_ERR_INVALID_ARGUMENT, "batch < 0");
    if (batch == 0) return ZS_OK;
    if (!out_logits) return fail(ZS_ERR_INVALID_ARGUMENT, "out_logits is required");
    zs_status s = lm_validate(h, hidden, hidden_ld, norm_w, weight, n_embd, n_vocab, out_logits,
                              logits_ld);
    if (s != ZS_OK) return s;
    DeviceGuard g(h->device);
    if (!g.ok) return fail(ZS_ERR_CUDA, "cudaSetDevice failed");
    if (lm_take_exact(h, batch, n_embd))
        return lm_exact_run(h, hidden, hidden_ld, norm_w, eps, weight, batch, n_embd, n_vocab,
                            out_logits, logits_ld, (cudaStream_t)stream);
    zs::LmArgs a;
    std::memset(&a, 0, sizeof(a));
    a.B = batch;
    a.E = n_embd;
    a.V = n_vocab;
    a.V_total = n_vocab;
    lm_geometry(h, a, batch, n_vocab, 1024);
    a.select = 0;
    a.out_logits = out_logits;
    a.logits_ld = logits_ld;
    return lm_run(h, hidden, hidden_ld, norm_w, eps, weight, a, (cudaStream_t)stream);
}

zs_status zs_lmhead_sample(zs_handle h, const float* hidden, int64_t hidden_ld,
                           const float* norm_w, float eps, const void* weight, int32_t batch,
                           int32_t n_embd, int32_t n_vocab, const zs_params* params,
                           int32_t params_per_row, const int32_t* history, int64_t history_ld,
                           const int32_t* history_len, uint64_t* rng_state, int32_t* out_ids,
                           float* out_logits, int64_t logits_ld, void* stream) {
    NvtxRange nvtx_range("zs_lmhead_sample");
    if (!h) return fail(ZS_ERR_INVALID_ARGUMENT, "null handle");
    if (!params) return fail(ZS_ERR_INVALID_ARGUMENT, "params is null");
    if (batch < 0) return fail(ZS_ERR_INVALID_ARGUMENT, "batch < 0");
    if (batch == 0) return ZS_OK;
    if (!out_ids) return fail(ZS_ERR_INVALID_ARGUMENT, "out_ids is required");
    zs_status s = lm_validate(h, hidden, hidden_ld, norm_w, weight, n_embd, n_vocab, out_logits,
                              logits_ld);
    if (s != ZS_OK) return s;
    if (!rng_state && needs_rng(params, params_per_row, batch))
        return fail(ZS_ERR_INVALID_ARGUMENT, "rng_state is null");
    const bool have_hist = history && history_len;
    cudaStream_t st = (cudaStream_t)stream;
    DeviceGuard g(h->device);
    if (!g.ok) return fail(ZS_ERR_CUDA, "cudaSetDevice failed");

    // Up to kExMaxRows rows (and by choice): the logits in f32, exactly as the
    // reference computes them, then zs_sample on them.
    if (lm_take_exact(h, batch, n_embd)) {
        float* lg = out_logits;
        int64_t ld = logits_ld;
        if (!lg) {
            ld = ((int64_t)n_vocab + 3) & ~(int64_t)3;
            s = grow((void**)&h->lm_logits, &h->lm_logits_bytes, (size_t)batch * ld * sizeof(float));
            if (s != ZS_OK) return s;
            lg = reinterpret_cast<float*>(h->lm_logits);
        }
        s = lm_exact_run(h, hidden, hidden_ld, norm_w, eps, weight, batch, n_embd, n_vocab, lg, ld,
                         st);
        if (s != ZS_OK) return s;
        return zs_sample(h, lg, ld, batch, n_vocab, params, params_per_row, history, history_ld,
                         history_len, rng_state, out_ids, nullptr, stream);
    }
    // Route: the fused epilogue holds up to kLmKeffMax keys per row and no penalty
    // window; otherwise the kernel writes the logits and zs_sample takes over.
    const int np = params_per_row ? batch : 1;
    int max_ksel = 1;
    bool fused = true;
    for (int i = 0; i < np; ++i) {
        const zs_params& p = params[i];
        int ks = 1;
        if (!(p.temp <= 0.0f)) ks = p.top_k > 0 ? std::min(p.top_k, n_vocab) : std::min(zs::kShortlistDefault, n_vocab);
        max_ksel = std::max(max_ksel, ks);
        if (ks > zs::kLmKeffMax) fused = false;
        if (have_hist && p.repeat_penalty != 1.0f && p.repeat_last_n > 0) fused = false;
    }
    // Up to kLmTwoPassMaxRows rows the two passes are faster (measured on B200, 151,936
    // x 896 weights, top-k 50: 298 against 379 us at 512 rows, 229 against 280 at 256;
    // fused 479 against 493 us at 1024): with few row tiles each row's selection sees
    // short runs of columns, over which its threshold ramps up from nothing.
    if (h->lm_route == ZS_LMHEAD_ROUTE_TWO_PASS ||
        (h->lm_route == ZS_LMHEAD_ROUTE_AUTO && batch <= kLmTwoPassMaxRows))
        fused = false;

    float* logits = out_logits;
    int64_t lld = logits_ld;
    if (!fused && !logits) {
        lld = ((int64_t)n_vocab + 3) & ~(int64_t)3;
        s = grow((void**)&h->lm_logits, &h->lm_logits_bytes, (size_t)batch * lld * sizeof(float));
        if (s != ZS_OK) return s;
        logits = reinterpret_cast<float*>(h->lm_logits);
    }
    zs::LmArgs a;
    std::memset(&a, 0, sizeof(a));
    a.B = batch;
    a.E = n_embd;
    a.V = n_vocab;
    a.V_total = n_vocab;

    // a row's S blocks of up to max_ksel keys stay within the merge's one-pass gather
    const int s_cap = fused ? std::min(zs::kNC, (zs::kCandCap - zs::kCandMargin) / max_ksel) : 1024;
    lm_geometry(h, a, batch, n_vocab, s_cap);
    a.select = fused ? 1 : 0;
    a.shared = to_dev(params[0]);
    const zs::Params* dparams = nullptr;
    s = upload_params(h, params, params_per_row, batch, st, &dparams);
    if (s != ZS_OK) return s;
    a.row_params = dparams;
    a.out_logits = logits;
    a.logits_ld = lld;
    if (fused) {
        // the blocks, then (more than one slice) a value order per row that the
        // row's slices share as a lower bound for their thresholds
        const size_t blocks = (size_t)batch * a.S * zs::kLmPartStride;
        s = grow((void**)&h->part, &h->part_bytes, blocks + (size_t)batch * sizeof(uint32_t));
        if (s != ZS_OK) return s;
        a.part = h->part;
        if (a.S > 1) a.tau = reinterpret_cast<uint32_t*>(h->part + blocks);
    }
    s = lm_run(h, hidden, hidden_ld, norm_w, eps, weight, a, st);
    if (s != ZS_OK) return s;
    if (!fused)
        return zs_sample(h, logits, lld, batch, n_vocab, params, params_per_row, history,
                         history_ld, history_len, rng_state, out_ids, nullptr, stream);
    zs::MergeArgs m;
    std::memset(&m, 0, sizeof(m));
    m.gathered = h->part;
    m.rank_stride = 0;
    m.G = 1;
    m.S = a.S;
    m.part_stride = zs::kLmPartStride;
    m.B = batch;
    m.row0 = 0;
    m.row1 = batch;
    m.V_total = n_vocab;
    m.shared = a.shared;
    m.row_params = dparams;
    m.rng = rng_state;
    m.out_ids = out_ids;
    m.status = h->status;
    m.force_slices = 1;
    return launch_merge(h, m, max_ksel, false, st);
}

zs_status zs_argmax(zs_handle h, const float* logits, int64_t ld, int32_t batch, int32_t n_vocab,
                    int32_t* out_ids, void* stream) {
    NvtxRange nvtx_range("zs_argmax");
    zs_params p;
    p.temp = 0.0f;
    p.top_k = 0;
    p.top_p = 1.0f;
    p.repeat_penalty = 1.0f;
    p.repeat_last_n = 64;
    return zs_sample(h, logits, ld, batch, n_vocab, &p, 0, nullptr, 0, nullptr, nullptr, out_ids,
                     nullptr, stream);
}

zs_status zs_check_device_status(zs_handle h, void* stream) {
    if (!h) return fail(ZS_ERR_INVALID_ARGUMENT, "null handle");
    DeviceGuard g(h->device);
    int v = 0;
    ZS_CUDA(cudaMemcpyAsync(&v, h->status, sizeof(int), cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    ZS_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    if (v != 0) {
        ZS_CUDA(cudaMemset(h->status, 0, sizeof(int)));
        return fail(ZS_ERR_DEVICE_TIMEOUT, "a sampler kernel gave up on a bounded wait");
    }
    return ZS_OK;
}

zs_status zs_selftest_wait_timeout(zs_handle h, void* stream) {
    if (!h) return fail(ZS_ERR_INVALID_ARGUMENT, "null handle");
    DeviceGuard g(h->device);
    if (!g.ok) return fail(ZS_ERR_CUDA, "cudaSetDevice failed");
    zs::zs_wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(h->status);
    ZS_CUDA(cudaGetLastError());
    return ZS_OK;
}

zs_status zs_logits_stats(zs_handle h, const float* logits, int64_t ld, int32_t batch,
                          int32_t n_vocab, int32_t topn, double* out_min, double* out_max,
                          double* out_z, int32_t* top_ids, double* top_p, void* stream) {
    NvtxRange nvtx_range("zs_logits_stats");
    if (!h) return fail(ZS_ERR_INVALID_ARGUMENT, "null handle");
    if (batch < 0 || topn < 0) return fail(ZS_ERR_INVALID_ARGUMENT, "batch or topn < 0");
    if (batch == 0) return ZS_OK;
    if (n_vocab <= 0) return fail(ZS_ERR_INVALID_ARGUMENT, "n_vocab <= 0");
    if (!logits || !out_min || !out_max || !out_z || !top_ids || !top_p || topn < 1)
        return fail(ZS_ERR_INVALID_ARGUMENT, "null buffer or topn < 1");
    if (((uintptr_t)logits & 3u) != 0) return fail(ZS_ERR_INVALID_ARGUMENT, "logits not 4-byte aligned");
    if (ld < n_vocab) return fail(ZS_ERR_INVALID_ARGUMENT, "ld < n_vocab");
    cudaStream_t st = (cudaStream_t)stream;
    DeviceGuard g(h->device);
    if (!g.ok) return fail(ZS_ERR_CUDA, "cudaSetDevice failed");
    // src/main.cpp:483: k = clamp(topk, 1, n_vocab)
    const int k = std::max(1, std::min(topn, n_vocab));
    zs_status s = grow((void**)&h->stats_rng, &h->stats_rng_bytes, (size_t)batch * 8);
    if (s == ZS_OK) s = grow((void**)&h->stats_ids, &h->stats_ids_bytes, (size_t)batch * 4);
    const int nchunk = (n_vocab + zs::kStatsChunk - 1) / zs::kStatsChunk;
    if (s == ZS_OK)
        s = grow((void**)&h->stats_part, &h->stats_part_bytes, (size_t)batch * nchunk * 16);
    if (s != ZS_OK) return s;
    // The top-k shortlist of a temp-1 call is the top-N in the display order
    // (value descending, then id ascending); its draw goes to scratch.
    ZS_CUDA(cudaMemsetAsync(h->stats_rng, 0, (size_t)batch * 8, st));
    zs_params p;
    p.temp = 1.0f;
    p.top_k = k;
    p.top_p = 1.0f;
    p.repeat_penalty = 1.0f;
    p.repeat_last_n = 0;
    zs_extras ex;
    std::memset(&ex, 0, sizeof(ex));
    ex.cand_ids = top_ids;
    ex.cand_ld = topn;
    s = zs_sample(h, logits, ld, batch, n_vocab, &p, 0, nullptr, 0, nullptr, h->stats_rng,
                  h->stats_ids, &ex, stream);
    if (s != ZS_OK) return s;
    zs::StatsArgs a;
    a.logits = logits;
    a.ld = ld;
    a.B = batch;
    a.n = n_vocab;
    a.nchunk = nchunk;
    a.part_mm = reinterpret_cast<float2*>(h->stats_part);
    a.part_z = reinterpret_cast<double*>(h->stats_part + (size_t)batch * nchunk * 8);
    a.top_ids = top_ids;
    a.topn = k;
    a.top_ld = topn;
    a.out_min = out_min;
    a.out_max = out_max;
    a.out_z = out_z;
    a.top_p = top_p;
    const dim3 grid(nchunk, std::min(batch, 65535));
    zs::zs_stats_minmax_kernel<<<grid, zs::kStatsThreads, 0, st>>>(a);
    ZS_CUDA(cudaGetLastError());
    zs::zs_stats_z_kernel<<<grid, zs::kStatsThreads, 0, st>>>(a);
    ZS_CUDA(cudaGetLastError());
    zs::zs_stats_final_kernel<<<std::min(batch, 65535), 32, 0, st>>>(a);
    ZS_CUDA(cudaGetLastError());
    return ZS_OK;
}

zs_status zs_shard_partial_bytes(int32_t batch, int32_t n_vocab_total, int32_t n_ranks,
                                 const zs_params* params, int32_t params_per_row,
                                 int64_t* out_bytes) {
    if (!out_bytes || !params || batch < 0 || n_vocab_total <= 0 || n_ranks <= 0)
        return fail(ZS_ERR_INVALID_ARGUMENT, "bad shard layout arguments");
    const Plan pl = make_plan(batch, shard_cols(n_vocab_total, n_ranks), n_vocab_total, params,
                              params_per_row, kShardLayoutCtas, kShardLayoutWarps, false, n_ranks);
    *out_bytes = pl.bytes;
    return ZS_OK;
}

zs_status zs_shard_partials(zs_handle h, const float* logits_local, int64_t ld, int32_t batch,
                            int32_t n_local, int32_t vocab_offset, int32_t n_vocab_total,
                            int32_t n_ranks, const zs_params* params, int32_t params_per_row,
                            const int32_t* history, int64_t history_ld,
                            const int32_t* history_len, void* partial_out, int32_t want_log_z,
                            void* stream) {
    NvtxRange nvtx_range("zs_shard_partials");
    zs_status s = validate_common(h, logits_local, ld, batch, n_local, params);
    if (s != ZS_OK) return s;
    if (n_vocab_total <= 0 || n_ranks <= 0 || n_local < 0 || vocab_offset < 0 ||
        (int64_t)vocab_offset + n_local > n_vocab_total)
        return fail(ZS_ERR_INVALID_ARGUMENT, "bad shard geometry");
    if (batch == 0) return ZS_OK;
    if (!partial_out || ((uintptr_t)partial_out & 15u))
        return fail(ZS_ERR_INVALID_ARGUMENT, "partial_out null or not 16-byte aligned");
    cudaStream_t st = (cudaStream_t)stream;
    DeviceGuard g(h->device);
    if (!g.ok) return fail(ZS_ERR_CUDA, "cudaSetDevice failed");
    const bool have_hist = history && history_len;
    const int cols = shard_cols(n_vocab_total, n_ranks);
    if (n_local > cols)
        return fail(ZS_ERR_INVALID_ARGUMENT,
                    "n_local above V / n_ranks + V % n_ranks (the largest equal-slice shard)");
    const zs::Params* dparams = nullptr;
    s = upload_params(h, params, params_per_row, batch, st, &dparams);
    if (s != ZS_OK) return s;
    Plan pl = make_plan(batch, cols, n_vocab_total, params, params_per_row, kShardLayoutCtas,
                        kShardLayoutWarps, have_hist, n_ranks);
    if (pl.any_large)
        return fail(ZS_ERR_INVALID_ARGUMENT, "vocab-sharded sampling needs top_k + repeat window <= 2048");
    // Same S on every rank; this rank's slice length covers its own columns.
    const int per = (std::max(n_local, 1) + pl.S - 1) / pl.S;
    pl.slice = std::max(4, (per + 3) & ~3);
    zs::Args a;
    std::memset(&a, 0, sizeof(a));
    a.logits = logits_local;
    a.ld = ld;
    a.B = batch;
    a.V = std::max(n_local, 0);
    a.id_offset = vocab_offset;
    a.V_total = n_vocab_total;
    a.shared = to_dev(params[0]);
    a.row_params = dparams;
    a.hist = have_hist ? history : nullptr;
    a.hist_ld = history_ld;
    a.hist_len = have_hist ? history_len : nullptr;
    a.mode = 1;
    a.status = h->status;
    // the geometry helpers need a valid base address even for an empty shard
    if (n_local <= 0) a.logits = (const float*)partial_out;
    if (pl.launch_cta) {
        s = ensure_fail_units(h, (int64_t)batch * pl.S);
        if (s != ZS_OK) return s;
    }
    a.fail_count = h->fail_count;
    a.fail_units = h->fail_units;
    return launch_partials(h, a, pl, (uint8_t*)partial_out, want_log_z != 0, st);
}

zs_status zs_shard_owner_rows(int32_t batch, int32_t n_ranks, int32_t rank, int32_t* row_begin,
                              int32_t* row_count) {
    if (!row_begin || !row_count || batch < 0 || n_ranks <= 0 || rank < 0 || rank >= n_ranks)
        return fail(ZS_ERR_INVALID_ARGUMENT, "bad owner-row arguments");
    int r0 = 0, n = 0;
    owner_rows(batch, n_ranks, rank, &r0, &n);
    *row_begin = r0;
    *row_count = n;
    return ZS_OK;
}

zs_status zs_shard_row_spans(int32_t batch, int32_t n_vocab_total, int32_t n_ranks,
                             const zs_params* params, int32_t params_per_row, int32_t row_begin,
                             int32_t row_count, int64_t* spans, int32_t* n_spans) {
    if (!spans || !n_spans || !params || batch < 0 || n_vocab_total <= 0 || n_ranks <= 0 ||
        row_begin < 0 || row_count < 0 || (int64_t)row_begin + row_count > batch)
        return fail(ZS_ERR_INVALID_ARGUMENT, "bad row-span arguments");
    const Plan pl = make_plan(batch, shard_cols(n_vocab_total, n_ranks), n_vocab_total, params,
                              params_per_row, kShardLayoutCtas, kShardLayoutWarps, false, n_ranks);
    int64_t sp[3][2];
    const int k = row_spans(pl, batch, row_begin, row_count, sp);
    for (int i = 0; i < 3; ++i) {
        spans[2 * i] = i < k ? sp[i][0] : 0;
        spans[2 * i + 1] = i < k ? sp[i][1] : 0;
    }
    *n_spans = k;
    return ZS_OK;
}

zs_status zs_shard_merge_rows(zs_handle h, const void* gathered, int32_t n_ranks, int32_t batch,
                              int32_t row_begin, int32_t row_count, int32_t n_vocab_total,
                              const zs_params* params, int32_t params_per_row,
                              uint64_t* rng_state, int32_t* out_ids, const zs_extras* extras,
                              void* stream) {
    NvtxRange nvtx_range("zs_shard_merge_rows");
    if (!h || !params || n_ranks <= 0 || batch < 0 || n_vocab_total <= 0 || row_begin < 0 ||
        row_count < 0 || (int64_t)row_begin + row_count > batch)
        return fail(ZS_ERR_INVALID_ARGUMENT, "bad merge arguments");
    if (batch == 0 || row_count == 0) return ZS_OK;
    if (!gathered || !out_ids) return fail(ZS_ERR_INVALID_ARGUMENT, "null buffer");
    if (!rng_state && needs_rng(params, params_per_row, batch))
        return fail(ZS_ERR_INVALID_ARGUMENT, "rng_state is null");
    cudaStream_t st = (cudaStream_t)stream;
    DeviceGuard g(h->device);
    if (!g.ok) return fail(ZS_ERR_CUDA, "cudaSetDevice failed");
    const zs::Params* dparams = nullptr;
    zs_status s = upload_params(h, params, params_per_row, batch, st, &dparams);
    if (s != ZS_OK) return s;
    const Plan pl = make_plan(batch, shard_cols(n_vocab_total, n_ranks), n_vocab_total, params,
                              params_per_row, kShardLayoutCtas, kShardLayoutWarps, false, n_ranks);
    zs::Args a;
    std::memset(&a, 0, sizeof(a));
    a.B = batch;
    a.V_total = n_vocab_total;
    a.shared = to_dev(params[0]);
    a.row_params = dparams;
    a.rng = rng_state;
    a.out_ids = out_ids;
    a.status = h->status;
    bool want_lse = false;
    if (extras) {
        a.info = reinterpret_cast<zs::RowInfo*>(extras->row_info);
        a.cand_ids = extras->cand_ids;
        a.cand_probs = extras->cand_probs;
        a.cand_ld = (extras->cand_ids || extras->cand_probs) ? extras->cand_ld : 0;
        want_lse = extras->want_log_z && extras->row_info;
    }
    zs::MergeArgs m = merge_args_for(a, pl, (const uint8_t*)gathered, n_ranks, pl.bytes);
    m.row0 = row_begin;
    m.row1 = row_begin + row_count;
    return launch_merge(h, m, pl.max_ksel, want_lse, st);
}

zs_status zs_shard_merge(zs_handle h, const void* gathered, int32_t n_ranks, int32_t batch,
                         int32_t n_vocab_total, const zs_params* params, int32_t params_per_row,
                         uint64_t* rng_state, int32_t* out_ids, const zs_extras* extras,
                         void* stream) {
    return zs_shard_merge_rows(h, gathered, n_ranks, batch, 0, batch, n_vocab_total, params,
                               params_per_row, rng_state, out_ids, extras, stream);
}

zs_status zs_sample_sharded(zs_handle h, const float* logits_local, int64_t ld, int32_t batch,
                            int32_t n_local, int32_t vocab_offset, int32_t n_vocab_total,
                            int32_t n_ranks, const zs_params* params, int32_t params_per_row,
                            const int32_t* history, int64_t history_ld,
                            const int32_t* history_len, uint64_t* rng_state, int32_t* out_ids,
                            const zs_extras* extras, void* nccl_comm, void* stream) {
    NvtxRange nvtx_range("zs_sample_sharded");
    if (!h || !nccl_comm) return fail(ZS_ERR_INVALID_ARGUMENT, "null handle or communicator");
    if (!load_nccl()) return fail(ZS_ERR_NCCL, "libnccl.so.2 not loadable (or too old)");
    const Clock::time_point t0 = Clock::now();
    int64_t bytes = 0;
    zs_status s = zs_shard_partial_bytes(batch, n_vocab_total, n_ranks, params, params_per_row, &bytes);
    if (s != ZS_OK) return s;
    if (batch == 0) return ZS_OK;
    if (!out_ids) return fail(ZS_ERR_INVALID_ARGUMENT, "out_ids is null");
    const bool with_rng = needs_rng(params, params_per_row, batch);
    if (!rng_state && with_rng) return fail(ZS_ERR_INVALID_ARGUMENT, "rng_state is null");
    int G = 0, rank = -1;
    int r = g_nccl.count(nccl_comm, &G);
    if (r == kNcclSuccess) r = g_nccl.user_rank(nccl_comm, &rank);
    if (r != kNcclSuccess) return fail(ZS_ERR_NCCL, nccl_msg("communicator size/rank", r));
    if (G != n_ranks || rank < 0 || rank >= G)
        return fail(ZS_ERR_INVALID_ARGUMENT, "n_ranks differs from the communicator's size");
    cudaStream_t st = (cudaStream_t)stream;
    // With extras every rank merges every row (row_info and candidate lists for the
    // whole batch); otherwise each rank merges only the rows it owns.
    const bool full = extras && (extras->row_info || extras->cand_ids || extras->cand_probs);
    const int R = (batch + G - 1) / G;
    const bool padded = !full && (int64_t)R * G != batch;
    const size_t slots_bytes = (size_t)bytes * G;
    const size_t ids_off = (slots_bytes + 255) & ~(size_t)255;
    const size_t st_off = ids_off + (((size_t)R * G * sizeof(int32_t) + 255) & ~(size_t)255);
    const size_t need = padded ? st_off + (size_t)R * G * sizeof(uint64_t) : slots_bytes;
    {
        DeviceGuard g(h->device);
        if (!g.ok) return fail(ZS_ERR_CUDA, "cudaSetDevice failed");
        s = grow((void**)&h->gather, &h->gather_bytes, need);
        if (s != ZS_OK) return s;
    }
    uint8_t* slots = h->gather;  // rank g's blocks at slots + g * bytes
    uint8_t* mine = slots + (size_t)rank * bytes;
    const bool want_lse = extras && extras->want_log_z && extras->row_info;
    s = zs_shard_partials(h, logits_local, ld, batch, n_local, vocab_offset, n_vocab_total, n_ranks,
                          params, params_per_row, history, history_ld, history_len, mine,
                          want_lse ? 1 : 0, stream);
    if (s != ZS_OK) return s;
    const Clock::time_point deadline =
        t0 + std::chrono::milliseconds(h->coll_timeout_ms > 0 ? h->coll_timeout_ms : 3600000);
    DeviceGuard g(h->device);
    if (full) {
        // in place: rank g's blocks already sit at slots + g * bytes
        r = nccl_settle(g_nccl.all_gather(mine, slots, (size_t)bytes, kNcclUint8, nccl_comm, st),
                        nccl_comm, deadline);
        if (r != kNcclSuccess) return fail(ZS_ERR_NCCL, nccl_msg("ncclAllGather", r));
        s = zs_shard_merge(h, slots, n_ranks, batch, n_vocab_total, params, params_per_row,
                           rng_state, out_ids, extras, stream);
        if (s != ZS_OK) return s;
        return wait_collectives(h, nccl_comm, st, t0);
    }
    // 1. every rank sends each owner the blocks of the owner's rows
    const Plan pl = make_plan(batch, shard_cols(n_vocab_total, n_ranks), n_vocab_total, params,
                              params_per_row, kShardLayoutCtas, kShardLayoutWarps, false, n_ranks);
    int my_r0 = 0, my_n = 0;
    owner_rows(batch, G, rank, &my_r0, &my_n);
    r = g_nccl.group_start();
    for (int peer = 0; peer < G && r == kNcclSuccess; ++peer) {
        if (peer == rank) continue;
        int o_r0 = 0, o_n = 0;
        owner_rows(batch, G, peer, &o_r0, &o_n);
        int64_t sp[3][2];
        const int ks = row_spans(pl, batch, o_r0, o_n, sp);
        for (int i = 0; i < ks && r == kNcclSuccess; ++i)
            r = g_nccl.send(mine + sp[i][0], (size_t)sp[i][1], kNcclUint8, peer, nccl_comm, st);
        const int kr = row_spans(pl, batch, my_r0, my_n, sp);
        uint8_t* from = slots + (size_t)peer * bytes;
        for (int i = 0; i < kr && r == kNcclSuccess; ++i)
            r = g_nccl.recv(from + sp[i][0], (size_t)sp[i][1], kNcclUint8, peer, nccl_comm, st);
    }
    {
        const int re = g_nccl.group_end();
        if (r == kNcclSuccess) r = re;
    }
    r = nccl_settle(r, nccl_comm, deadline);
    if (r != kNcclSuccess) return fail(ZS_ERR_NCCL, nccl_msg("block exchange (ncclSend/ncclRecv)", r));
    // 2. the owner merges its rows into [G][R] arrays (the caller's when B = G * R)
    int32_t* ids_buf = padded ? (int32_t*)(h->gather + ids_off) : out_ids;
    uint64_t* st_buf = padded ? (uint64_t*)(h->gather + st_off) : rng_state;
    if (padded && with_rng)
        ZS_CUDA(cudaMemcpyAsync(st_buf, rng_state, (size_t)batch * sizeof(uint64_t),
                                cudaMemcpyDeviceToDevice, st));
    s = zs_shard_merge_rows(h, slots, n_ranks, batch, my_r0, my_n, n_vocab_total, params,
                            params_per_row, with_rng ? st_buf : nullptr, ids_buf, nullptr, stream);
    if (s != ZS_OK) return s;
    // 3. every rank gets every owner's ids and Rng states (in place)
    r = g_nccl.group_start();
    if (r == kNcclSuccess)
        r = g_nccl.all_gather(ids_buf + (size_t)rank * R, ids_buf, (size_t)R, kNcclInt32, nccl_comm, st);
    if (r == kNcclSuccess && with_rng)
        r = g_nccl.all_gather(st_buf + (size_t)rank * R, st_buf, (size_t)R, kNcclUint64, nccl_comm, st);
    {
        const int re = g_nccl.group_end();
        if (r == kNcclSuccess) r = re;
    }
    r = nccl_settle(r, nccl_comm, deadline);
    if (r != kNcclSuccess) return fail(ZS_ERR_NCCL, nccl_msg("ids/states all-gather", r));
    if (padded) {
        ZS_CUDA(cudaMemcpyAsync(out_ids, ids_buf, (size_t)batch * sizeof(int32_t),
                                cudaMemcpyDeviceToDevice, st));
        if (with_rng)
            ZS_CUDA(cudaMemcpyAsync(rng_state, st_buf, (size_t)batch * sizeof(uint64_t),
                                    cudaMemcpyDeviceToDevice, st));
    }
    return wait_collectives(h, nccl_comm, st, t0);
}

#ifdef ZS_DEBUG_CHECKS
// Bounds-checking builds only: the first recorded violation {site, value, block, count}.
int zs_debug_read(unsigned long long* out4) {
    return (int)cudaMemcpyFromSymbol(out4, zs::zs_debug_record, 4 * sizeof(unsigned long long));
}
#endif

}  // extern "C"

// ---------------------------------------------------------------------------
// zs_sample_noalloc: zs_sample's select and merge kernels over the fixed static
// scratch of zs_noalloc_scratch.cu.  Nothing here allocates device or host memory.
// ---------------------------------------------------------------------------
cudaError_t zs_noalloc_scratch_address(void** ptr);  // zs_noalloc_scratch.cu

namespace {

constexpr int kNoAllocMaxDevices = 64;
constexpr size_t kNoAllocHeadBytes = 256;  // [0] status word, [4] fail counter

// Per-device launch geometry and scratch address, set up once by the first call
// on that device.  `ctx` carries only the geometry launch_merge reads; its
// buffer pointers stay null.
struct NoAllocDevice {
    bool ready = false;
    uint8_t* scratch = nullptr;
    zs_context ctx;
};
NoAllocDevice g_noalloc[kNoAllocMaxDevices];
std::mutex g_noalloc_mu;

zs_status noalloc_setup(int dev, NoAllocDevice** out) {
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    NoAllocDevice& d = g_noalloc[dev];
    if (!d.ready) {
        cudaDeviceProp prop;
        ZS_CUDA(cudaGetDeviceProperties(&prop, dev));
        if (prop.major != 10) return fail(ZS_ERR_NO_DEVICE, "zs_sample_noalloc: not an sm_100 device");
        d.ctx.device = dev;
        d.ctx.num_sms = prop.multiProcessorCount;
        d.ctx.select_smem = sizeof(zs::FastSmem);
        d.ctx.merge_smem = sizeof(zs::CandState);
        d.ctx.warp_merge_smem = sizeof(zs::WarpMergeSmem);
        ZS_CUDA(cudaFuncSetAttribute(zs::zs_select_kernel<false>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)d.ctx.select_smem));
        ZS_CUDA(cudaFuncSetAttribute(zs::zs_merge_kernel<false>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)d.ctx.merge_smem));
        ZS_CUDA(cudaFuncSetAttribute(zs::zs_warp_merge_kernel<false>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)d.ctx.warp_merge_smem));
        zs_status sw = setup_wselect<zs::WCfgS>(&d.ctx.wsel_smem[0], &d.ctx.wsel_warps[0],
                                                d.ctx.num_sms);
        if (sw == ZS_OK)
            sw = setup_wselect<zs::WCfgL>(&d.ctx.wsel_smem[1], &d.ctx.wsel_warps[1], d.ctx.num_sms);
        if (sw != ZS_OK) return sw;
        int per_sm = 0;
        ZS_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, zs::zs_select_kernel<false>,
                                                              zs::kThreads, d.ctx.select_smem));
        d.ctx.select_ctas_per_sm = std::max(1, per_sm);
        d.ctx.select_ctas = d.ctx.select_ctas_per_sm * d.ctx.num_sms;
        void* p = nullptr;
        ZS_CUDA(zs_noalloc_scratch_address(&p));  // with `dev` current
        d.scratch = (uint8_t*)p;
        d.ready = true;
    }
    *out = &d;
    return ZS_OK;
}

// Scratch of one call: head, the CTA kernel's fail list, the partial blocks.
size_t noalloc_bytes(const Plan& pl, int64_t B) {
    const size_t units = pl.launch_cta ? (size_t)(B * pl.S) : 0;
    return kNoAllocHeadBytes + ((units * sizeof(int32_t) + 255) & ~(size_t)255) + (size_t)pl.bytes;
}

// Re-cuts the CTA kernel's rows into S slices (the warp layouts do not change).
void replan_slices(Plan& pl, int B, int V, int S) {
    const int per = (V + S - 1) / S;
    pl.slice = std::max(4, (per + 3) & ~3);
    pl.S = std::max(1, (V + pl.slice - 1) / pl.slice);
    place_areas(pl, B);
}

}  // namespace

extern "C" zs_status zs_sample_noalloc(const float* logits, int64_t ld, int32_t batch,
                                       int32_t n_vocab, const zs_params* params,
                                       const int32_t* history, int64_t history_ld,
                                       const int32_t* history_len, uint64_t* rng_state,
                                       int32_t* out_ids, int32_t* device_status, void* stream) {
    NvtxRange nvtx_range("zs_sample_noalloc");
    if (batch < 0) return fail(ZS_ERR_INVALID_ARGUMENT, "batch < 0");
    if (!params) return fail(ZS_ERR_INVALID_ARGUMENT, "params is null");
    if (batch == 0) return ZS_OK;
    if (!out_ids) return fail(ZS_ERR_INVALID_ARGUMENT, "out_ids is null");
    cudaStream_t st = (cudaStream_t)stream;
    if (n_vocab <= 0) {  // sample.cpp:34 -- returns 0 before touching the Rng
        ZS_CUDA(cudaMemsetAsync(out_ids, 0, (size_t)batch * sizeof(int32_t), st));
        return ZS_OK;
    }
    if (!logits) return fail(ZS_ERR_INVALID_ARGUMENT, "logits is null");
    if (((uintptr_t)logits & 3u) != 0) return fail(ZS_ERR_INVALID_ARGUMENT, "logits not 4-byte aligned");
    if (ld < n_vocab) return fail(ZS_ERR_INVALID_ARGUMENT, "ld < n_vocab");
    if (batch > 1 && ld > (int64_t)1 << 40) return fail(ZS_ERR_INVALID_ARGUMENT, "ld too large");
    if (!rng_state && needs_rng(params, 0, batch))
        return fail(ZS_ERR_INVALID_ARGUMENT, "rng_state is null");
    const bool have_hist = history && history_len;
    if (have_hist && history_ld < 0) return fail(ZS_ERR_INVALID_ARGUMENT, "history_ld < 0");
    int dev = -1;
    ZS_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kNoAllocMaxDevices)
        return fail(ZS_ERR_INVALID_ARGUMENT, "zs_sample_noalloc: device ordinal above 63");
    NoAllocDevice* d = nullptr;
    zs_status s = noalloc_setup(dev, &d);
    if (s != ZS_OK) return s;
    Plan pl = make_plan(batch, n_vocab, n_vocab, params, 0, d->ctx.select_ctas, d->ctx.wsel_warps,
                        have_hist);
    if (pl.any_large)
        return fail(ZS_ERR_INVALID_ARGUMENT,
                    "zs_sample_noalloc: top_k + repeat window above 2048 (or window above 512) "
                    "needs zs_sample");
    const size_t cap = ZS_NOALLOC_SCRATCH_BYTES;
    // Fewer slices per row when the default cut does not fit (same results).
    while (pl.S > 1 && noalloc_bytes(pl, batch) > cap) replan_slices(pl, batch, n_vocab, pl.S - 1);
    if (noalloc_bytes(pl, batch) > cap) {
        char msg[256];
        std::snprintf(msg, sizeof(msg),
                      "zs_sample_noalloc: %d rows need %zu bytes of scratch, the fixed scratch "
                      "holds %zu; split the batch or use zs_sample",
                      batch, noalloc_bytes(pl, batch), cap);
        return fail(ZS_ERR_INVALID_ARGUMENT, msg);
    }
    const int64_t units = pl.launch_cta ? (int64_t)batch * pl.S : 0;
    if (units > INT32_MAX) return fail(ZS_ERR_INVALID_ARGUMENT, "zs_sample_noalloc: batch too large");
    uint8_t* head = d->scratch;
    int32_t* fail_units = (int32_t*)(d->scratch + kNoAllocHeadBytes);
    uint8_t* part = d->scratch + kNoAllocHeadBytes + (((size_t)units * sizeof(int32_t) + 255) & ~(size_t)255);

    zs::Args a;
    std::memset(&a, 0, sizeof(a));
    a.logits = logits;
    a.ld = ld;
    a.B = batch;
    a.V = n_vocab;
    a.V_total = n_vocab;
    a.shared = to_dev(params[0]);
    a.hist = have_hist ? history : nullptr;
    a.hist_ld = history_ld;
    a.hist_len = have_hist ? history_len : nullptr;
    a.rng = rng_state;
    a.out_ids = out_ids;
    a.mode = 0;
    a.status = device_status ? (int*)device_status : (int*)head;
    a.fail_count = (unsigned*)(head + 4);
    a.fail_units = fail_units;
    // The fail counter must start every call at zero; the status word is cleared too.
    ZS_CUDA(cudaMemsetAsync(head, 0, kNoAllocHeadBytes, st));
    s = launch_partials(&d->ctx, a, pl, part, false, st);
    if (s != ZS_OK) return s;
    const zs::MergeArgs m = merge_args_for(a, pl, part, 1, 0);
    return launch_merge(&d->ctx, m, pl.max_ksel, false, st);
}
