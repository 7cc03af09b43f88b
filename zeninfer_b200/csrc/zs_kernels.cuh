// zs_kernels.cuh -- the sampler's device code.
//
// zs_select_kernel streams every logits row once from HBM and leaves, per
// work unit (row, vocab slice), a partial block: the unit's candidate keys
// (a superset of its top-k after the repetition penalty), the sum-exp
// scalars and an id-0 flag.  zs_merge_kernel then merges a row's blocks --
// from the slices of one GPU, or from every rank after the vocab-shard
// all-gather -- sorts the shortlist and runs the f64 tail of sample_token
// (src/sample.cpp:52-101).  Rows whose shortlist does not fit shared memory go
// through zs_large_kernel instead.
//
// Per select CTA: one producer warp issues 1-D bulk copies (cp.async.bulk, no
// tensor map, no multicast) of 16 KB stages into a 4-stage shared-memory ring,
// completion tracked by mbarrier transaction counts.  Eight consumer warps
// filter each stage against the current threshold key with plain float
// compares; survivors are appended to a shared candidate buffer.  The first
// stage of a unit sets the threshold from the per-thread maxima; when the
// buffer fills, a compaction keeps a superset of the best K_eff and raises it.
// The streaming kernel does no per-row sorting or f64 work, so nothing stalls
// the copy engine between rows.
#pragma once

#include <math.h>

#include <type_traits>

#include <cooperative_groups.h>

#include "zs_device.cuh"

namespace zs {

constexpr int kConsumerWarps = 8;
constexpr int kNC = kConsumerWarps * 32;  // consumer threads
constexpr int kThreads = kNC + 32;        // + one producer warp
constexpr int kTileElems = 4096;          // floats per ring stage (16 KB)
constexpr int kHalfElems = kTileElems / 2;
constexpr int kStages = 4;
constexpr int kKeffFastMax = 2048;        // top-k + penalty window handled in shared memory
constexpr int kWinFastMax = 512;          // penalty window handled in shared memory
constexpr int kCandMargin = 16;           // head/tail elements appended outside the tile check
constexpr int kSlackMin = 64;             // a compaction may keep slack(K) extra keys: whole
constexpr int kSlackMax = 1024;           // radix buckets (tie groups) instead of splitting them
constexpr int kCompactMinGrowth = 512;    // compact once the buffer grew by max(K_eff, this)
constexpr int kCompactGrowthSmall = 128;  // ... for one-pass shortlists, whose compaction is cheap
constexpr int kCandCap = 5136;            // >= kKeffFastMax + kSlackMax + kHalfElems + kCandMargin
constexpr int kOnePassMaxKeff = 256;      // shortlists up to this filter a stage in one pass
constexpr int kCandRegs = (kCandCap + kNC - 1) / kNC;
constexpr int kSortMax = 4096;            // bitonic size bound (kKeffFastMax + kWinFastMax -> 4096)
constexpr int kProbOffset = 2048;         // f64 probabilities alias cand[2048..4096)
constexpr int kShortlistDefault = 256;    // kTopPShortlist, src/sample.cpp:12

// Warp-independent select (zs_wselect_kernel): rows whose shortlist + penalty
// window fits a warp's candidate slot.
constexpr int kWTile = 1024;               // floats per ring stage (4 KB)
constexpr int kWStages = 3;
constexpr int kWStepElems = 128;           // floats one warp step covers (32 lanes x float4)
constexpr int kWMinElems = 2048;           // smallest share of the batch per warp

// The two warp-kernel configurations: short shortlists (every default of the
// reference) and longer ones.  A longer shortlist needs a bigger candidate slot
// per warp, so fewer warps fit an SM; with fewer threads per CTA each thread may
// use more registers, which the register-resident compaction of a bigger slot needs.
struct WCfgS {
    static constexpr int kCap = 640;      // candidate keys per warp
    static constexpr int kWarps = 12;     // warps per CTA (one CTA per SM)
    static constexpr int kKeffMax = 320;  // shortlist + penalty window
    static constexpr int kWinMax = 64;    // penalty window
    static constexpr int kClass = 0;
    static constexpr uint32_t kSlackDiv = 0;  // intermediate compactions are exact
};
struct WCfgL {
    static constexpr int kCap = 2048;
    static constexpr int kWarps = 7;
    static constexpr int kKeffMax = 1280;
    static constexpr int kWinMax = 256;
    static constexpr int kClass = 1;
    static constexpr uint32_t kSlackDiv = 4;  // intermediate compactions keep <= keff + keff/4
};

static_assert(kCandCap >= kKeffFastMax + kSlackMax + kHalfElems + kCandMargin,
              "candidate buffer too small for half-stage passes");
static_assert(kCandCap >= kOnePassMaxKeff + 2 * 128 + 256 + kTileElems + kCandMargin,
              "candidate buffer too small for one-pass stages");
static_assert(kKeffFastMax + kSlackMax + kWinFastMax <= kSortMax, "sort bound");

__host__ __device__ constexpr uint32_t slack_for(uint32_t k) {
    return k / 2 < (uint32_t)kSlackMin ? (uint32_t)kSlackMin
                                       : (k / 2 > (uint32_t)kSlackMax ? (uint32_t)kSlackMax : k / 2);
}
static_assert(kSortMax <= kCandCap, "sort region exceeds the candidate buffer");
static_assert(kProbOffset + kKeffFastMax / 1 * 1 <= kCandCap, "probability region");

// Bounds-checking build (-DZS_DEBUG_CHECKS): every candidate-buffer and partial
// access is checked; the first violation (site, value, block) is recorded in
// zs_debug_record and the access is skipped instead of faulting.
#ifdef ZS_DEBUG_CHECKS
__device__ unsigned long long zs_debug_record[4];
#define ZS_CHECK(cond, site, val)                                                            \
    ((cond) ? true                                                                           \
            : (atomicCAS(&zs_debug_record[0], 0ull, (unsigned long long)(site)) == 0ull      \
                   ? (zs_debug_record[1] = (unsigned long long)(val),                        \
                      zs_debug_record[2] = (unsigned long long)blockIdx.x,                   \
                      atomicAdd(&zs_debug_record[3], 1ull), false)                           \
                   : (atomicAdd(&zs_debug_record[3], 1ull), false)))
#else
__device__ __forceinline__ bool zs_check_off() { return true; }
#define ZS_CHECK(cond, site, val) zs_check_off()
#endif

struct Params {  // zen::SamplingParams layout
    float temp;
    int32_t top_k;
    float top_p;
    float repeat_penalty;
    int32_t repeat_last_n;
};

struct RowInfo {  // zs_row_info layout
    float max_logit;
    int32_t k;
    int32_t m;
    int32_t pos;
    double r;
    double sum;
    double boundary;
    double log_z;
};

// Partial block of one (row, slice): header then `count` keys sorted descending.
struct PartialHeader {
    uint32_t count;
    uint32_t flags;
    float lse_m;
    float lse_s;
};
constexpr uint32_t kPartHasId0 = 1u;
constexpr uint32_t kPartX0Nan = 2u;
// The block's piece was filtered from a speculative opening threshold whose value
// order is in the header's third word (that word holds no log-sum-exp then).
constexpr uint32_t kPartSpec = 4u;
// Speculative opening thresholds (zs_wselect_kernel): pieces of at least
// kSpecMinCols columns whose row has a shortlist of at least kSpecMinKeff keys.
constexpr uint32_t kSpecMinKeff = 128;
constexpr int kSpecMinCols = 32768;
constexpr int kPartialHeaderBytes = 16;

struct StageMeta {
    int32_t unit;
    int32_t start;
    int32_t n;
    int32_t flags;
};
constexpr int kMetaFirst = 1, kMetaLast = 2, kMetaDone = 4;

constexpr int kStatusTimeout = 4;  // ZS_ERR_DEVICE_TIMEOUT

struct Args {
    const float* logits;
    int64_t ld;
    int32_t B;
    int32_t V;          // columns held here
    int32_t id_offset;  // global id of local column 0 (vocab shard)
    int32_t V_total;    // vocabulary size n of sample_token
    Params shared;
    const Params* row_params;  // device [B] or null
    const int32_t* hist;
    int64_t hist_ld;
    const int32_t* hist_len;
    uint64_t* rng;
    int32_t* out_ids;
    RowInfo* info;
    int32_t* cand_ids;
    double* cand_probs;
    int32_t cand_ld;
    int32_t S;      // slices per row
    int32_t slice;  // columns per slice (multiple of 4)
    int32_t n_units;
    int32_t mode;   // 0: zs_sample (blocks in handle scratch); 1: vocab shard (caller's blocks)
    // Speculative thresholds: units whose guess was too high are listed here
    // (fail_count, fail_units) and redone by a second launch with
    // `redo` set, which takes its units from that list and does not speculate.
    unsigned* fail_count;
    int32_t* fail_units;
    int32_t redo;
    uint8_t* part;  // partial blocks [B][S]
    int64_t part_stride;
    int* status;
    // large-k path workspace
    uint8_t* large_ws;
    int64_t large_ws_per_cta;
    // Warp-piece layout (zs_wselect_kernel): the batch flattened to wl_E =
    // B * wl_Vn columns is cut into wl_NW equal contiguous shares, one per warp;
    // a share is cut at row ends into pieces, and piece j of warp w writes its
    // block at wpart + (w * wl_P + j) * wl_stride.
    uint8_t* wpart;
    int64_t wl_E;
    int64_t wl_stride;
    int32_t wl_NW;
    int32_t wl_P;
    int32_t wl_Vn;
    int32_t wl_class;  // rows this warp launch serves: WCfgS::kClass or WCfgL::kClass
    // Speculative opening thresholds allowed (zs_wselect_kernel; the merge checks
    // each row and lists the rows it cannot certify for an exact redo).
    int32_t spec;
    // zs_large_kernel: when set, the rows to redo are spec_rows[0 .. *spec_count)
    const unsigned* spec_count;
    const int32_t* spec_rows;
};

// Layout of one warp configuration's blocks (see Args).
struct WLayout {
    int64_t off;
    int64_t E;
    int64_t stride;
    int32_t NW;
    int32_t P;
    int32_t Vn;
};

struct MergeArgs {
    const uint8_t* gathered;
    // history only to route rows the same way as the select kernel did
    const int32_t* hist;
    int64_t hist_ld;
    const int32_t* hist_len;
    int64_t rank_stride;
    int32_t G;
    int32_t S;
    int64_t part_stride;
    int32_t B;
    int32_t V_total;
    Params shared;
    const Params* row_params;
    uint64_t* rng;
    int32_t* out_ids;
    RowInfo* info;
    int32_t* cand_ids;
    double* cand_probs;
    int32_t cand_ld;
    int* status;
    // warp-piece blocks (see Args) of the two warp configurations, at wl[c].off
    // inside each rank's area
    WLayout wl[2];
    // every row's blocks are S slice blocks (zs_lmhead_kernel's output)
    int32_t force_slices;
    // rows merged by this launch: [row0, row1) of the B rows the blocks describe
    // (the row-owner merge of the vocab-sharded mode takes a share of them)
    int32_t row0, row1;
    // rows whose speculative thresholds the merge cannot certify go to this list
    // (drawn afterwards by zs_large_kernel); null when no block can be speculative
    unsigned* spec_count;
    int32_t* spec_rows;
    int32_t spec_redo_all;  // list every speculative row (tests of the redo path)
};

struct RowPlan {
    Params p;
    int32_t ksel;  // shortlist size (1 for greedy)
    int32_t win;   // penalty window length
    int32_t keff;  // ksel + win
    int32_t hist_len;
    bool greedy;
    bool penal;
    bool wfast;  // zs_wselect_kernel<WCfgS>: keff <= 320, window <= 64
    bool wbig;   // zs_wselect_kernel<WCfgL>: the other rows with keff <= 1280, window <= 256
    bool fast;   // zs_select_kernel: the other rows with keff <= kKeffFastMax
    bool large;  // zs_large_kernel: the rest
};

__device__ __forceinline__ Params load_params(const Params* rp, const Params& shared, int row) {
    return rp ? rp[row] : shared;
}

// The sequential f64 loops of sample_token's tail (src/sample.cpp:69-101) for one
// thread: the same additions in the same order as the plain loops, with the
// operands loaded eight at a time ahead of the dependent additions.

// sum of p[0..n), in index order
__device__ __forceinline__ double seq_sum(const double* p, uint32_t n) {
    double s = 0.0;
    uint32_t i = 0;
    if (n >= 8u) {
        double v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = p[j];
        for (i = 8; i + 8u <= n; i += 8u) {
            double u[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) u[j] = p[i + j];
#pragma unroll
            for (int j = 0; j < 8; ++j) s += v[j];
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = u[j];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) s += v[j];
    }
    for (; i < n; ++i) s += p[i];
    return s;
}

// The nucleus loop `while (m < n && acc < top_p) acc += p[m++]`; returns m, acc.
__device__ __forceinline__ int seq_nucleus(const double* p, int n, double top_p, double& acc_out) {
    double acc = 0.0;
    int m = 0;
    while (m < n && acc < top_p) {
        double v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = (m + j < n) ? p[m + j] : 0.0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (m < n && acc < top_p) {
                acc += v[j];
                ++m;
            }
        }
    }
    acc_out = acc;
    return m;
}

// The inverse-CDF walk: the first i < m with r < acc_i (acc_i the running sum of
// p[0..i]); returns it, or -1 when none, with acc_i and acc_{i-1} (or the total).
__device__ __forceinline__ int seq_cdf(const double* p, int m, double r, double& acc_out,
                                       double& prev_out) {
    double acc = 0.0, prev = 0.0;
    for (int i0 = 0; i0 < m; i0 += 8) {
        double v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = (i0 + j < m) ? p[i0 + j] : 0.0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            if (i0 + j < m) {
                prev = acc;
                acc += v[j];
                if (r < acc) {
                    acc_out = acc;
                    prev_out = prev;
                    return i0 + j;
                }
            }
        }
    }
    acc_out = acc;
    prev_out = prev;
    return -1;
}

__device__ __forceinline__ RowPlan plan_row(const Params& p, int V_total, const int32_t* hist,
                                            const int32_t* hist_len, int64_t hist_ld, int row) {
    RowPlan r;
    r.p = p;
    r.greedy = (p.temp <= 0.0f);
    if (r.greedy) r.ksel = 1;
    else if (p.top_k > 0) r.ksel = p.top_k < V_total ? p.top_k : V_total;
    else r.ksel = kShortlistDefault < V_total ? kShortlistDefault : V_total;
    r.hist_len = 0;
    r.win = 0;
    if (p.repeat_penalty != 1.0f && hist != nullptr && hist_len != nullptr) {
        int len = hist_len[row];
        if ((int64_t)len > hist_ld) len = (int)hist_ld;  // never read past the row
        const int keep = p.repeat_last_n > 0 ? p.repeat_last_n : 0;
        r.hist_len = len;
        r.win = len > 0 ? (len < keep ? len : keep) : 0;
    }
    r.penal = r.win > 0;
    r.keff = r.ksel + r.win;
    r.wfast = (r.keff <= WCfgS::kKeffMax) && (r.win <= WCfgS::kWinMax);
    r.wbig = !r.wfast && (r.keff <= WCfgL::kKeffMax) && (r.win <= WCfgL::kWinMax);
    r.fast = !r.wfast && !r.wbig && (r.keff <= kKeffFastMax) && (r.win <= kWinFastMax);
    r.large = !r.wfast && !r.wbig && !r.fast;
    return r;
}

// ---- warp-piece layout ----
__host__ __device__ __forceinline__ int64_t wl_bound(int64_t E, int32_t NW, int32_t w) {
    return w >= NW ? E : ((int64_t)w * E) / NW;
}

// The warp whose share holds flattened column x.
__host__ __device__ __forceinline__ int32_t wl_warp_of(int64_t E, int32_t NW, int64_t x) {
    return (int32_t)(((x + 1) * (int64_t)NW - 1) / E);
}

struct WPiece {
    int32_t row;
    int32_t c0, c1;  // columns of the piece
    int32_t e0, e1;  // 16-byte aligned sub-range moved by bulk copies
    int32_t ntiles;
    bool active;     // the row belongs to the warp path
};

__device__ __forceinline__ WPiece wl_piece(const Args& a, int64_t b0, int64_t b1, int32_t r0, int j) {
    WPiece pc;
    pc.row = r0 + j;
    const int64_t rs = (int64_t)pc.row * a.wl_Vn;
    int64_t c0 = b0 > rs ? b0 - rs : 0;
    int64_t c1 = b1 - rs < (int64_t)a.wl_Vn ? b1 - rs : (int64_t)a.wl_Vn;
    c1 = c1 < a.V ? c1 : a.V;  // a shard may hold fewer columns than the layout's row
    c0 = c0 < c1 ? c0 : c1;
    pc.c0 = (int32_t)c0;
    pc.c1 = (int32_t)c1;
    const RowPlan rp = plan_row(load_params(a.row_params, a.shared, pc.row), a.V_total, a.hist,
                                a.hist_len, a.hist_ld, pc.row);
    pc.active = a.wl_class == WCfgS::kClass ? rp.wfast : rp.wbig;
    const uintptr_t p0 = (uintptr_t)(a.logits + (int64_t)pc.row * a.ld + pc.c0);
    const int pad = (int)(((16u - (unsigned)(p0 & 15u)) & 15u) >> 2);
    const int e0 = pc.c0 + pad;
    if (e0 >= pc.c1) {
        pc.e0 = pc.e1 = pc.c1;
    } else {
        pc.e0 = e0;
        pc.e1 = e0 + ((pc.c1 - e0) & ~3);
    }
    pc.ntiles = pc.active ? (pc.e1 - pc.e0 + kWTile - 1) / kWTile : 0;
    return pc;
}

struct UnitGeom {
    int32_t row, s;
    int32_t v0, v1;  // columns of the unit
    int32_t e0, e1;  // 16-byte aligned sub-range moved by bulk copies
};

__device__ __forceinline__ UnitGeom unit_geom(const Args& a, int u) {
    UnitGeom g;
    g.row = u / a.S;
    g.s = u - g.row * a.S;
    const int64_t v0 = (int64_t)g.s * a.slice;
    g.v0 = (int32_t)(v0 < a.V ? v0 : a.V);
    g.v1 = (int32_t)((int64_t)g.v0 + a.slice < a.V ? g.v0 + a.slice : a.V);
    const uintptr_t p0 = (uintptr_t)(a.logits + (int64_t)g.row * a.ld + g.v0);
    const int pad = (int)(((16u - (unsigned)(p0 & 15u)) & 15u) >> 2);
    int e0 = g.v0 + pad;
    if (e0 >= g.v1) {
        g.e0 = g.e1 = g.v1;
    } else {
        g.e0 = e0;
        g.e1 = e0 + ((g.v1 - e0) & ~3);
    }
    return g;
}

// ---------------------------------------------------------------------------
// Shared state of the consumer warps
// ---------------------------------------------------------------------------
struct CandState {
    uint64_t cand[kCandCap];
    uint32_t hist[256];
    uint32_t scan[kConsumerWarps + 1];
    uint64_t red64[kConsumerWarps];
    uint64_t red64b[kConsumerWarps];
    float redf[2 * kConsumerWarps];
    union {
        int32_t win[kWinFastMax];  // penalty window (end of a unit)
        uint64_t prop[kNC];        // per-thread threshold proposals
    };
    uint64_t thr;
    uint64_t thr2;
    uint4 part_hdr;
    double d_sum;
    double d_rescale;
    double lse_delta;
    uint32_t count;
    uint32_t removed;
    uint32_t sel_digit, sel_above, sel_cnt;
    uint32_t spec_ord;  // merge: largest speculative threshold order among the row's blocks
    int32_t abort;
    int32_t x0_nan;
    int32_t m;
    float lse_m, lse_s;
};

struct FastSmem {
    float ring[kStages][kTileElems];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    StageMeta meta[kStages];
    CandState st;
};

// ---- block primitives over the kNC consumer threads ----

__device__ __forceinline__ void csync() { consumer_sync<kNC>(); }
__device__ __forceinline__ bool csync_or(bool pred) { return consumer_sync_or<kNC>(pred); }

// Inclusive scan across the consumer threads; ends synchronised.
__device__ __forceinline__ uint32_t block_incl_scan(uint32_t v, uint32_t* s_scan, int ctid,
                                                    uint32_t& total) {
    const int lane = ctid & 31, warp = ctid >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(kFull, v, o);
        if (lane >= o) v += t;
    }
    if (lane == 31) s_scan[warp] = v;
    csync();
    if (warp == 0) {
        uint32_t w = lane < kConsumerWarps ? s_scan[lane] : 0u;
#pragma unroll
        for (int o = 1; o < kConsumerWarps; o <<= 1) {
            const uint32_t t = __shfl_up_sync(kFull, w, o);
            if (lane >= o) w += t;
        }
        if (lane < kConsumerWarps) s_scan[lane] = w;
    }
    csync();
    const uint32_t pre = warp ? s_scan[warp - 1] : 0u;
    total = s_scan[kConsumerWarps - 1];
    csync();
    return v + pre;
}

__device__ __forceinline__ uint64_t warp_min_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t t = __shfl_xor_sync(kFull, v, o);
        v = t < v ? t : v;
    }
    return v;
}

__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const uint64_t t = __shfl_xor_sync(kFull, v, o);
        v = t > v ? t : v;
    }
    return v;
}

// Appends key k (if pred) with one atomic per warp.  All 32 lanes must call.
__device__ __forceinline__ void warp_append(CandState& st, bool pred, uint64_t k, int lane) {
    const unsigned m = __ballot_sync(kFull, pred);
    if (m) {
        const int leader = __ffs(m) - 1;
        uint32_t base = 0;
        if (lane == leader) base = atomicAdd(&st.count, (uint32_t)__popc(m));
        base = __shfl_sync(kFull, base, leader);
        const uint32_t at = base + __popc(m & lanemask_lt());
        if (pred && ZS_CHECK(at < (uint32_t)kCandCap, 1, at)) st.cand[at] = k;
    }
}

// Appends the components of v (ids id..id+3) whose keys beat tau: one warp
// scan and one shared atomic per warp.  All 32 lanes must call.
__device__ __forceinline__ void append4(CandState& st, bool hit, const float4& v, int32_t id,
                                        uint64_t tau, int lane) {
    const uint64_t k0 = make_key(v.x, id), k1 = make_key(v.y, id + 1);
    const uint64_t k2 = make_key(v.z, id + 2), k3 = make_key(v.w, id + 3);
    const bool a0 = hit && k0 > tau, a1 = hit && k1 > tau, a2 = hit && k2 > tau, a3 = hit && k3 > tau;
    const uint32_t c = (uint32_t)a0 + (uint32_t)a1 + (uint32_t)a2 + (uint32_t)a3;
    uint32_t incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += t;
    }
    const uint32_t total = __shfl_sync(kFull, incl, 31);
    if (total == 0) return;
    uint32_t base = 0;
    if (lane == 31) base = atomicAdd(&st.count, total);
    base = __shfl_sync(kFull, base, 31);
    uint32_t pos = base + incl - c;
    if (!ZS_CHECK(pos + c <= (uint32_t)kCandCap, 2, pos + c)) return;
    if (a0) st.cand[pos++] = k0;
    if (a1) st.cand[pos++] = k1;
    if (a2) st.cand[pos++] = k2;
    if (a3) st.cand[pos] = k3;
}

// Appends one element without warp cooperation (head/tail columns).
__device__ __forceinline__ void single_append(CandState& st, float x, int32_t id,
                                              uint64_t tau_key) {
    const uint64_t k = make_key(x, id);
    if (k > tau_key) {
        const uint32_t at = atomicAdd(&st.count, 1u);
        if (ZS_CHECK(at < (uint32_t)kCandCap, 3, at)) st.cand[at] = k;
    }
}

// Online log-sum-exp in base 2: s = sum 2^((x - m) * c).
__device__ __forceinline__ void lse_add4(float& m, float& s, const float4& v, float vm, float c) {
    const float mn = fmaxf(m, vm);
    if (mn > m) {
        s *= fast_exp2((m - mn) * c);
        m = mn;
    }
    if (m > -INFINITY) {
        s += fast_exp2((v.x - m) * c) + fast_exp2((v.y - m) * c) + fast_exp2((v.z - m) * c) +
             fast_exp2((v.w - m) * c);
    }
}

__device__ __forceinline__ void lse_add1(float& m, float& s, float x, float c) {
    const float mn = fmaxf(m, x);
    if (mn > m) {
        s *= fast_exp2((m - mn) * c);
        m = mn;
    }
    if (m > -INFINITY) s += fast_exp2((x - m) * c);
}

__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2, float c) {
    const float M = fmaxf(m, m2);
    if (!(M > -INFINITY)) {
        m = M;
        s = 0.0f;
        return;
    }
    const float a = (m > -INFINITY) ? s * fast_exp2((m - M) * c) : 0.0f;
    const float b = (m2 > -INFINITY) ? s2 * fast_exp2((m2 - M) * c) : 0.0f;
    m = M;
    s = a + b;
}

// Reduces the per-thread (m, s) pairs into st.lse_m / st.lse_s.
__device__ __forceinline__ void block_lse(CandState& st, float m, float s, float c, int ctid) {
    const int lane = ctid & 31, warp = ctid >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float m2 = __shfl_xor_sync(kFull, m, o);
        const float s2 = __shfl_xor_sync(kFull, s, o);
        lse_merge(m, s, m2, s2, c);
    }
    if (lane == 0) {
        st.redf[2 * warp] = m;
        st.redf[2 * warp + 1] = s;
    }
    csync();
    if (ctid == 0) {
        float M = st.redf[0], Sx = st.redf[1];
        for (int w = 1; w < kConsumerWarps; ++w) lse_merge(M, Sx, st.redf[2 * w], st.redf[2 * w + 1], c);
        st.lse_m = M;
        st.lse_s = Sx;
    }
    csync();
}

// Threshold fast-test value for a threshold key.
__device__ __forceinline__ float tau_value(uint64_t tau_key) {
    if (tau_key == 0ull) return -INFINITY;
    const uint32_t o = (uint32_t)(tau_key >> 32);
    return o == 0u ? -INFINITY : value_of_ord(o);
}

// Shortlists up to kGroupMaxK use a cheaper threshold than a radix select: every
// consumer thread proposes the largest key of its own share of the keys, and the
// kk-th largest of those 256 proposals is a valid threshold (the kk proposals at
// or above it are kk distinct keys), usually only a little below the exact kk-th
// key.  Exact order comes later from the final sort.
constexpr uint32_t kGroupMaxK = kNC;

__device__ __forceinline__ void select_bucket(CandState& st, uint32_t need, int lane);

// kk-th largest of the per-thread proposals (0 = no key); 0 when fewer than kk
// threads proposed a key.  The proposals go to shared memory and warp 0 alone
// runs an exact radix select over them (8 keys per lane, warp-private
// histogram), so the block pays two barriers.  Every thread gets the result.
__device__ uint64_t kth_of_proposals(CandState& st, uint64_t mine, uint32_t kk, int ctid) {
    const int lane = ctid & 31, warp = ctid >> 5;
    st.prop[ctid] = mine;
    csync();
    if (warp == 0) {
        constexpr int Q = kNC / 32;
        uint64_t k[Q];
        uint64_t lo = ~0ull, hi = 0ull;
        uint32_t have = 0;
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            k[q] = st.prop[lane + 32 * q];
            if (k[q]) {
                lo = k[q] < lo ? k[q] : lo;
                hi = k[q] > hi ? k[q] : hi;
                ++have;
            }
        }
        lo = warp_min_u64(lo);
        hi = warp_max_u64(hi);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) have += __shfl_xor_sync(kFull, have, o);
        uint64_t T = 0ull;
        if (have >= kk) {
            if (kk == 1) {
                T = hi;
            } else {
                const uint64_t diff = lo ^ hi;
                int shift = diff ? ((63 - __clzll((long long)diff)) >> 3) << 3 : 0;
                uint64_t mask = shift >= 56 ? 0ull : (~0ull << (shift + 8));
                uint64_t prefix = lo & mask;
                uint32_t need = kk;
                for (;;) {
#pragma unroll
                    for (int q = 0; q < 8; ++q) st.hist[lane * 8 + q] = 0u;
                    __syncwarp();
#pragma unroll
                    for (int q = 0; q < Q; ++q)
                        if (k[q] != 0ull && (k[q] & mask) == prefix)
                            atomicAdd(&st.hist[(uint32_t)(k[q] >> shift) & 255u], 1u);
                    __syncwarp();
                    select_bucket(st, need, lane);
                    __syncwarp();
                    const uint32_t digit = st.sel_digit, above = st.sel_above, cnt = st.sel_cnt;
                    __syncwarp();
                    prefix |= (uint64_t)digit << shift;
                    mask |= 0xffull << shift;
                    need -= above;
                    if (cnt == need || shift == 0) break;  // whole bucket in: its minimum is the kk-th
                    shift -= 8;
                }
                uint64_t m = ~0ull;
#pragma unroll
                for (int q = 0; q < Q; ++q)
                    if (k[q] != 0ull && (k[q] & mask) == prefix && k[q] < m) m = k[q];
                T = warp_min_u64(m);
            }
        }
        if (lane == 0) st.thr = T;
    }
    csync();
    return st.thr;
}

// Warp 0 finds the radix bucket holding the need-th largest key: hist[] holds
// counts per digit; scanning digits from 255 down, the bucket is where the
// running count reaches need.  Writes sel_digit / sel_above / sel_cnt.
__device__ __forceinline__ void select_bucket(CandState& st, uint32_t need, int lane) {
    // lane l owns digits 255-8l .. 248-8l (descending)
    uint32_t h[8];
    uint32_t sum = 0;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        h[q] = st.hist[255 - 8 * lane - q];
        sum += h[q];
    }
    uint32_t incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += t;
    }
    const uint32_t before = incl - sum;
    if (before < need && incl >= need) {
        uint32_t cum = before;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            if (cum < need && cum + h[q] >= need) {
                st.sel_digit = 255u - 8u * (uint32_t)lane - (uint32_t)q;
                st.sel_above = cum;
                st.sel_cnt = h[q];
            }
            cum += h[q];
        }
    }
}

// Keeps the kk largest of the n > kk keys in cand[0..) -- plus at most `slack`
// more, when a whole radix bucket is cheaper to keep than to split -- and
// returns the smallest kept key, the new filter threshold.  Radix select on
// the 64-bit key with 8-bit digits, starting below the keys' common prefix;
// histogram increments are aggregated per warp with match.any.
__device__ uint64_t compact_top(CandState& st, uint32_t n, uint32_t kk, uint32_t slack,
                                int ctid) {
    const int lane = ctid & 31, warp = ctid >> 5;
    if (!ZS_CHECK(n <= (uint32_t)kCandCap && n > kk, 6, ((uint64_t)n << 32) | kk)) n = min(n, (uint32_t)kCandCap);
    uint64_t lo = ~0ull, hi = 0ull;
    for (uint32_t i = ctid; i < n; i += kNC) {
        const uint64_t k = st.cand[i];
        lo = k < lo ? k : lo;
        hi = k > hi ? k : hi;
    }
    lo = warp_min_u64(lo);
    hi = warp_max_u64(hi);
    if (lane == 0) {
        st.red64[warp] = lo;
        st.red64b[warp] = hi;
    }
    st.hist[ctid] = 0u;
    csync();
    uint64_t a = st.red64[0], b = st.red64b[0];
#pragma unroll
    for (int w = 1; w < kConsumerWarps; ++w) {
        a = st.red64[w] < a ? st.red64[w] : a;
        b = st.red64b[w] > b ? st.red64b[w] : b;
    }
    const uint64_t diff = a ^ b;  // n >= 2 unique keys: nonzero
    int shift = diff ? ((63 - __clzll((long long)diff)) >> 3) << 3 : 0;
    uint64_t mask = shift >= 56 ? 0ull : (~0ull << (shift + 8));
    uint64_t prefix = a & mask;
    uint32_t need = kk;
    for (;;) {
        for (uint32_t i = ctid; i < n; i += kNC) {
            const uint64_t k = st.cand[i];
            if ((k & mask) == prefix) atomicAdd(&st.hist[(uint32_t)(k >> shift) & 255u], 1u);
        }
        csync();
        if (warp == 0) select_bucket(st, need, lane);
        csync();
        const uint32_t digit = st.sel_digit, above = st.sel_above, cnt = st.sel_cnt;
        prefix |= (uint64_t)digit << shift;
        mask |= 0xffull << shift;
        need -= above;
        // keeping the whole bucket is exact or close enough; else split it further
        if (cnt <= need + slack || shift == 0) break;
        shift -= 8;
        st.hist[ctid] = 0u;
        csync();
    }
    // Threshold = smallest key of the selected bucket (all of it is kept).
    uint64_t mn = ~0ull;
    for (uint32_t i = ctid; i < n; i += kNC) {
        const uint64_t k = st.cand[i];
        if ((k & mask) == prefix && k < mn) mn = k;
    }
    mn = warp_min_u64(mn);
    if (lane == 0) st.red64[warp] = mn;
    csync();
    uint64_t T = st.red64[0];
#pragma unroll
    for (int w = 1; w < kConsumerWarps; ++w) T = st.red64[w] < T ? st.red64[w] : T;
    // Move the kept keys to the front: read all, then place with warp ballots.
    uint64_t loc[kCandRegs];
#pragma unroll
    for (int j = 0; j < kCandRegs; ++j) {
        const uint32_t i = ctid + j * kNC;
        loc[j] = (i < n) ? st.cand[i] : 0ull;
    }
    if (ctid == 0) st.count = 0u;
    csync();
    uint32_t wk = 0;
#pragma unroll
    for (int j = 0; j < kCandRegs; ++j) wk += __popc(__ballot_sync(kFull, loc[j] >= T));
    uint32_t base = 0;
    if (lane == 0 && wk) base = atomicAdd(&st.count, wk);
    base = __shfl_sync(kFull, base, 0);
    const unsigned below = lanemask_lt();
#pragma unroll
    for (int j = 0; j < kCandRegs; ++j) {
        const unsigned m = __ballot_sync(kFull, loc[j] >= T);
        if (loc[j] >= T) st.cand[base + __popc(m & below)] = loc[j];
        base += __popc(m);
    }
    csync();
    return T;
}

// Keeps the keys >= T of cand[0..n) at the front and returns how many.
__device__ __forceinline__ uint32_t keep_at_least(CandState& st, uint32_t n, uint64_t T, int ctid) {
    const int lane = ctid & 31;
    uint64_t loc[kCandRegs];
#pragma unroll
    for (int j = 0; j < kCandRegs; ++j) {
        const uint32_t i = ctid + j * kNC;
        loc[j] = (i < n) ? st.cand[i] : 0ull;
    }
    if (ctid == 0) st.count = 0u;
    csync();
    uint32_t wk = 0;
#pragma unroll
    for (int j = 0; j < kCandRegs; ++j) wk += __popc(__ballot_sync(kFull, loc[j] >= T));
    uint32_t base = 0;
    if (lane == 0 && wk) base = atomicAdd(&st.count, wk);
    base = __shfl_sync(kFull, base, 0);
    const unsigned below = lanemask_lt();
#pragma unroll
    for (int j = 0; j < kCandRegs; ++j) {
        const unsigned m = __ballot_sync(kFull, loc[j] >= T);
        if (loc[j] >= T) st.cand[base + __popc(m & below)] = loc[j];
        base += __popc(m);
    }
    csync();
    return st.count;
}

// Reduces cand[0..n) (n > kk) to a set that contains its kk largest keys and
// returns the new threshold (the smallest kept key).  Shortlists up to
// kGroupMaxK use the per-thread-maximum proposal (a few barriers); when that
// keeps too much, or for larger shortlists, the radix select finishes the job.
__device__ uint64_t compact_select(CandState& st, uint32_t n, uint32_t kk, int ctid) {
    const uint32_t slack = slack_for(kk);
    if (kk <= kGroupMaxK) {
        uint64_t mine = 0ull;
        for (uint32_t i = ctid; i < n; i += kNC) {
            const uint64_t k = st.cand[i];
            mine = k > mine ? k : mine;
        }
        const uint64_t T = kth_of_proposals(st, mine, kk, ctid);
        if (T != 0ull) {
            const uint32_t kept = keep_at_least(st, n, T, ctid);
            if (kept <= kk + 2 * slack + 256u) return T;
            n = kept;
        }
    }
    return compact_top(st, n, kk, slack, ctid);
}

// Sorts keys[0..n) descending, n <= SLOTS, in registers: a bitonic network over
// SLOTS slots (SLOTS / 32 per lane, slot = lane * P + j; unused slots hold 0,
// which sorts last).
template <int SLOTS>
__device__ __forceinline__ void warp_sort_desc_slots(uint64_t* keys, uint32_t n, int lane) {
    constexpr int P = SLOTS / 32;
    uint64_t k[P];
#pragma unroll
    for (int j = 0; j < P; ++j) {
        const uint32_t i = (uint32_t)lane * P + j;
        k[j] = i < n ? keys[i] : 0ull;
    }
#pragma unroll
    for (int size = 2; size <= SLOTS; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= P) {
#pragma unroll
                for (int j = 0; j < P; ++j) {
                    const int i = lane * P + j;
                    const uint64_t p = __shfl_xor_sync(kFull, k[j], stride / P);
                    const bool desc = (i & size) == 0, lower = (i & stride) == 0;
                    const uint64_t hi = k[j] > p ? k[j] : p, lo = k[j] > p ? p : k[j];
                    k[j] = (lower == desc) ? hi : lo;
                }
            } else {
#pragma unroll
                for (int j = 0; j < P; ++j) {
                    if ((j & stride) == 0) {
                        const int i = lane * P + j;
                        const bool desc = (i & size) == 0;
                        const uint64_t a = k[j], b = k[j | stride];
                        if (desc ? (a < b) : (a > b)) {
                            k[j] = b;
                            k[j | stride] = a;
                        }
                    }
                }
            }
        }
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < P; ++j) {
        const uint32_t i = (uint32_t)lane * P + j;
        if (i < n) keys[i] = k[j];
    }
    __syncwarp();
}

// Sorts cand[0..n) descending.  n <= kNC: every thread ranks one key against
// all others (keys are unique).  n <= kNC * 8: each warp sorts one of eight
// chunks in registers (a bitonic network of up to 256 slots), then three levels
// of pairwise merges (merge path) through cand[kSortScratch ..) join them.
// Larger n: bitonic over the next power of two in shared memory.
constexpr uint32_t kChunkSortMax = (uint32_t)kNC * 8u;  // 2048: chunks of <= 256
constexpr int kSortScratch = 2048;                       // cand[2048 .. 2048 + n) is free
static_assert(kSortScratch + (int)kChunkSortMax <= kCandCap, "sort scratch");

__device__ void sort_desc(CandState& st, uint32_t n, int ctid) {
    if (n <= 1) return;
    if (n <= (uint32_t)kNC) {
        const uint64_t k = (uint32_t)ctid < n ? st.cand[ctid] : 0ull;
        uint32_t rank = 0;
        if ((uint32_t)ctid < n) {
            uint32_t i = 0;
            for (; i + 8u <= n; i += 8u) {  // eight broadcast loads in flight
                uint64_t y[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) y[j] = st.cand[i + j];
#pragma unroll
                for (int j = 0; j < 8; ++j) rank += y[j] > k ? 1u : 0u;
            }
            for (; i < n; ++i) rank += st.cand[i] > k ? 1u : 0u;
        }
        csync();
        if ((uint32_t)ctid < n) st.cand[rank] = k;
        csync();
        return;
    }
    if (n <= kChunkSortMax) {
        constexpr uint32_t NW = (uint32_t)kConsumerWarps;
        const int lane = ctid & 31;
        const uint32_t w = (uint32_t)ctid >> 5;
        const uint32_t c = (n + NW - 1) / NW;  // 33..256; every chunk holds at least one key
        const uint32_t b0 = min(n, w * c), nc = min(n, b0 + c) - b0;
        if (c <= 64u) warp_sort_desc_slots<64>(st.cand + b0, nc, lane);
        else if (c <= 128u) warp_sort_desc_slots<128>(st.cand + b0, nc, lane);
        else warp_sort_desc_slots<256>(st.cand + b0, nc, lane);
        csync();
        // Three merge levels (8 runs -> 4 -> 2 -> 1), ping-ponging between cand and
        // cand + kSortScratch.  At each level a pair's threads split its output into
        // equal spans; a thread finds where its span starts in the two runs by a
        // binary search on that diagonal (merge path) and merges the span.
        uint64_t* src = st.cand;
        uint64_t* dst = st.cand + kSortScratch;
        for (uint32_t lvl = 0; lvl < 3u; ++lvl) {
            const uint32_t run = c << lvl;                  // input run length
            const uint32_t tpp = (uint32_t)kNC >> (2u - lvl);  // threads per pair: 64, 128, 256
            const uint32_t pair = (uint32_t)ctid / tpp, t = (uint32_t)ctid % tpp;
            const uint32_t a0 = min(n, 2u * pair * run), a1 = min(n, a0 + run);
            const uint32_t b1 = min(n, a1 + run);
            const uint32_t la = a1 - a0, lb = b1 - a1, tot = la + lb;
            const uint32_t per = (tot + tpp - 1) / tpp;
            const uint32_t d0 = min(tot, t * per), d1 = min(tot, d0 + per);
            if (d0 < d1) {
                const uint64_t* A = src + a0;
                const uint64_t* B = src + a1;
                // a = how many of the first d0 outputs come from A (A first on ties)
                uint32_t lo = d0 > lb ? d0 - lb : 0u, hi = d0 < la ? d0 : la;
                while (lo < hi) {
                    const uint32_t mid = (lo + hi) >> 1;
                    if (A[mid] >= B[d0 - 1u - mid]) lo = mid + 1u;
                    else hi = mid;
                }
                uint32_t ia = lo, ib = d0 - lo;
                for (uint32_t k = d0; k < d1; ++k) {
                    const bool take_a = ib >= lb || (ia < la && A[ia] >= B[ib]);
                    dst[a0 + k] = take_a ? A[ia++] : B[ib++];
                }
            }
            csync();
            uint64_t* tmp = src;
            src = dst;
            dst = tmp;
        }
        for (uint32_t i = ctid; i < n; i += kNC) st.cand[i] = src[i];  // src: the last output
        csync();
        return;
    }
    uint32_t N = 2;
    while (N < n) N <<= 1;
    if (!ZS_CHECK(N <= (uint32_t)kCandCap, 5, N)) return;
    for (uint32_t i = n + ctid; i < N; i += kNC) st.cand[i] = 0ull;
    csync();
    for (uint32_t k = 2; k <= N; k <<= 1) {
        for (uint32_t j = k >> 1; j > 0; j >>= 1) {
            for (uint32_t i = ctid; i < (N >> 1); i += kNC) {
                const uint32_t lo = ((i & ~(j - 1)) << 1) | (i & (j - 1));
                const uint32_t hi = lo | j;
                const uint64_t x = st.cand[lo], y = st.cand[hi];
                const bool desc = (lo & k) == 0;
                if (desc ? (x < y) : (x > y)) {
                    st.cand[lo] = y;
                    st.cand[hi] = x;
                }
            }
            csync();
        }
    }
}

// Repetition penalty (src/sample.cpp:40-50) for the ids of this unit: drop the
// raw keys of penalised ids from cand[0..n) (they become 0) and append the
// penalised values, compounding once per occurrence in the window.
//
// When have_lse, the unit's sum-exp (relative to lse_m, base-2 scale lse_c) was
// accumulated over raw values; st.lse_delta receives the change that replacing
// each penalised id's raw value by its penalised value makes to it.
__device__ void penalty_fixup(CandState& st, const float* row_logits, const int32_t* window,
                              int W, float pen, int32_t id_offset, int32_t v0, int32_t v1,
                              int32_t V_total, uint32_t n, bool have_lse, float lse_m,
                              float lse_c, int ctid) {
    for (int i = ctid; i < W; i += kNC) st.win[i] = window[i];
    if (ctid == 0) {
        st.removed = 0u;
        st.lse_delta = 0.0;
    }
    csync();
    for (uint32_t i = ctid; i < n; i += kNC) {
        const int32_t gid = key_id(st.cand[i]);
        for (int j = 0; j < W; ++j) {
            if (st.win[j] == gid) {
                st.cand[i] = 0ull;
                atomicAdd(&st.removed, 1u);
                break;
            }
        }
    }
    csync();
    const int32_t lo = id_offset + v0, hi = id_offset + v1;
    for (int j = ctid; j < W; j += kNC) {
        const int32_t gid = st.win[j];
        if (gid < 0 || gid >= V_total || gid < lo || gid >= hi) continue;
        bool first = true;
        for (int q = 0; q < j; ++q)
            if (st.win[q] == gid) {
                first = false;
                break;
            }
        if (!first) continue;
        int mult = 1;
        for (int q = j + 1; q < W; ++q) mult += (st.win[q] == gid) ? 1 : 0;
        const float raw = row_logits[gid - id_offset];
        float v = raw;
        for (int c = 0; c < mult; ++c) v = (v > 0.0f) ? v / pen : v * pen;
        const uint32_t at = atomicAdd(&st.count, 1u);
        if (ZS_CHECK(at < (uint32_t)kCandCap, 4, at)) st.cand[at] = make_key(v, gid);
        if (gid == 0) st.x0_nan = (v != v) ? 1 : 0;
        if (have_lse && lse_m > -INFINITY) {
            const double d = exp2(((double)v - (double)lse_m) * (double)lse_c) -
                             exp2(((double)raw - (double)lse_m) * (double)lse_c);
            atomicAdd(&st.lse_delta, d);
        }
    }
    csync();
}

// Shortlists longer than this (only the large-shortlist path has them) run the
// f64 tail in blocked order.
constexpr uint32_t kBlockedTail = 4096;

// The f64 tail of sample_token (src/sample.cpp:69-101) for a long sorted shortlist
// whose exps are in prob[0..kk): the same quantities, with the additions grouped.
// The shortlist is cut into segments of `seg` entries (256 or more, at most 4096
// segments); a warp sums a segment (each lane its entries in order, then a fixed
// shuffle tree), thread 0 adds the segment sums in order and walks entry by entry
// only inside the segment where the nucleus prefix or the draw crosses.  Grouped
// sums differ from one-by-one ones in their last bits only.  Segment sums live in
// st.cand, which the large-shortlist path does not otherwise use here.
__device__ __forceinline__ double lm_seg_sum(const double* prob, uint32_t lo, uint32_t hi, int lane) {
    double s = 0.0;
    for (uint32_t i = lo + lane; i < hi; i += 32) s += prob[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
    return s;
}

__device__ void finalize_blocked(CandState& st, const uint64_t* cand, double* prob, uint32_t kk,
                                 const Params& p, float max_l, float inv_temp, bool have_lse,
                                 bool x0_nan, float lse_m, float lse_s, int row, uint64_t* rng,
                                 int32_t* out_ids, RowInfo* info, int32_t* cand_ids,
                                 double* cand_probs, int32_t cand_ld, int ctid) {
    double* ss = reinterpret_cast<double*>(st.cand);  // one sum per segment
    const int lane = ctid & 31, warp = ctid >> 5;
    const uint32_t seg = 256u * ((kk + 256u * 4096u - 1) / (256u * 4096u));
    const uint32_t nseg = (kk + seg - 1) / seg;
    for (uint32_t g = warp; g < nseg; g += kConsumerWarps) {
        const double t = lm_seg_sum(prob, g * seg, min(kk, (g + 1) * seg), lane);
        if (lane == 0) ss[g] = t;
    }
    csync();
    if (ctid == 0) {
        double t = 0.0;
        for (uint32_t g = 0; g < nseg; ++g) t += ss[g];
        st.d_sum = t;
    }
    csync();
    const double sum = st.d_sum;
    for (uint32_t c0 = 0; c0 < kk; c0 += 4 * kNC) {  // loads ahead of the stores
        double e4[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t i = c0 + j * kNC + ctid;
            e4[j] = i < kk ? prob[i] : 0.0;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t i = c0 + j * kNC + ctid;
            if (i >= kk) continue;
            const double pi = e4[j] / sum;
            prob[i] = pi;
            if ((int32_t)i < cand_ld) {
                if (cand_ids) cand_ids[(int64_t)row * cand_ld + i] = key_id(cand[i]);
                if (cand_probs) cand_probs[(int64_t)row * cand_ld + i] = pi;
            }
        }
    }
    csync();
    for (uint32_t g = warp; g < nseg; g += kConsumerWarps) {
        const double t = lm_seg_sum(prob, g * seg, min(kk, (g + 1) * seg), lane);
        if (lane == 0) ss[g] = t;
    }
    csync();
    const bool nucleus = p.top_p < 1.0f;
    if (ctid == 0) {
        int m = (int)kk;
        double rescale = 1.0;
        if (nucleus) {
            const double tp = (double)p.top_p;
            double acc = 0.0;
            uint32_t g = 0;
            while (g < nseg && acc + ss[g] < tp) acc += ss[g++];
            uint32_t i = g < nseg ? g * seg : kk;
            while (i < kk && acc < tp) acc += prob[i++];
            m = (int)i;
            if (m == 0) {
                m = 1;
                acc = prob[0];
            }
            rescale = acc;
        }
        st.m = m;
        st.d_rescale = rescale;
    }
    csync();
    const int m = st.m;
    const double rs = st.d_rescale;
    if (nucleus) {
        for (int i = ctid; i < m; i += kNC) prob[i] /= rs;
        csync();
    }
    const uint32_t nseg_m = ((uint32_t)m + seg - 1) / seg;
    for (uint32_t g = warp; g < nseg_m; g += kConsumerWarps) {
        const double t = lm_seg_sum(prob, g * seg, min((uint32_t)m, (g + 1) * seg), lane);
        if (lane == 0) ss[g] = t;
    }
    csync();
    if (ctid == 0) {
        uint64_t st_rng = rng[row];
        const double r = rng_uniform(st_rng);
        rng[row] = st_rng;
        double acc = 0.0, prev = 0.0;
        uint32_t g = 0;
        while (g < nseg_m && !(r < acc + ss[g])) acc += ss[g++];
        int i = g < nseg_m ? (int)(g * seg) : m;
        int pos = m - 1;
        bool hit = false;
        for (; i < m; ++i) {
            prev = acc;
            acc += prob[i];
            if (r < acc) {
                pos = i;
                hit = true;
                break;
            }
        }
        const double d = hit ? fmin(r - prev, acc - r) : r - acc;
        if (out_ids) out_ids[row] = key_id(cand[pos < 0 ? 0 : pos]);
        if (info) {
            RowInfo ri;
            ri.max_logit = max_l;
            ri.k = (int32_t)kk;
            ri.m = m;
            ri.pos = pos;
            ri.r = r;
            ri.sum = sum;
            ri.boundary = d;
            ri.log_z = (have_lse && !x0_nan)
                           ? log((double)lse_s) + ((double)lse_m - (double)max_l) * (double)inv_temp
                           : __longlong_as_double(0x7ff8000000000000ll);
            info[row] = ri;
        }
    }
    csync();
}

// Certified parallel tail for calls that want only the drawn id (no row info, no
// candidate lists).  sample_token's tail (src/sample.cpp:69-101) makes two
// decisions from sequential f64 sums: where the nucleus ends (the first m with
// acc_m >= top_p) and where the draw lands (the first i with r < acc'_i).  Here
// the same sums are parallel prefix sums E_k of e = exp((x - max) / temp) in
// another order, so they differ from the sequential ones, but by little: every
// sum of at most 4096 terms in [0, 1] is off by at most (4 kk + 80) 2^-53 < 2e-12
// relative to its exact value, in either order, divisions included.  So a
// decision whose compared quantities lie further than kTailMargin (1e-10) apart
// on the parallel sums is the sequential decision too; when one does not, the
// caller runs the sequential loops instead (a draw within 1e-10 of a CDF
// boundary: about one row in 10^9).  Nothing is written until the result is
// certified; then the id and the advanced Rng state are stored.  Returns whether
// it drew (the same on every thread).
constexpr uint32_t kFastTailMin = 128;  // shorter shortlists: the sequential loops are short
constexpr double kTailMargin = 1e-10;

__device__ bool fast_tail(CandState& st, const uint64_t* cand, const double* e, uint32_t kk,
                          const Params& p, int row, uint64_t* rng, int32_t* out_ids, int ctid) {
    const int lane = ctid & 31, warp = ctid >> 5;
    // contiguous segments, at most 16 terms a thread (kk <= kBlockedTail)
    const uint32_t per = (kk + kNC - 1) / kNC;
    const uint32_t s0 = min(kk, (uint32_t)ctid * per), s1 = min(kk, s0 + per);
    double seg = 0.0;
    for (uint32_t i = s0; i < s1; ++i) seg += e[i];
    // block exclusive scan of the segment sums
    double inc = seg;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(kFull, inc, o);
        if (lane >= o) inc += t;
    }
    if (lane == 31) st.red64[warp] = (uint64_t)__double_as_longlong(inc);
    if (ctid == 0) {
        uint64_t sr = rng[row];
        st.lse_delta = rng_uniform(sr);  // the draw (not stored unless certified)
        st.thr2 = sr;
        st.sel_above = 0u;               // 1: a decision is too close to call
        st.m = (int)kk;
        st.sel_cnt = 0xffffffffu;        // the drawn position
    }
    csync();
    double pre = inc - seg, T = 0.0;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
        const double t = __longlong_as_double((long long)st.red64[w]);
        if (w < warp) pre += t;
        T += t;
    }
    const double r = st.lse_delta;
    if (!(T > 0.0) || !(T < INFINITY)) {  // NaN or inf terms: the same on every thread
        csync();
        return false;
    }
    // nucleus end: the first m (1..kk) with E_m / T >= top_p
    const bool nucleus = p.top_p < 1.0f;
    const double top_p = (double)p.top_p;
    if (nucleus) {
        if (!(top_p > 0.0)) {  // the loop takes no term: left to the sequential code
            csync();
            return false;
        }
        double E = pre;
        for (uint32_t i = s0; i < s1; ++i) {
            const double Ep = E;
            E += e[i];
            const double a = Ep / T, b = E / T;
            if (a < top_p && b >= top_p) {  // the crossing (E is nondecreasing)
                if (!(a < top_p - kTailMargin && b >= top_p + kTailMargin)) st.sel_above = 1u;
                st.m = (int)(i + 1);
                st.d_rescale = E;
            }
        }
        if (ctid == (int)((kk - 1) / per)) {  // the thread holding the last term
            if (E / T < top_p && !(E / T < top_p - kTailMargin)) st.sel_above = 1u;
        }
    }
    csync();
    const uint32_t m = (uint32_t)st.m;
    const double Em = (nucleus && m < kk) ? st.d_rescale : T;
    // the draw: the first i < m with r < E_{i+1} / E_m
    {
        double E = pre;
        for (uint32_t i = s0; i < s1 && i < m; ++i) {
            const double Ep = E;
            E += e[i];
            const double a = Ep / Em, b = E / Em;
            if (a <= r && r < b) {
                if (!(a < r - kTailMargin && b > r + kTailMargin)) st.sel_above = 1u;
                st.sel_cnt = i;
            }
        }
    }
    csync();
    if (st.sel_above != 0u || st.sel_cnt == 0xffffffffu) {  // read by every thread alike
        csync();
        return false;
    }
    if (ctid == 0) {
        rng[row] = st.thr2;
        if (out_ids) out_ids[row] = key_id(cand[st.sel_cnt]);
    }
    csync();
    return true;
}

// f64 tail of sample_token (src/sample.cpp:52-101) over the sorted shortlist
// cand[0..kk): softmax in shortlist order, nucleus prefix, inverse-CDF draw.
// `prob` holds kk doubles of scratch.  Generic pointers: shared or global.
__device__ void finalize_row(CandState& st, const uint64_t* cand, double* prob, uint32_t kk,
                             const RowPlan& rp, bool x0_nan, bool have_lse, float lse_m,
                             float lse_s, int row, uint64_t* rng, int32_t* out_ids,
                             RowInfo* info, int32_t* cand_ids, double* cand_probs,
                             int32_t cand_ld, int ctid) {
    const Params& p = rp.p;
    const float inv_t_lse = rp.greedy ? 1.0f : 1.0f / p.temp;
    if (rp.greedy) {
        if (ctid == 0) {
            const int32_t id = (x0_nan || kk == 0) ? 0 : key_id(cand[0]);
            if (out_ids) out_ids[row] = id;
            if (info) {
                RowInfo ri;
                ri.max_logit = x0_nan ? __int_as_float(0x7fc00000) : (kk ? key_value(cand[0]) : 0.0f);
                ri.k = 0;
                ri.m = 0;
                ri.pos = -1;
                ri.r = 0.0;
                ri.sum = 0.0;
                ri.boundary = 0.0;
                // relative to the row's f32 max, which is the greedy pick
                ri.log_z = (have_lse && !x0_nan)
                               ? log((double)lse_s) + ((double)lse_m - (double)ri.max_logit) * (double)inv_t_lse
                               : __longlong_as_double(0x7ff8000000000000ll);
                info[row] = ri;
            }
        }
        csync();
        return;
    }
    ZS_CHECK(kk <= 2048u || prob != reinterpret_cast<double*>(st.cand + kProbOffset), 12, kk);
    const float inv_temp = 1.0f / p.temp;
    const float max_l = (x0_nan || kk == 0) ? __int_as_float(0x7fc00000) : key_value(cand[0]);
    if (kk > kBlockedTail) {
        // long shortlists: the exponent in double, exp itself in f32 (relative
        // error about 1e-7, far inside the 1e-5 probability rule); four keys loaded
        // ahead of the stores, which may alias them as far as the compiler knows
        for (uint32_t c0 = 0; c0 < kk; c0 += 4 * kNC) {
            uint64_t k4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t i = c0 + j * kNC + ctid;
                k4[j] = i < kk ? cand[i] : 0ull;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t i = c0 + j * kNC + ctid;
                if (i < kk)
                    prob[i] = (double)expf(
                        (float)(((double)key_value(k4[j]) - (double)max_l) * (double)inv_temp));
            }
        }
    } else {
        for (uint32_t i = ctid; i < kk; i += kNC)
            prob[i] = exp(((double)key_value(cand[i]) - (double)max_l) * (double)inv_temp);
    }
    csync();
    if (kk > kBlockedTail) {
        finalize_blocked(st, cand, prob, kk, p, max_l, inv_temp, have_lse, x0_nan, lse_m, lse_s,
                         row, rng, out_ids, info, cand_ids, cand_probs, cand_ld, ctid);
        return;
    }
    if (info == nullptr && !(cand_ld > 0 && (cand_ids != nullptr || cand_probs != nullptr)) &&
        kk >= kFastTailMin && fast_tail(st, cand, prob, kk, p, row, rng, out_ids, ctid))
        return;
    if (ctid == 0) {
        st.d_sum = seq_sum(prob, kk);
    }
    csync();
    const double sum = st.d_sum;
    for (uint32_t i = ctid; i < kk; i += kNC) {
        const double pi = prob[i] / sum;
        prob[i] = pi;
        if ((int32_t)i < cand_ld) {
            if (cand_ids) cand_ids[(int64_t)row * cand_ld + i] = key_id(cand[i]);
            if (cand_probs) cand_probs[(int64_t)row * cand_ld + i] = pi;
        }
    }
    csync();
    const bool nucleus = p.top_p < 1.0f;
    if (ctid == 0) {
        int m = (int)kk;
        double rescale = 1.0;
        if (nucleus) {
            double acc = 0.0;
            m = seq_nucleus(prob, (int)kk, (double)p.top_p, acc);
            // The reference's rescale loop adds prob[0..m) in the same order from 0,
            // so its sum is acc itself (prob[0] when no entry was taken).
            if (m == 0) {
                m = 1;
                rescale = prob[0];
            } else {
                rescale = acc;
            }
        }
        st.m = m;
        st.d_rescale = rescale;
    }
    csync();
    const int m = st.m;
    if (nucleus) {
        const double rs = st.d_rescale;
        for (int i = ctid; i < m; i += kNC) prob[i] /= rs;
        csync();
    }
    if (ctid == 0) {
        uint64_t s = rng[row];
        const double r = rng_uniform(s);
        rng[row] = s;
        double acc = 0.0, prev = 0.0;
        const int hit_at = seq_cdf(prob, m, r, acc, prev);
        const bool hit = hit_at >= 0;
        const int pos = hit ? hit_at : m - 1;
        double d;
        if (hit) {
            const double da = r - prev, db = acc - r;
            d = da < db ? da : db;
        } else {
            d = r - acc;
        }
        ZS_CHECK(pos < (int)kk || kk == 0, 17, ((uint64_t)(uint32_t)pos << 32) | kk);
        if (out_ids) out_ids[row] = (kk == 0) ? 0 : key_id(cand[pos < 0 ? 0 : pos]);
        if (info) {
            RowInfo ri;
            ri.max_logit = max_l;
            ri.k = (int32_t)kk;
            ri.m = m;
            ri.pos = pos;
            ri.r = r;
            ri.sum = sum;
            ri.boundary = d;
            ri.log_z = (have_lse && !x0_nan)
                           ? log((double)lse_s) + ((double)lse_m - (double)max_l) * (double)inv_temp
                           : __longlong_as_double(0x7ff8000000000000ll);
            info[row] = ri;
        }
    }
    csync();
}

// The partial blocks of one row: S slice blocks of zs_select_kernel, or the
// blocks of the warps whose shares cover the row (zs_wselect_kernel, in the
// layout of the row's warp configuration).
struct BlockSet {
    int32_t n;       // blocks per rank
    int32_t w_lo;    // first warp (warp layout)
    int64_t stride;  // bytes per block
    bool warp;
    WLayout L;       // warp layout
};

__device__ __forceinline__ BlockSet row_blocks(const MergeArgs& a, int row, const RowPlan& rp) {
    BlockSet bs;
    bs.warp = !a.force_slices && (rp.wfast || rp.wbig);
    if (bs.warp) {
        bs.L = a.wl[rp.wfast ? WCfgS::kClass : WCfgL::kClass];
        const int64_t x0 = (int64_t)row * bs.L.Vn;
        bs.w_lo = wl_warp_of(bs.L.E, bs.L.NW, x0);
        const int32_t w_hi = wl_warp_of(bs.L.E, bs.L.NW, x0 + bs.L.Vn - 1);
        bs.n = w_hi - bs.w_lo + 1;
        bs.stride = bs.L.stride;
    } else {
        bs.w_lo = 0;
        bs.n = a.S;
        bs.stride = a.part_stride;
    }
    return bs;
}

// Block idx of rank g for `row`; nullptr for a warp whose share is empty.
__device__ __forceinline__ const uint8_t* block_at(const MergeArgs& a, const BlockSet& bs, int g,
                                                   int row, int idx) {
    const uint8_t* base = a.gathered + (int64_t)g * a.rank_stride;
    if (!bs.warp) return base + ((int64_t)row * a.S + idx) * a.part_stride;
    const int32_t w = bs.w_lo + idx;
    const int64_t b0 = wl_bound(bs.L.E, bs.L.NW, w), b1 = wl_bound(bs.L.E, bs.L.NW, w + 1);
    if (b0 >= b1) return nullptr;
    const int32_t j = row - (int32_t)(b0 / bs.L.Vn);
    return base + bs.L.off + ((int64_t)w * bs.L.P + j) * bs.L.stride;
}

// Streams the keys of partial blocks (unsorted; 0 = removed) through the
// threshold filter and leaves the exact top-ksel, sorted, in st.cand[0..kk).
// Also merges the partials' sum-exp scalars and id-0 flags.  Returns kk.  Runs
// in its own launch, after every partial block is complete; each header is
// read once by thread 0 and shared, so all threads take the same path.
__device__ uint32_t merge_partials(CandState& st, const MergeArgs& a, const BlockSet& bs,
                                   int row, uint32_t ksel, float lse_c, bool& x0_nan,
                                   float& lse_m, float& lse_s, int ctid) {
    const int lane = ctid & 31;
    const uint32_t cap = (uint32_t)((bs.stride - kPartialHeaderBytes) / 8);
    const int nb = a.G * bs.n;
    if (ctid == 0) st.spec_ord = 0u;
    csync();
    if (nb <= kNC) {
        // Every block header at once (one thread each), offsets by a scan, then
        // all keys gathered in parallel: one memory latency per phase instead of
        // one per block.
        const uint8_t* pp = nullptr;
        uint32_t c = 0u;
        float m = -INFINITY, sx = 0.0f;
        bool z = false;
        if (ctid < nb) {
            pp = block_at(a, bs, ctid / bs.n, row, ctid % bs.n);
            if (pp != nullptr) {
                uint4 hv = __ldcg(reinterpret_cast<const uint4*>(pp));
                if (!ZS_CHECK(hv.x <= cap, 8, ((uint64_t)row << 32) | hv.x)) hv.x = 0u;
                c = hv.x < cap ? hv.x : cap;
                m = __uint_as_float(hv.z);
                sx = __uint_as_float(hv.w);
                z = (hv.y & kPartHasId0) && (hv.y & kPartX0Nan);
                if (hv.y & kPartSpec) {
                    atomicMax(&st.spec_ord, hv.z);
                    m = -INFINITY;  // that word is the threshold, not a log-sum-exp
                    sx = 0.0f;
                }
            }
        }
        uint32_t tot;
        const uint32_t incl = block_incl_scan(c, st.scan, ctid, tot);
        if (tot + kCandMargin <= (uint32_t)kCandCap) {  // tot is the same on every thread
            st.hist[ctid] = incl - c;
            st.prop[ctid] = reinterpret_cast<uint64_t>(pp);
            csync();
            // four keys per thread per round: their loads are in flight together
            for (uint32_t i0 = ctid; i0 < tot; i0 += 4 * kNC) {
                unsigned long long kv[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t i = i0 + j * kNC;
                    kv[j] = 0ull;
                    if (i < tot) {
                        int lo = 0, hi = nb - 1;  // the last block starting at or before i
                        while (lo < hi) {
                            const int mid = (lo + hi + 1) >> 1;
                            if (st.hist[mid] <= i) lo = mid;
                            else hi = mid - 1;
                        }
                        const unsigned long long* keys = reinterpret_cast<const unsigned long long*>(
                            st.prop[lo] + kPartialHeaderBytes);
                        kv[j] = __ldcg(keys + (i - st.hist[lo]));
                    }
                }
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (i0 + j * kNC < tot) st.cand[i0 + j * kNC] = kv[j];
            }
            block_lse(st, m, sx, lse_c, ctid);
            x0_nan = csync_or(z);
            lse_m = st.lse_m;
            lse_s = st.lse_s;
            uint32_t n = tot;
            if (!bs.warp) {
                n = keep_at_least(st, n, 1ull, ctid);  // zero keys mark removed candidates
            } else {
                if (ctid == 0) st.count = n;
                csync();
            }
            // up to kNC keys are ranked whole (the shortlist is their prefix), which
            // is cheaper than selecting the top-ksel first
            if (n > ksel && n > (uint32_t)kNC) {
                compact_select(st, n, ksel, ctid);
                n = st.count;
            }
            sort_desc(st, n, ctid);
            return n < ksel ? n : ksel;
        }
        csync();
    }
    if (ctid == 0) st.count = 0u;
    uint64_t tau = 0ull;
    bool full = false;  // same on every thread: no room for another chunk
    float M = -INFINITY, Sx = 0.0f;
    bool nan0 = false;
    for (int g = 0; g < a.G; ++g) {
        for (int s = 0; s < bs.n; ++s) {
            const uint8_t* pp = block_at(a, bs, g, row, s);
            if (pp == nullptr) continue;  // the same on every thread
            if (ctid == 0) {
                uint4 hv = __ldcg(reinterpret_cast<const uint4*>(pp));
                if (!ZS_CHECK(hv.x <= cap, 8, ((uint64_t)row << 32) | hv.x)) hv.x = 0u;
                hv.x = hv.x < cap ? hv.x : cap;
                st.part_hdr = hv;
            }
            csync();
            const uint4 hv = st.part_hdr;
            csync();
            const uint32_t cnt = hv.x, flags = hv.y;
            if (flags & kPartSpec) {
                if (ctid == 0 && hv.z > st.spec_ord) st.spec_ord = hv.z;
            } else {
                lse_merge(M, Sx, __uint_as_float(hv.z), __uint_as_float(hv.w), lse_c);
            }
            if ((flags & kPartHasId0) && (flags & kPartX0Nan)) nan0 = true;
            const unsigned long long* keys =
                reinterpret_cast<const unsigned long long*>(pp + kPartialHeaderBytes);
            for (uint32_t b = 0; b < cnt; b += kNC) {
                if (full) tau = compact_select(st, st.count, ksel, ctid);
                const uint32_t i = b + ctid;
                const uint64_t k = (i < cnt) ? __ldcg(keys + i) : 0ull;
                warp_append(st, k > tau, k, lane);
                // Each thread tests the count after its own append; the OR is exact.
                full = csync_or(st.count + kNC + kCandMargin > (uint32_t)kCandCap);
            }
        }
    }
    csync();
    uint32_t n = st.count;
    if (n > ksel) {
        compact_select(st, n, ksel, ctid);
        n = st.count;
    }
    sort_desc(st, n, ctid);
    x0_nan = nan0;
    lse_m = M;
    lse_s = Sx;
    return n < ksel ? n : ksel;
}

// ---------------------------------------------------------------------------
// The streaming kernel
// ---------------------------------------------------------------------------

__device__ __forceinline__ void set_status(int* status, int code) {
    if (status) atomicExch(status, code);
}

__device__ void producer_loop(FastSmem& sm, const Args& a) {
    const uint64_t pol = l2_evict_first_policy();
    int stage = 0;
    uint32_t eparity = 1u;  // fresh barriers: the phase "before" completes immediately
    uint32_t pending = 0u;  // stages with a copy issued whose completion we have not seen
    uint32_t pend_parity = 0u;
    bool ok = true;
    const int n_work = a.redo ? (int)*(volatile unsigned*)a.fail_count : a.n_units;
    for (int w = blockIdx.x; w < n_work && ok; w += gridDim.x) {
        const int u = a.redo ? a.fail_units[w] : w;
        const int row = u / a.S;
        const RowPlan rp = plan_row(load_params(a.row_params, a.shared, row), a.V_total, a.hist,
                                    a.hist_len, a.hist_ld, row);
        if (!rp.fast) continue;
        const UnitGeom g = unit_geom(a, u);
        const int span = g.e1 - g.e0;
        const int ntiles = span > 0 ? (span + kTileElems - 1) / kTileElems : 0;
        const float* src_row = a.logits + (int64_t)row * a.ld;
        int t = 0;
        do {
            if (!mbar_wait_bounded(&sm.empty[stage], eparity)) {
                ok = false;
                break;
            }
            const int start = g.e0 + t * kTileElems;
            const int n = ntiles ? min(kTileElems, g.e1 - start) : 0;
            StageMeta md;
            md.unit = u;
            md.start = start;
            md.n = n;
            md.flags = (t == 0 ? kMetaFirst : 0) | (t >= ntiles - 1 ? kMetaLast : 0);
            sm.meta[stage] = md;
            if (n > 0) {
                mbar_arrive_expect_tx(&sm.full[stage], (uint32_t)n * 4u);
                bulk_load(sm.ring[stage], src_row + start, (uint32_t)n * 4u, &sm.full[stage], pol);
                pending |= 1u << stage;
                // this use of the stage completes full-barrier phase parity (eparity ^ 1)
                if (eparity) pend_parity &= ~(1u << stage);
                else pend_parity |= 1u << stage;
            } else {
                pending &= ~(1u << stage);
                mbar_arrive(&sm.full[stage]);
            }
            if (++stage == kStages) {
                stage = 0;
                eparity ^= 1u;
            }
        } while (++t < ntiles);
    }
    if (ok && mbar_wait_bounded(&sm.empty[stage], eparity)) {
        StageMeta md;
        md.unit = -1;
        md.start = 0;
        md.n = 0;
        md.flags = kMetaDone;
        sm.meta[stage] = md;
        // The copy this stage held before was consumed (its empty phase completed).
        pending &= ~(1u << stage);
        mbar_arrive(&sm.full[stage]);
    } else {
        // The consumers notice on their own: their next bounded wait runs out.
        set_status(a.status, kStatusTimeout);
    }
    // Leave no bulk copy in flight behind us.
    for (int s = 0; s < kStages; ++s)
        if (pending & (1u << s)) mbar_wait_bounded(&sm.full[s], (pend_parity >> s) & 1u);
}

// End of a unit: shrink the candidates to a set holding the unit's top-keff,
// patch in the repetition penalty, and write the partial block (unsorted).  The
// exact selection, order and draw happen in zs_merge_kernel.
template <bool LSE>
__device__ void end_unit(FastSmem& sm, const Args& a, const RowPlan& rp, const UnitGeom& g,
                         float lm, float ls, float lc, bool spec_used, int32_t unit, int ctid) {
    CandState& st = sm.st;
    uint32_t n = st.count;
    // Every key of the unit at or above the speculative threshold is here; with
    // fewer than keff of them the unit's top-keff is incomplete: queue a redo.
    if (spec_used && n < (uint32_t)rp.keff && ctid == 0) {
        const unsigned slot = atomicAdd(a.fail_count, 1u);
        a.fail_units[slot] = unit;
    }
    // Shrink only when the block could not hold the candidates plus the penalty
    // appends; the merge kernel selects exactly anyway.
    const uint32_t block_keys = (uint32_t)((a.part_stride - kPartialHeaderBytes) / 8);
    if (n > (uint32_t)rp.keff && n + (uint32_t)rp.win > block_keys) {
        compact_select(st, n, (uint32_t)rp.keff, ctid);
        n = st.count;
    }
    ZS_CHECK(n <= (uint32_t)kCandCap, 9, n);
    const float* row_logits = a.logits + (int64_t)g.row * a.ld;
    float M = -INFINITY, Sx = 0.0f;
    if (LSE) {
        block_lse(st, lm, ls, lc, ctid);
        M = st.lse_m;
        Sx = st.lse_s;
    }
    if (rp.penal) {
        const int32_t* window = a.hist + (int64_t)g.row * a.hist_ld + (rp.hist_len - rp.win);
        penalty_fixup(st, row_logits, window, rp.win, rp.p.repeat_penalty, a.id_offset, g.v0,
                      g.v1, a.V_total, n, LSE, M, lc, ctid);
        n = st.count;
        if (LSE) Sx = (float)((double)Sx + st.lse_delta);
    }
    const bool x0n = st.x0_nan != 0;
    ZS_CHECK(g.row >= 0 && g.row < a.B && g.s >= 0 && g.s < a.S, 15, ((uint64_t)g.row << 32) | (uint32_t)g.s);
    uint8_t* pp = a.part + ((int64_t)g.row * a.S + g.s) * a.part_stride;
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(pp + kPartialHeaderBytes);
    const uint32_t cap = (uint32_t)((a.part_stride - kPartialHeaderBytes) / 8);
    ZS_CHECK(n <= cap, 7, n);
    const uint32_t kk = n < cap ? n : cap;
    for (uint32_t i = ctid; i < kk; i += kNC) __stcg(keys + i, (unsigned long long)st.cand[i]);
    if (ctid == 0) {
        const bool has0 = (a.id_offset + g.v0 == 0) && (g.v1 > g.v0);
        uint4 hv;
        hv.x = kk;
        hv.y = (has0 ? kPartHasId0 : 0u) | ((has0 && x0n) ? kPartX0Nan : 0u);
        hv.z = __float_as_uint(M);
        hv.w = __float_as_uint(Sx);
        *reinterpret_cast<uint4*>(pp) = hv;
    }
    csync();
    if (ctid == 0) {
        st.count = 0u;
        st.x0_nan = 0;
    }
}

// Appends the components of v (ids id..id+3) that beat the threshold, one
// shared atomic per survivor.  Components strictly above tau_f beat tau_key by
// value alone; only ties with the threshold value need the id comparison.
__device__ __forceinline__ void append_lane(CandState& st, const float4& v, int32_t id,
                                            uint64_t tau_key, float tau_f) {
    const float xs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float x = xs[q];
        if (x > tau_f || (x == tau_f && make_key(x, id + q) > tau_key)) {
            const uint32_t at = atomicAdd(&st.count, 1u);
            if (ZS_CHECK(at < (uint32_t)kCandCap, 18, at)) st.cand[at] = make_key(x, id + q);
        }
    }
}

// Threshold for the first stage of a unit: each thread proposes its largest key
// among the float4s it filters (the same j0/j1 split as filter_range), and the
// keff-th largest proposal minus one is a filter key that lets at least keff keys
// of this tile through.  Returns 0 when that is not usable (too few elements, or
// the proposal is a NaN), which keeps exact per-element comparisons.
__device__ __forceinline__ uint64_t tile_threshold(CandState& st, const float4* t4, int n4,
                                                   int gid0, uint32_t keff, int lane, int warp,
                                                   int ctid) {
    uint64_t mine = 0ull;
    for (int base = warp * 32; base < n4; base += 2 * kNC) {
        const int j0 = base + lane, j1 = j0 + kNC;
        if (j0 < n4) {
            const float4 v = t4[j0];
            const int id = gid0 + 4 * j0;
            uint64_t k = make_key(v.x, id);
            uint64_t t = make_key(v.y, id + 1); k = t > k ? t : k;
            t = make_key(v.z, id + 2); k = t > k ? t : k;
            t = make_key(v.w, id + 3); k = t > k ? t : k;
            mine = k > mine ? k : mine;
        }
        if (j1 < n4) {
            const float4 v = t4[j1];
            const int id = gid0 + 4 * j1;
            uint64_t k = make_key(v.x, id);
            uint64_t t = make_key(v.y, id + 1); k = t > k ? t : k;
            t = make_key(v.z, id + 2); k = t > k ? t : k;
            t = make_key(v.w, id + 3); k = t > k ? t : k;
            mine = k > mine ? k : mine;
        }
    }
    const uint64_t T = kth_of_proposals(st, mine, keff, ctid);
    if (T == 0ull || (uint32_t)(T >> 32) == 0u) return 0ull;
    return T - 1ull;  // keys are integers: "> T-1" is ">= T"
}

// Filters float4s [j_begin, j_end) of a ring stage against the threshold.
template <bool LSE>
__device__ __forceinline__ void filter_range(CandState& st, const float4* t4, int j_begin,
                                             int j_end, int gid0, uint64_t tau_key, float tau_f,
                                             float lc, float& lm, float& ls, int lane, int warp) {
    // No usable value threshold yet (start of a unit, or the K-th best is a NaN):
    // exact key comparisons with warp-aggregated appends.
    if ((uint32_t)(tau_key >> 32) == 0u) {
        for (int base = j_begin + warp * 32; base < j_end; base += kNC) {
            const int j = base + lane;
            const bool ok = j < j_end;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (ok) v = t4[j];
            if (LSE && ok) lse_add4(lm, ls, v, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)), lc);
            append4(st, ok, v, gid0 + 4 * j, tau_key, lane);
        }
        return;
    }
    // Two float4 per thread per step: j and j + kNC.
    for (int base = j_begin + warp * 32; base < j_end; base += 2 * kNC) {
        const int j0 = base + lane, j1 = j0 + kNC;
        const bool ok0 = j0 < j_end, ok1 = j1 < j_end;
        float4 v0 = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY), v1 = v0;
        if (ok0) v0 = t4[j0];
        if (ok1) v1 = t4[j1];
        if (LSE) {
            if (ok0) lse_add4(lm, ls, v0, fmaxf(fmaxf(v0.x, v0.y), fmaxf(v0.z, v0.w)), lc);
            if (ok1) lse_add4(lm, ls, v1, fmaxf(fmaxf(v1.x, v1.y), fmaxf(v1.z, v1.w)), lc);
        }
        const bool h0 = ok0 && ((v0.x >= tau_f) | (v0.y >= tau_f) | (v0.z >= tau_f) | (v0.w >= tau_f));
        const bool h1 = ok1 && ((v1.x >= tau_f) | (v1.y >= tau_f) | (v1.z >= tau_f) | (v1.w >= tau_f));
        // A warp-uniform branch around the rare append path: without the vote the
        // compiler predicates it, and every warp issues it on every step.
        if (__any_sync(kFull, h0 | h1)) {
            if (h0) append_lane(st, v0, gid0 + 4 * j0, tau_key, tau_f);
            if (h1) append_lane(st, v1, gid0 + 4 * j1, tau_key, tau_f);
        }
    }
}

// One thread waits for the stage; everyone else sleeps on the named barrier,
// which also ORs each thread's `want` into `any_want` (the same for everyone).
// Returns false (for every thread) when the wait ran out.
__device__ __forceinline__ bool stage_ready(FastSmem& sm, int stage, uint32_t parity,
                                            const Args& a, int ctid, bool want, bool& any_want) {
    if (ctid == 0 && !mbar_wait_bounded(&sm.full[stage], parity)) {
        *(volatile int32_t*)&sm.st.abort = 1;
        set_status(a.status, kStatusTimeout);
    }
    any_want = csync_or(want);
    if (*(volatile int32_t*)&sm.st.abort) return false;
    mbar_try_wait(&sm.full[stage], parity);  // completed: acquires the stage for this thread
    return true;
}

template <bool LSE>
__device__ void consumer_loop(FastSmem& sm, const Args& a, int ctid) {
    CandState& st = sm.st;
    const int lane = ctid & 31, warp = ctid >> 5;
    int stage = 0;
    uint32_t fparity = 0u;
    uint64_t tau_key = 0ull;
    float tau_f = -INFINITY;
    float lm = -INFINITY, ls = 0.0f, lc = 1.4426950408889634f;
    uint32_t compact_at = (uint32_t)(kCandCap - kTileElems - kCandMargin);
    bool two_pass = false;
    // Speculative threshold: after the first stage, raise the threshold to the
    // spec_k-th best key seen so far (spec_k well below keff, scaled by the share
    // of the unit that stage covers).  If fewer than keff keys of the unit end up
    // above it, the guess was too high and the unit is redone without it.
    bool spec_pending = false, spec_used = false;
    uint32_t spec_k = 0;
    int32_t cur_unit = 0;
    RowPlan rp;
    UnitGeom g;
    rp.fast = false;
    g.row = 0;
    bool compact_now = false;
    if (!stage_ready(sm, stage, fparity, a, ctid, false, compact_now)) return;
    for (;;) {
        const StageMeta md = sm.meta[stage];
        if (md.flags & kMetaDone) break;
#ifdef ZS_DEBUG_CHECKS
        if (!ZS_CHECK(md.unit >= 0 && md.unit < a.n_units && md.n >= 0 && md.n <= kTileElems &&
                          (md.flags & ~(kMetaFirst | kMetaLast)) == 0,
                      13, ((uint64_t)(uint32_t)md.unit << 32) | (uint32_t)md.flags)) {
            set_status(a.status, kStatusTimeout);
            return;
        }
#endif
        const float* row_logits;
        if (md.flags & kMetaFirst) {
            g = unit_geom(a, md.unit);
            ZS_CHECK(g.row >= 0 && g.row < a.B && g.v0 >= 0 && g.v0 <= g.v1 && g.v1 <= a.V && g.e0 <= g.e1,
                     14, ((uint64_t)(uint32_t)g.row << 32) | (uint32_t)g.v0);
            rp = plan_row(load_params(a.row_params, a.shared, g.row), a.V_total, a.hist,
                          a.hist_len, a.hist_ld, g.row);
            tau_key = 0ull;
            tau_f = -INFINITY;
            lm = -INFINITY;
            ls = 0.0f;
            lc = (rp.greedy ? 1.0f : 1.0f / rp.p.temp) * 1.4426950408889634f;
            two_pass = rp.keff > kOnePassMaxKeff;
            cur_unit = md.unit;
            {
                const uint64_t n_unit = (uint64_t)(g.v1 - g.v0);
                const uint64_t n_first = (uint64_t)md.n + (uint64_t)(g.e0 - g.v0);
                spec_k = n_unit ? (uint32_t)(((uint64_t)rp.keff * n_first * 8 + n_unit - 1) / n_unit) + 8u
                                : 0u;
                spec_pending = !a.redo && n_unit >= 4ull * (uint64_t)rp.keff &&
                               spec_k < (uint32_t)rp.keff;
                spec_used = false;
            }
            compact_at = min((uint32_t)(kCandCap - (two_pass ? kHalfElems : kTileElems) - kCandMargin),
                             (uint32_t)rp.keff + slack_for((uint32_t)rp.keff) +
                                 (uint32_t)max(rp.keff, two_pass ? kCompactMinGrowth : kCompactGrowthSmall));
            row_logits = a.logits + (int64_t)g.row * a.ld;
            for (int i = g.v0 + ctid; i < g.e0; i += kNC) {
                const float x = row_logits[i];
                if (LSE) lse_add1(lm, ls, x, lc);
                single_append(st, x, a.id_offset + i, tau_key);
            }
            if (ctid == 0 && a.id_offset + g.v0 == 0 && g.v1 > g.v0) {
                const float x0 = row_logits[0];
                st.x0_nan = (x0 != x0) ? 1 : 0;
            }
        }
        row_logits = a.logits + (int64_t)g.row * a.ld;
        ZS_CHECK(md.n <= kTileElems && md.start >= 0 && md.start + md.n <= a.V, 10,
                 ((uint64_t)md.start << 32) | (uint32_t)md.n);
        const float4* t4 = reinterpret_cast<const float4*>(sm.ring[stage]);
        const int n4 = md.n >> 2;
        const int gid0 = a.id_offset + md.start;
        if (!two_pass) {
            if (tau_key == 0ull && (uint32_t)rp.keff <= kGroupMaxK) {
                // Threshold from this stage before filtering it: the keff-th largest
                // of the per-thread maxima over this stage's float4s.
                tau_key = tile_threshold(st, t4, n4, gid0, (uint32_t)rp.keff, lane, warp, ctid);
                tau_f = tau_value(tau_key);
            }
            filter_range<LSE>(st, t4, 0, n4, gid0, tau_key, tau_f, lc, lm, ls, lane, warp);
        } else {
            // Large shortlists: two half-stage passes, with the buffer check between.
            const int h = n4 < kHalfElems / 4 ? n4 : kHalfElems / 4;
            filter_range<LSE>(st, t4, 0, h, gid0, tau_key, tau_f, lc, lm, ls, lane, warp);
            if (n4 > h) {
                if (csync_or(st.count >= compact_at)) {
                    tau_key = compact_select(st, st.count, (uint32_t)rp.keff, ctid);
                    tau_f = tau_value(tau_key);
                }
                filter_range<LSE>(st, t4, h, n4, gid0, tau_key, tau_f, lc, lm, ls, lane, warp);
            }
        }
        const bool last = (md.flags & kMetaLast) != 0;
        if (last) {
            for (int i = g.e1 + ctid; i < g.v1; i += kNC) {
                const float x = row_logits[i];
                if (LSE) lse_add1(lm, ls, x, lc);
                single_append(st, x, a.id_offset + i, tau_key);
            }
        }
        const int prev = stage;
        if (++stage == kStages) {
            stage = 0;
            fparity ^= 1u;
        }
        // The next stage was issued long ago (its slot was freed kStages tiles back),
        // so thread 0 can wait for it before the barrier that ends this tile.  Each
        // thread tests the count after its own appends; the last appender sees the
        // final count, so the OR over threads is exactly "count >= compact_at".
        const bool want = !last && st.count >= compact_at;
        if (!stage_ready(sm, stage, fparity, a, ctid, want, compact_now)) return;
        if (ctid == 0) mbar_arrive(&sm.empty[prev]);  // everyone is done with ring[prev]
        if (last) {
            end_unit<LSE>(sm, a, rp, g, lm, ls, lc, spec_used, cur_unit, ctid);
            tau_key = 0ull;
            tau_f = -INFINITY;
            csync();
        } else if (spec_pending) {
            spec_pending = false;
            const uint32_t n = st.count;  // stable: every append of the stage is in
            if (n > spec_k) {
                tau_key = compact_select(st, n, spec_k, ctid);
                tau_f = tau_value(tau_key);
                spec_used = true;
            }
        } else if (compact_now) {
            tau_key = compact_select(st, st.count, (uint32_t)rp.keff, ctid);
            tau_f = tau_value(tau_key);
        }
    }
}

template <bool LSE>
__global__ void __launch_bounds__(kThreads, 2) zs_select_kernel(const Args a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    FastSmem& sm = *reinterpret_cast<FastSmem*>(smem_raw);
    const int tid = threadIdx.x;
    grid_dep_trigger();  // the merge may be scheduled; it waits for this grid to end
    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], 1);
        }
        mbar_fence_init();
        sm.st.count = 0u;
        sm.st.abort = 0;
        sm.st.x0_nan = 0;
    }
    __syncthreads();
    if (tid >= kNC) {
        if (tid == kNC) producer_loop(sm, a);
        return;
    }
    consumer_loop<LSE>(sm, a, tid);
}

// Merge of gathered partial blocks (vocab shard): one CTA per row at a time.
template <bool LSE>
__global__ void __launch_bounds__(kNC, 3) zs_merge_kernel(const MergeArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    CandState& st = *reinterpret_cast<CandState*>(smem_raw);
    const int ctid = threadIdx.x;
    grid_dep_wait();  // the partial blocks come from the kernel before this one
    for (int row = a.row0 + blockIdx.x; row < a.row1; row += gridDim.x) {
        const RowPlan rp = plan_row(load_params(a.row_params, a.shared, row), a.V_total, a.hist,
                                    a.hist_len, a.hist_ld, row);
        if (rp.large) continue;  // drawn by zs_large_kernel
        const float lc = (rp.greedy ? 1.0f : 1.0f / rp.p.temp) * 1.4426950408889634f;
        bool x0n;
        float mm, ss;
        ZS_CHECK(rp.ksel <= kKeffFastMax, 16, rp.ksel);
        const BlockSet bs = row_blocks(a, row, rp);
        const uint32_t kk = merge_partials(st, a, bs, row, (uint32_t)rp.ksel, lc, x0n, mm, ss, ctid);
        csync();
        if (st.spec_ord != 0u) {  // the same on every thread
            // Exact only if the row's ksel-th key is at or above every block's
            // speculative threshold (all keys dropped there were below it).
            const bool fail = a.spec_redo_all || kk < (uint32_t)rp.ksel ||
                              ((uint64_t)st.spec_ord << 32) > st.cand[kk - 1];
            if (fail) {
                if (ctid == 0 && a.spec_count) a.spec_rows[atomicAdd(a.spec_count, 1u)] = row;
                csync();
                continue;
            }
        }
        finalize_row(st, st.cand, reinterpret_cast<double*>(st.cand + kProbOffset), kk, rp, x0n,
                     LSE, mm, ss, row, a.rng, a.out_ids, a.info, a.cand_ids, a.cand_probs,
                     a.cand_ld, ctid);
    }
}

// Keeps the kk largest of the unique keys keys[0..n) (n > kk >= 1, n <= 32 * R)
// at the front of keys and returns the smallest key kept.  With slack 0 that is
// exactly kk keys and the kk-th largest.  With slack > 0 the walk may stop once
// its bucket holds at most `slack` keys more than still needed, and keeps the
// whole bucket (up to kk + slack keys, *kept says how many).  The keys sit in
// registers (R per lane); a binary radix walk from the highest bit in which the
// keys differ narrows the bucket holding the kk-th key, one warp-wide count
// (redux.sync) per bit, with no shared-memory atomics.
template <int R>
struct KeyMask {  // lane masks over R register keys: 32 or 64 bits
    static_assert(R >= 1 && R <= 64, "at most 64 keys per lane");
    using T = typename std::conditional<(R > 32), unsigned long long, uint32_t>::type;
    __device__ static __forceinline__ uint32_t popc(T m) {
        return (uint32_t)(sizeof(T) == 8 ? __popcll((unsigned long long)m) : __popc((uint32_t)m));
    }
};

template <int R>
__device__ __forceinline__ uint64_t warp_topk_keep(uint64_t* keys, uint32_t n, uint32_t kk,
                                                   int lane, uint32_t slack = 0u,
                                                   uint32_t* kept = nullptr) {
    using M = typename KeyMask<R>::T;
    uint64_t k[R];
    M alive = 0;
#pragma unroll
    for (int j = 0; j < R; ++j) {
        const uint32_t i = (uint32_t)lane + 32u * j;
        const bool v = i < n;
        k[j] = v ? keys[i] : 0ull;
        alive |= (M)v << j;
    }
    uint64_t lo = ~0ull, hi = 0ull;
#pragma unroll
    for (int j = 0; j < R; ++j) {
        if ((alive >> j) & 1u) {
            lo = k[j] < lo ? k[j] : lo;
            hi = k[j] > hi ? k[j] : hi;
        }
    }
    lo = warp_min_u64(lo);
    hi = warp_max_u64(hi);
    uint64_t T = hi;
    uint32_t n_keep = 1u;
    if (kk > 1u) {
        uint32_t need = kk, cnt = n;
        for (int bit = 63 - __clzll((long long)(lo ^ hi)); bit >= 0 && cnt - need > slack; --bit) {
            M ones = 0;
#pragma unroll
            for (int j = 0; j < R; ++j) ones |= (M)((k[j] >> bit) & 1ull) << j;
            ones &= alive;
            const uint32_t c1 = __reduce_add_sync(kFull, KeyMask<R>::popc(ones));
            if (c1 >= need) {
                alive = ones;
                cnt = c1;
            } else {
                alive &= ~ones;
                need -= c1;
                cnt -= c1;
            }
        }
        // The whole bucket is kept: its minimum is the kk-th key when the bucket
        // holds exactly the keys still needed, else at most `slack` more pass.
        uint64_t m = ~0ull;
#pragma unroll
        for (int j = 0; j < R; ++j)
            if ((alive >> j) & 1u) m = k[j] < m ? k[j] : m;
        T = warp_min_u64(m);
        n_keep = kk - need + cnt;
    }
    if (kept) *kept = n_keep;
    M keep = 0;
#pragma unroll
    for (int j = 0; j < R; ++j) keep |= (M)(k[j] >= T) << j;  // padding keys are 0 < T
    const uint32_t c = KeyMask<R>::popc(keep);
    uint32_t incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += t;
    }
    __syncwarp();  // every lane has its keys in registers before any is overwritten
    uint32_t at = incl - c;
#pragma unroll
    for (int j = 0; j < R; ++j)
        if ((keep >> j) & 1u) keys[at++] = k[j];
    __syncwarp();
    return T;
}

// warp_topk_keep at the smallest register width that holds n keys: the walk's
// cost per bit grows with the width, and most compactions see a few hundred keys
// in a buffer sized for thousands.
template <int RMAX>
__device__ __forceinline__ uint64_t warp_topk_keep_fit(uint64_t* keys, uint32_t n, uint32_t kk,
                                                       int lane, uint32_t slack = 0u,
                                                       uint32_t* kept = nullptr) {
    if (RMAX > 8 && n <= 256u) return warp_topk_keep<8>(keys, n, kk, lane, slack, kept);
    return warp_topk_keep<RMAX>(keys, n, kk, lane, slack, kept);
}

// ---------------------------------------------------------------------------
// Warp-per-row merge for shortlists up to kWarpMergeMaxK: each warp merges one
// row's partial blocks in its own shared-memory slot with warp-synchronous
// steps only (no block barriers), so a CTA keeps eight rows in flight.
// ---------------------------------------------------------------------------
constexpr int kWarpCap = 512;               // candidate keys per warp (4 KB: every CTA resident)
constexpr uint32_t kWarpMergeMaxK = 256;

struct WarpSlot {
    uint64_t cand[kWarpCap];
};

struct WarpMergeSmem {
    WarpSlot w[kConsumerWarps];
};

// Keeps the keys >= T of keys[0..n) at the front (in order); returns how many.
__device__ uint32_t warp_keep(uint64_t* keys, uint32_t n, uint64_t T, int lane) {
    uint32_t out = 0;
    const unsigned below = lanemask_lt();
    for (uint32_t b = 0; b < n; b += 32) {
        const uint32_t i = b + lane;
        const uint64_t k = i < n ? keys[i] : 0ull;
        const bool keep = i < n && k >= T;
        const unsigned m = __ballot_sync(kFull, keep);
        __syncwarp();
        if (keep) keys[out + __popc(m & below)] = k;
        out += __popc(m);
        __syncwarp();
    }
    return out;
}

// Sorts keys[0..n) descending, n <= 256, with the smallest network that holds n.
__device__ __forceinline__ void warp_sort256_desc(uint64_t* keys, uint32_t n, int lane) {
    if (n <= 1u) return;
    if (n <= 32u) warp_sort_desc_slots<32>(keys, n, lane);
    else if (n <= 64u) warp_sort_desc_slots<64>(keys, n, lane);
    else if (n <= 128u) warp_sort_desc_slots<128>(keys, n, lane);
    else warp_sort_desc_slots<256>(keys, n, lane);
}

// fast_tail for one warp (kk <= 256: at most 8 terms a lane): the same parallel
// prefix sums and the same certification, with shuffles and votes in place of
// shared memory.  Returns whether it drew (the same on every lane).
__device__ bool warp_fast_tail(const uint64_t* cand, const double* e, uint32_t kk, const Params& p,
                               int row, uint64_t* rng, int32_t* out_ids, int lane) {
    const uint32_t per = (kk + 31u) / 32u;
    const uint32_t s0 = min(kk, (uint32_t)lane * per), s1 = min(kk, s0 + per);
    double seg = 0.0;
    for (uint32_t i = s0; i < s1; ++i) seg += e[i];
    double inc = seg;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(kFull, inc, o);
        if (lane >= o) inc += t;
    }
    const double T = __shfl_sync(kFull, inc, 31);
    const double pre = inc - seg;
    if (!(T > 0.0) || !(T < INFINITY)) return false;  // NaN or inf terms (uniform)
    uint64_t sr = 0ull;
    double r = 0.0;
    if (lane == 0) {
        sr = rng[row];
        r = rng_uniform(sr);  // not stored unless certified
    }
    r = __shfl_sync(kFull, r, 0);
    bool bad = false;
    uint32_t m = kk;
    double Em = T;
    if (p.top_p < 1.0f) {
        const double top_p = (double)p.top_p;
        if (!(top_p > 0.0)) return false;  // the loop takes no term: sequential code
        double E = pre;
        int mloc = -1;
        double eloc = 0.0;
        for (uint32_t i = s0; i < s1; ++i) {
            const double Ep = E;
            E += e[i];
            const double a = Ep / T, b = E / T;
            if (a < top_p && b >= top_p) {
                if (!(a < top_p - kTailMargin && b >= top_p + kTailMargin)) bad = true;
                mloc = (int)(i + 1);
                eloc = E;
            }
        }
        if (s1 == kk && s0 < s1 && E / T < top_p && !(E / T < top_p - kTailMargin)) bad = true;
        const unsigned hit = __ballot_sync(kFull, mloc >= 0);
        if (hit) {
            const int src = __ffs(hit) - 1;
            m = (uint32_t)__shfl_sync(kFull, mloc, src);
            const double em = __shfl_sync(kFull, eloc, src);
            if (m < kk) Em = em;
        }
    }
    int pos = -1;
    {
        double E = pre;
        for (uint32_t i = s0; i < s1 && i < m; ++i) {
            const double Ep = E;
            E += e[i];
            const double a = Ep / Em, b = E / Em;
            if (a <= r && r < b) {
                if (!(a < r - kTailMargin && b > r + kTailMargin)) bad = true;
                pos = (int)i;
            }
        }
    }
    const unsigned found = __ballot_sync(kFull, pos >= 0);
    if (__any_sync(kFull, bad) || found == 0u) return false;
    pos = __shfl_sync(kFull, pos, __ffs(found) - 1);
    if (lane == 0) {
        rng[row] = sr;
        if (out_ids) out_ids[row] = key_id(cand[pos]);
    }
    __syncwarp();
    return true;
}

// f64 tail of sample_token (src/sample.cpp:52-101) over the sorted shortlist
// cand[0..kk), by one warp: the same expressions and summation order as
// finalize_row (sequential sums on lane 0).
__device__ void warp_finalize(const uint64_t* cand, double* prob, uint32_t kk, const RowPlan& rp,
                              bool x0_nan, bool have_lse, float lse_m, float lse_s, int row,
                              uint64_t* rng, int32_t* out_ids, RowInfo* info, int32_t* cand_ids,
                              double* cand_probs, int32_t cand_ld, int lane) {
    const Params& p = rp.p;
    const double qnan = __longlong_as_double(0x7ff8000000000000ll);
    if (rp.greedy) {
        if (lane == 0) {
            const int32_t id = (x0_nan || kk == 0) ? 0 : key_id(cand[0]);
            if (out_ids) out_ids[row] = id;
            if (info) {
                RowInfo ri;
                ri.max_logit = x0_nan ? __int_as_float(0x7fc00000) : (kk ? key_value(cand[0]) : 0.0f);
                ri.k = 0;
                ri.m = 0;
                ri.pos = -1;
                ri.r = 0.0;
                ri.sum = 0.0;
                ri.boundary = 0.0;
                ri.log_z = (have_lse && !x0_nan)
                               ? log((double)lse_s) + ((double)lse_m - (double)ri.max_logit)
                               : qnan;
                info[row] = ri;
            }
        }
        __syncwarp();
        return;
    }
    const float inv_temp = 1.0f / p.temp;
    const float max_l = (x0_nan || kk == 0) ? __int_as_float(0x7fc00000) : key_value(cand[0]);
    for (uint32_t i = lane; i < kk; i += 32)
        prob[i] = exp(((double)key_value(cand[i]) - (double)max_l) * (double)inv_temp);
    __syncwarp();
    if (info == nullptr && !(cand_ld > 0 && (cand_ids != nullptr || cand_probs != nullptr)) &&
        kk >= kFastTailMin && warp_fast_tail(cand, prob, kk, p, row, rng, out_ids, lane))
        return;
    double sum = 0.0;
    if (lane == 0) sum = seq_sum(prob, kk);
    sum = __shfl_sync(kFull, sum, 0);
    for (uint32_t i = lane; i < kk; i += 32) {
        const double pi = prob[i] / sum;
        prob[i] = pi;
        if ((int32_t)i < cand_ld) {
            if (cand_ids) cand_ids[(int64_t)row * cand_ld + i] = key_id(cand[i]);
            if (cand_probs) cand_probs[(int64_t)row * cand_ld + i] = pi;
        }
    }
    __syncwarp();
    const bool nucleus = p.top_p < 1.0f;
    int m = (int)kk;
    double rescale = 1.0;
    if (lane == 0 && nucleus) {
        double acc = 0.0;
        m = seq_nucleus(prob, (int)kk, (double)p.top_p, acc);
        // the reference's rescale loop repeats these additions: its sum is acc
        if (m == 0) {
            m = 1;
            rescale = prob[0];
        } else {
            rescale = acc;
        }
    }
    m = __shfl_sync(kFull, m, 0);
    rescale = __shfl_sync(kFull, rescale, 0);
    if (nucleus) {
        for (int i = lane; i < m; i += 32) prob[i] /= rescale;
        __syncwarp();
    }
    if (lane == 0) {
        uint64_t st = rng[row];
        const double r = rng_uniform(st);
        rng[row] = st;
        double acc = 0.0, prev = 0.0;
        const int hit_at = seq_cdf(prob, m, r, acc, prev);
        const bool hit = hit_at >= 0;
        const int pos = hit ? hit_at : m - 1;
        double d;
        if (hit) {
            const double da = r - prev, db = acc - r;
            d = da < db ? da : db;
        } else {
            d = r - acc;
        }
        if (out_ids) out_ids[row] = (kk == 0) ? 0 : key_id(cand[pos < 0 ? 0 : pos]);
        if (info) {
            RowInfo ri;
            ri.max_logit = max_l;
            ri.k = (int32_t)kk;
            ri.m = m;
            ri.pos = pos;
            ri.r = r;
            ri.sum = sum;
            ri.boundary = d;
            ri.log_z = (have_lse && !x0_nan)
                           ? log((double)lse_s) + ((double)lse_m - (double)max_l) * (double)inv_temp
                           : qnan;
            info[row] = ri;
        }
    }
    __syncwarp();
}

// One warp merges one row: reads the headers of up to 32 blocks at once (one
// lane each), gathers their keys 256 at a time into registers (so one memory
// latency covers them), keeps the candidates to the top-ksel whenever cand
// (CAP keys) fills, sorts, and runs the f64 tail and draw.  The f64
// probabilities use cand[CAP - 256 .. CAP).
template <int CAP, bool LSE>
__device__ void warp_merge_row(uint64_t* cand, const MergeArgs& a, int row, const RowPlan& rp,
                               unsigned below, int lane) {
    static_assert(CAP >= 2 * (int)kWarpMergeMaxK, "probabilities alias the top of cand");
    constexpr int J = 8;  // keys per lane per gather round
    const uint32_t ksel = (uint32_t)rp.ksel;
    const float lc = (rp.greedy ? 1.0f : 1.0f / rp.p.temp) * 1.4426950408889634f;
    const BlockSet bs = row_blocks(a, row, rp);
    const uint32_t block_cap = (uint32_t)((bs.stride - kPartialHeaderBytes) / 8);
    const int nb = a.G * bs.n;
    uint32_t count = 0;
    uint64_t tau = 0ull;
    float M = -INFINITY, Sx = 0.0f;
    bool nan0 = false;
    uint32_t spec_ord = 0u;
    for (int g0 = 0; g0 < nb; g0 += 32) {
        const int b = g0 + lane;
        unsigned long long base = 0ull;
        uint32_t c = 0u;
        float m = -INFINITY, sx = 0.0f;
        bool z = false;
        if (b < nb) {
            const uint8_t* pp = block_at(a, bs, b / bs.n, row, b % bs.n);
            if (pp != nullptr) {
                const uint4 hv = __ldcg(reinterpret_cast<const uint4*>(pp));
                c = hv.x < block_cap ? hv.x : block_cap;
                m = __uint_as_float(hv.z);
                sx = __uint_as_float(hv.w);
                z = (hv.y & kPartHasId0) && (hv.y & kPartX0Nan);
                if (hv.y & kPartSpec) {
                    spec_ord = hv.z > spec_ord ? hv.z : spec_ord;
                    m = -INFINITY;  // that word is the threshold, not a log-sum-exp
                    sx = 0.0f;
                }
                base = reinterpret_cast<unsigned long long>(pp + kPartialHeaderBytes);
            }
        }
        if (LSE) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float m2 = __shfl_xor_sync(kFull, m, o);
                const float s2 = __shfl_xor_sync(kFull, sx, o);
                lse_merge(m, sx, m2, s2, lc);
            }
            lse_merge(M, Sx, m, sx, lc);
        }
        nan0 = nan0 || __any_sync(kFull, z);
        uint32_t incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(kFull, incl, o);
            if (lane >= o) incl += t;
        }
        const uint32_t tot = __shfl_sync(kFull, incl, 31);
        // lanes past the group never own a key index
        const uint32_t off = (b < nb) ? incl - c : 0xffffffffu;
        for (uint32_t i0 = 0; i0 < tot; i0 += 32u * J) {
            uint64_t k[J];
#pragma unroll
            for (int jj = 0; jj < J; ++jj) {
                const uint32_t i = i0 + 32u * jj + (uint32_t)lane;
                int lo = 0, hi = 31;  // the last block starting at or before i
#pragma unroll
                for (int step = 0; step < 5; ++step) {
                    const int mid = (lo + hi + 1) >> 1;
                    if (__shfl_sync(kFull, off, mid) <= i) lo = mid;
                    else hi = mid - 1;
                }
                const unsigned long long bq = __shfl_sync(kFull, base, lo);
                const uint32_t oq = __shfl_sync(kFull, off, lo);
                k[jj] = (i < tot) ? __ldcg(reinterpret_cast<const unsigned long long*>(bq) + (i - oq))
                                  : 0ull;
            }
#pragma unroll
            for (int jj = 0; jj < J; ++jj) {
                if (count + 32 > (uint32_t)CAP) {
                    tau = warp_topk_keep_fit<CAP / 32>(cand, count, ksel, lane);
                    count = ksel;  // exactly ksel keys >= tau
                }
                const bool pass = k[jj] > tau;
                const unsigned mk = __ballot_sync(kFull, pass);
                if (pass) cand[count + __popc(mk & below)] = k[jj];
                count += __popc(mk);
                __syncwarp();
            }
        }
    }
    // Up to 256 keys are sorted whole (the shortlist is their prefix), which is
    // cheaper than selecting the top-ksel first; more are cut to ksel first.
    if (count > kWarpMergeMaxK) {
        warp_topk_keep_fit<CAP / 32>(cand, count, ksel, lane);
        count = ksel;
    }
    warp_sort256_desc(cand, count, lane);
    const uint32_t kk = count < ksel ? count : ksel;
    spec_ord = __reduce_max_sync(kFull, spec_ord);
    if (spec_ord != 0u) {
        // Exact only if the row's ksel-th key is at or above every block's
        // speculative threshold (all keys dropped there were below it).
        if (a.spec_redo_all || kk < ksel || ((uint64_t)spec_ord << 32) > cand[kk - 1]) {
            if (lane == 0 && a.spec_count) a.spec_rows[atomicAdd(a.spec_count, 1u)] = row;
            __syncwarp();
            return;
        }
    }
    warp_finalize(cand, reinterpret_cast<double*>(cand + (CAP - (int)kWarpMergeMaxK)), kk, rp,
                  nan0, LSE, M, Sx, row, a.rng, a.out_ids, a.info, a.cand_ids, a.cand_probs,
                  a.cand_ld, lane);
}

template <bool LSE>
__global__ void __launch_bounds__(kNC, 4) zs_warp_merge_kernel(const MergeArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    WarpMergeSmem& sm = *reinterpret_cast<WarpMergeSmem*>(smem_raw);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    WarpSlot& ws = sm.w[warp];
    const unsigned below = lanemask_lt();
    grid_dep_wait();  // the partial blocks come from the kernel before this one
    // row r goes to CTA r mod grid: spread over the SMs before doubling up in a CTA
    for (int row = a.row0 + warp * gridDim.x + blockIdx.x; row < a.row1;
         row += gridDim.x * kConsumerWarps) {
        const RowPlan rp = plan_row(load_params(a.row_params, a.shared, row), a.V_total, a.hist,
                                    a.hist_len, a.hist_ld, row);
        if (rp.large) continue;  // drawn by zs_large_kernel
        warp_merge_row<kWarpCap, LSE>(ws.cand, a, row, rp, below, lane);
    }
}

// ---------------------------------------------------------------------------
// zs_wselect_kernel: warp-independent streaming select for the rows of the warp
// path (shortlist + penalty window within the configuration's limits, WCfgS or WCfgL).
//
// Each warp owns an equal contiguous share of the batch flattened to
// B * wl_Vn columns, cut at row ends into pieces.  It streams its share through
// its own ring of kWStages 4 KB stages: lane 0 issues 1-D bulk copies (no tensor
// map, no multicast) into the stage the warp has just finished, kWStages tiles
// ahead, across piece boundaries.  Candidates live in the warp's own shared
// slot; the count and the threshold are warp-uniform registers, appends are
// ballots (no atomics), compactions exact warp radix selects.  No warp ever
// waits for another, so there is no block barrier in the kernel.  At the end of
// a piece the penalty is patched in, the piece's top-ksel (final values) is
// selected exactly, and the keys go out as one unsorted block.
// ---------------------------------------------------------------------------
template <class C>
struct __align__(128) WarpSel {
    float ring[kWStages][kWTile];
    uint64_t cand[C::kCap];
    uint32_t hist[256];  // radix histogram; the penalty window at a piece's end
    uint64_t full[kWStages];
};

template <class C>
struct WSelSmem {
    WarpSel<C> w[C::kWarps];
};

// Issue side of a warp: the next (piece, tile) to copy.  Every lane keeps the
// same cursor; lane 0 issues.
struct WIssue {
    int32_t j;
    int32_t t;
    WPiece pc;
};

struct WShare {
    int64_t b0, b1;  // flattened columns of the warp's share
    int32_t r0;      // first row
    int32_t np;      // pieces
};

template <class C>
__device__ __forceinline__ bool wl_issue(const Args& a, WarpSel<C>& ws, int stage, WIssue& is,
                                         const WShare& sh, uint64_t pol, int lane) {
    while (is.j < sh.np && is.t >= is.pc.ntiles) {
        ++is.j;
        is.t = 0;
        if (is.j < sh.np) is.pc = wl_piece(a, sh.b0, sh.b1, sh.r0, is.j);
    }
    if (is.j >= sh.np) return false;
    const int start = is.pc.e0 + is.t * kWTile;
    const int n = min(kWTile, is.pc.e1 - start);
    if (lane == 0) {
        // The warp's reads of this stage (all consumed into registers before the
        // __syncwarp that precedes this call) come before the copy's writes.
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(&ws.full[stage], (uint32_t)n * 4u);
        bulk_load(ws.ring[stage], a.logits + (int64_t)is.pc.row * a.ld + start, (uint32_t)n * 4u,
                  &ws.full[stage], pol);
    }
    ++is.t;
    return true;
}

// Ballot append of `key` where pred; count stays warp-uniform.
template <int CAP>
__device__ __forceinline__ void wappend(uint64_t* cand, uint32_t& count, bool pred, uint64_t key,
                                        unsigned below) {
    const unsigned m = __ballot_sync(kFull, pred);
    if (pred && ZS_CHECK(count + __popc(m & below) < (uint32_t)CAP, 20, count))
        cand[count + __popc(m & below)] = key;
    count += (uint32_t)__popc(m);
}

// Threshold modes of the warp filter.
constexpr int kWAll = 0;    // no threshold yet: every element is a candidate
constexpr int kWFast = 1;   // float threshold: x > tau_f, or x == tau_f with id < tau_id
constexpr int kWExact = 2;  // the threshold key is a NaN: compare whole keys

// Per-warp streaming state of one piece.
struct WState {
    uint32_t count;
    uint64_t tau_key;
    float tau_f;
    int32_t tau_id;
    int32_t mode;
    uint64_t kb;  // greedy: this lane's best key
    float vb;     // greedy: its value
    float lm, ls; // online log-sum-exp (base 2) of this lane's elements
};

// Shrinks the candidates to the exact top-keff and raises the threshold to the
// keff-th key.  For a non-NaN threshold value t, key(x, id) > key(t, tid) is
// exactly x > t, or x == t and id < tid (-0 == +0, NaN below everything).
template <class C>
__device__ __forceinline__ void wcompact(WarpSel<C>& ws, WState& w, uint32_t keff, int lane) {
    // The long configuration stops its radix walk early (keeping up to keff/4
    // keys more): with 64 keys per lane every bit of the walk is costly, and a
    // tie group at the keff-th key would otherwise send it through the id bits.
    uint32_t kept = keff;
    w.tau_key = warp_topk_keep_fit<C::kCap / 32>(ws.cand, w.count, keff, lane, C::kSlackDiv ? keff / C::kSlackDiv : 0u, &kept);
    w.count = kept;
    w.tau_f = tau_value(w.tau_key);
    w.tau_id = key_id(w.tau_key);
    w.mode = ((uint32_t)(w.tau_key >> 32) == 0u) ? kWExact : kWFast;
}

// Appends the components of v (ids id..id+3) selected by p0..p3.  Positions
// come from a bit-sliced warp prefix sum of the per-lane counts: one ballot per
// possible count, so the common step (at most one hit per lane) costs two.
template <class C>
__device__ __forceinline__ void wappend4(WarpSel<C>& ws, WState& w, const float4& v, int32_t id,
                                         bool p0, bool p1, bool p2, bool p3, unsigned below) {
    const uint32_t c = (uint32_t)p0 + (uint32_t)p1 + (uint32_t)p2 + (uint32_t)p3;
    const unsigned b1 = __ballot_sync(kFull, c >= 1u);
    const unsigned b2 = __ballot_sync(kFull, c >= 2u);
    uint32_t pos = (uint32_t)__popc(b1 & below), tot = (uint32_t)__popc(b1);
    if (b2) {
        const unsigned b3 = __ballot_sync(kFull, c >= 3u);
        const unsigned b4 = __ballot_sync(kFull, c >= 4u);
        pos += (uint32_t)(__popc(b2 & below) + __popc(b3 & below) + __popc(b4 & below));
        tot += (uint32_t)(__popc(b2) + __popc(b3) + __popc(b4));
    }
    uint32_t at = w.count + pos;
    ZS_CHECK(at + c <= (uint32_t)C::kCap, 20, at + c);
    if (p0) ws.cand[at++] = make_key(v.x, id);
    if (p1) ws.cand[at++] = make_key(v.y, id + 1);
    if (p2) ws.cand[at++] = make_key(v.z, id + 2);
    if (p3) ws.cand[at] = make_key(v.w, id + 3);
    w.count += tot;
}

// Does (x, id) beat the threshold of mode w.mode?
__device__ __forceinline__ bool wpass(const WState& w, bool ok, float x, int32_t id) {
    if (w.mode == kWFast) return ok && (x > w.tau_f || (x == w.tau_f && id < w.tau_id));
    if (w.mode == kWAll) return ok;
    return ok && make_key(x, id) > w.tau_key;
}

template <class C, bool LSE>
__device__ __forceinline__ void wfilter1(WarpSel<C>& ws, WState& w, bool ok, float x, int32_t id,
                                         bool greedy, uint32_t keff, float lc, unsigned below,
                                         int lane) {
    if (LSE && ok) lse_add1(w.lm, w.ls, x, lc);
    if (greedy) {
        if (ok && x >= w.vb) {
            const uint64_t k = make_key(x, id);
            if (k > w.kb) {
                w.kb = k;
                w.vb = x;
            }
        }
        return;
    }
    const bool p = wpass(w, ok, x, id);
    wappend<C::kCap>(ws.cand, w.count, p, make_key(x, id), below);
    if (w.count > (uint32_t)(C::kCap - kWStepElems)) wcompact(ws, w, keff, lane);
}

template <class C, bool LSE>
__device__ __forceinline__ void wfilter_tile(WarpSel<C>& ws, WState& w, const float4* t4, int n4,
                                             int32_t gid0, bool greedy, uint32_t keff, float lc,
                                             unsigned below, int lane) {
#pragma unroll 2
    for (int base = 0; base < n4; base += 32) {
        const int jj = base + lane;
        const bool ok = jj < n4;
        const float4 v = ok ? t4[jj] : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
        const int32_t id = gid0 + 4 * jj;
        if (LSE && ok) lse_add4(w.lm, w.ls, v, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)), lc);
        if (greedy) {
            // running best of this lane; strict key order keeps the first index
            const float vm = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
            if (ok && vm >= w.vb) {
                const float xs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    if (xs[q] >= w.vb) {
                        const uint64_t k = make_key(xs[q], id + q);
                        if (k > w.kb) {
                            w.kb = k;
                            w.vb = xs[q];
                        }
                    }
                }
            }
            continue;
        }
        // cheap pre-test: can any component reach the threshold value?
        const float tf = w.mode == kWFast ? w.tau_f : -INFINITY;
        const bool h = ok && (w.mode != kWFast || v.x >= tf || v.y >= tf || v.z >= tf || v.w >= tf);
        if (__any_sync(kFull, h)) {
            wappend4(ws, w, v, id, h && wpass(w, true, v.x, id), h && wpass(w, true, v.y, id + 1),
                     h && wpass(w, true, v.z, id + 2), h && wpass(w, true, v.w, id + 3), below);
            if (w.count > (uint32_t)(C::kCap - kWStepElems)) wcompact(ws, w, keff, lane);
        }
    }
}

// Threshold mode, one whole tile at a time: a 32-bit mask per lane marks the
// elements that reach the threshold value (float compares only); if any lane
// has one, the marked elements are re-read from the stage, tested exactly, and
// written at positions from one warp scan.  Returns false, having appended
// nothing, when the tile's survivors could not fit even after a compaction; the
// caller then filters it with the per-step path.
template <class C, bool LSE>
__device__ __forceinline__ bool wfilter_tile_fast(WarpSel<C>& ws, WState& w, const float* tile, int n4,
                                                  int32_t gid0, uint32_t keff, float lc, int lane) {
    const float4* t4 = reinterpret_cast<const float4*>(tile);
    const float tf = w.tau_f;
    // one bit per float4 whose largest component reaches the threshold value
    // (fmaxf ignores NaN, which never passes)
    uint32_t fmask = 0u;
#pragma unroll
    for (int q = 0; q < kWTile / kWStepElems; ++q) {
        const int jj = lane + 32 * q;
        if (jj < n4) {
            const float4 v = t4[jj];
            const float vm = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
            if (LSE) lse_add4(w.lm, w.ls, v, vm, lc);
            fmask |= (uint32_t)(vm >= tf) << q;
        }
    }
    if (!__any_sync(kFull, fmask != 0u)) return true;
    // exact test of the flagged float4s' components: bit 4q + r of em
    uint32_t em = 0u;
    for (uint32_t m = fmask; m != 0u; m &= m - 1u) {
        const int q = __ffs(m) - 1;
        const int jj = lane + 32 * q;
        const float4 v = t4[jj];
        const int32_t id = gid0 + 4 * jj;
        const float xs[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int r = 0; r < 4; ++r)
            if (xs[r] > tf || (xs[r] == tf && id + r < w.tau_id)) em |= 1u << (4 * q + r);
    }
    const uint32_t c = (uint32_t)__popc(em);
    uint32_t incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(kFull, incl, o);
        if (lane >= o) incl += t;
    }
    const uint32_t tot = __shfl_sync(kFull, incl, 31);
    if (w.count + tot > (uint32_t)C::kCap) {
        const uint32_t slack = C::kSlackDiv ? keff / C::kSlackDiv : 0u;
        if (tot > (uint32_t)C::kCap - keff - slack) return false;
        // The marked elements beat the old threshold; some may fall below the
        // new one, which costs room but not exactness (the final select is exact).
        wcompact(ws, w, keff, lane);
    }
    uint32_t at = w.count + incl - c;
    for (uint32_t m = em; m != 0u; m &= m - 1u) {
        const int b = __ffs(m) - 1;
        const int e = 4 * (lane + 32 * (b >> 2)) + (b & 3);
        ws.cand[at++] = make_key(tile[e], gid0 + e);
    }
    w.count += tot;
    __syncwarp();
    return true;
}

// Opening threshold of a piece, from its first tile: the keff-th largest of the
// tile's float4 maxima (keff <= 256, one float4 per lane and step).  Each float4
// maximum is a different element, so at least keff elements of the tile reach
// it, and nothing below it can be in the piece's top-keff.  A 32-bit radix walk
// over the maxima' ords, one redux.sync count per bit.  Returns that ord, 0 when
// it is a NaN's (no usable threshold).
__device__ __forceinline__ uint32_t wfirst_threshold(const float4* t4, int n4, uint32_t keff,
                                                     int lane) {
    constexpr int Q = kWTile / kWStepElems;
    uint32_t o[Q];
    uint32_t alive = 0u;
#pragma unroll
    for (int q = 0; q < Q; ++q) {
        const int jj = lane + 32 * q;
        o[q] = 0u;
        if (jj < n4) {
            const float4 v = t4[jj];
            o[q] = ord_of(fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
            alive |= 1u << q;
        }
    }
    uint32_t need = keff, cnt = (uint32_t)n4;
    for (int bit = 31; bit >= 0 && cnt != need; --bit) {
        uint32_t ones = 0u;
#pragma unroll
        for (int q = 0; q < Q; ++q) ones |= ((o[q] >> bit) & 1u) << q;
        ones &= alive;
        const uint32_t c1 = __reduce_add_sync(kFull, (uint32_t)__popc(ones));
        if (c1 >= need) {
            alive = ones;
            cnt = c1;
        } else {
            alive &= ~ones;
            need -= c1;
            cnt -= c1;
        }
    }
    uint32_t m = 0xffffffffu;
#pragma unroll
    for (int q = 0; q < Q; ++q)
        if ((alive >> q) & 1u) m = o[q] < m ? o[q] : m;
    return __reduce_min_sync(kFull, m);
}

// The need-th largest of the value orders o[q] (bit q of `alive`) over the warp,
// or with slack > 0 a value order at or below it with at most need + slack orders
// at or above it: a radix walk from the highest bit in which the orders differ,
// one redux.sync count per bit, stopping once its bucket is that small.
template <int Q>
__device__ __forceinline__ uint32_t warp_kth_ord(const uint32_t (&o)[Q], uint32_t alive,
                                                 uint32_t need, uint32_t cnt, uint32_t slack = 0u) {
    uint32_t lo = 0xffffffffu, hi = 0u;
#pragma unroll
    for (int q = 0; q < Q; ++q)
        if ((alive >> q) & 1u) {
            lo = o[q] < lo ? o[q] : lo;
            hi = o[q] > hi ? o[q] : hi;
        }
    lo = __reduce_min_sync(kFull, lo);
    hi = __reduce_max_sync(kFull, hi);
    for (int bit = (lo == hi) ? -1 : 31 - __clz(lo ^ hi); bit >= 0 && cnt - need > slack; --bit) {
        uint32_t ones = 0u;
#pragma unroll
        for (int q = 0; q < Q; ++q) ones |= ((o[q] >> bit) & 1u) << q;
        ones &= alive;
        const uint32_t c1 = __reduce_add_sync(kFull, (uint32_t)__popc(ones));
        if (c1 >= need) {
            alive = ones;
            cnt = c1;
        } else {
            alive &= ~ones;
            need -= c1;
            cnt -= c1;
        }
    }
    uint32_t m = 0xffffffffu;
#pragma unroll
    for (int q = 0; q < Q; ++q)
        if ((alive >> q) & 1u) m = o[q] < m ? o[q] : m;
    return __reduce_min_sync(kFull, m);
}

// Speculative opening threshold of a long piece: a sample of 32 x Q float4s in
// 128-byte chunks spread evenly over the piece's aligned columns, read with plain
// loads (the piece's stream reads those lines again soon, mostly from L2).  The
// threshold is the value order of the need-th largest sample float4 maximum, need
// four standard deviations (plus 4) above the expected number of sample elements
// at or above the piece's keff-th value: the piece then keeps about 2 to 4 x keff
// keys instead of ramping up from its first tile.  Nothing makes this exact: the
// merge checks each row against the thresholds its blocks carry.  Returns 0 when
// such a sample cannot cut the piece usefully.
template <int Q>
__device__ __forceinline__ uint32_t wspec_threshold(const float* row_logits, const WPiece& pc,
                                                    uint32_t keff, int lane) {
    static_assert(Q % 8 == 0 && Q <= 32, "sample float4s per lane");
    constexpr int S4 = 32 * Q;  // sample float4s
    constexpr int NC = S4 / 8;  // 128-byte chunks, eight lanes each
    const int64_t n4 = (pc.e1 - pc.e0) >> 2;
    if (n4 < 8 * NC || n4 > (1 << 25)) return 0u;
    const float j = (4.0f * S4) * (float)keff / (float)(pc.c1 - pc.c0);
    const uint32_t need = (uint32_t)ceilf(j + 4.0f * sqrtf(j) + 4.0f);
    if (need > (uint32_t)S4 / 4u) return 0u;  // a quarter of the sample passes: no gain
    const float4* base = reinterpret_cast<const float4*>(row_logits + pc.e0);
    // chunk c starts at float4 (n4 - 8) * c / (NC - 1): 32-bit arithmetic (a row
    // has at most 2^31 / 4 float4s; the product stays below 2^32 for NC <= 128)
    const uint32_t span = (uint32_t)(n4 - 8);
    // every chunk requested from L2 first, so the batches below wait about one
    // memory latency in all, not one each
    if ((lane & 7) == 0) {
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            const uint32_t c = 4u * q + (uint32_t)(lane >> 3);
            prefetch_l2(base + span * c / (uint32_t)(NC - 1));
        }
    }
    uint32_t o[Q];
#pragma unroll
    for (int q0 = 0; q0 < Q; q0 += 8) {
        float4 v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const uint32_t c = 4u * (q0 + q) + (uint32_t)(lane >> 3);  // this lane group's chunk
            v[q] = base[span * c / (uint32_t)(NC - 1) + (uint32_t)(lane & 7)];
        }
#pragma unroll
        for (int q = 0; q < 8; ++q)
            o[q0 + q] = ord_of(fmaxf(fmaxf(v[q].x, v[q].y), fmaxf(v[q].z, v[q].w)));
    }
    // any order with need to 1.5 x need sample maxima at or above it will do
    return warp_kth_ord<Q>(o, Q == 32 ? 0xffffffffu : ((1u << Q) - 1u), need, (uint32_t)S4,
                           need / 2u);
}

template <class C, bool LSE>
__device__ void wend_piece(const Args& a, WarpSel<C>& ws, WState& w, const WPiece& pc,
                           const RowPlan& rp, bool greedy_np, float lc, int32_t gw, int32_t j,
                           uint32_t spec_ord, unsigned below, int lane) {
    const float* row_logits = a.logits + (int64_t)pc.row * a.ld;
    if (greedy_np) {
        const uint64_t kb = warp_max_u64(w.kb);
        if (lane == 0 && kb != 0ull) ws.cand[0] = kb;
        w.count = kb != 0ull ? 1u : 0u;
        __syncwarp();
    }
    const bool has0 = (a.id_offset + pc.c0 == 0) && (pc.c1 > pc.c0);
    bool x0n = false;
    if (has0) {
        const float x0 = row_logits[0];
        x0n = (x0 != x0);
    }
    float M = -INFINITY, Sx = 0.0f;
    if (LSE) {
        M = w.lm;
        Sx = w.ls;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float m2 = __shfl_xor_sync(kFull, M, o);
            const float s2 = __shfl_xor_sync(kFull, Sx, o);
            lse_merge(M, Sx, m2, s2, lc);
        }
    }
    if (rp.penal && w.count + (uint32_t)rp.win > (uint32_t)C::kCap) {
        // keep the raw top-keff (keff = ksel + window) and make room for the window
        wcompact(ws, w, (uint32_t)rp.keff, lane);
    }
    if (rp.penal) {
        // src/sample.cpp:40-50 for the ids of this piece: raw keys out, penalised
        // values in (each entry of the window applies the penalty once more).
        int32_t* hw = reinterpret_cast<int32_t*>(ws.hist);
        const int32_t* window = a.hist + (int64_t)pc.row * a.hist_ld + (rp.hist_len - rp.win);
        for (int i = lane; i < rp.win; i += 32) hw[i] = window[i];
        __syncwarp();
        for (uint32_t i = lane; i < w.count; i += 32) {
            const int32_t id = key_id(ws.cand[i]);
            for (int q = 0; q < rp.win; ++q)
                if (hw[q] == id) {
                    ws.cand[i] = 0ull;
                    break;
                }
        }
        __syncwarp();
        w.count = warp_keep(ws.cand, w.count, 1ull, lane);
        const int32_t lo = a.id_offset + pc.c0, hi = a.id_offset + pc.c1;
        const float pen = rp.p.repeat_penalty;
        double dl = 0.0;
        bool z_hit = false, z_nan = false;
        for (int base = 0; base < rp.win; base += 32) {
            const int jw = base + lane;
            bool app = false;
            uint64_t key = 0ull;
            if (jw < rp.win) {
                const int32_t gid = hw[jw];
                if (gid >= 0 && gid < a.V_total && gid >= lo && gid < hi) {
                    bool first = true;
                    for (int q = 0; q < jw; ++q)
                        if (hw[q] == gid) {
                            first = false;
                            break;
                        }
                    if (first) {
                        int mult = 1;
                        for (int q = jw + 1; q < rp.win; ++q) mult += (hw[q] == gid) ? 1 : 0;
                        const float raw = row_logits[gid - a.id_offset];
                        float v = raw;
                        for (int c = 0; c < mult; ++c) v = (v > 0.0f) ? v / pen : v * pen;
                        key = make_key(v, gid);
                        app = true;
                        if (gid == 0) {
                            z_hit = true;
                            z_nan = (v != v);
                        }
                        if (LSE && M > -INFINITY)
                            dl += exp2(((double)v - (double)M) * (double)lc) -
                                  exp2(((double)raw - (double)M) * (double)lc);
                    }
                }
            }
            wappend<C::kCap>(ws.cand, w.count, app, key, below);
        }
        const unsigned zm = __ballot_sync(kFull, z_hit);
        if (zm) x0n = __shfl_sync(kFull, z_nan, __ffs(zm) - 1);
        if (LSE) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dl += __shfl_xor_sync(kFull, dl, o);
            Sx = (float)((double)Sx + dl);
        }
        __syncwarp();
    }
    // The row's top-ksel restricted to this piece is within the piece's own
    // top-ksel (final values): that is all the block has to carry.
    const uint32_t ksel = (uint32_t)rp.ksel;
    if (w.count > ksel) {
        warp_topk_keep_fit<C::kCap / 32>(ws.cand, w.count, ksel, lane);
        w.count = ksel;
    }
    uint8_t* pp = a.wpart + ((int64_t)gw * a.wl_P + j) * a.wl_stride;
    const uint32_t cap = (uint32_t)((a.wl_stride - kPartialHeaderBytes) / 8);
    ZS_CHECK(w.count <= cap && j < a.wl_P, 21, ((uint64_t)j << 32) | w.count);
    const uint32_t n = w.count < cap ? w.count : cap;
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(pp + kPartialHeaderBytes);
    for (uint32_t i = lane; i < n; i += 32) __stcg(keys + i, (unsigned long long)ws.cand[i]);
    if (lane == 0) {
        uint4 hv;
        hv.x = n;
        hv.y = (has0 ? kPartHasId0 : 0u) | ((has0 && x0n) ? kPartX0Nan : 0u) |
               (spec_ord ? kPartSpec : 0u);
        hv.z = spec_ord ? spec_ord : __float_as_uint(M);  // no log-sum-exp with a speculation
        hv.w = __float_as_uint(Sx);
        __stcg(reinterpret_cast<uint4*>(pp), hv);
    }
    __syncwarp();
}

// SPEC: the instantiation that may start long pieces from a sampled threshold
// (kept apart so the others carry none of its code).
template <class C, bool LSE, bool SPEC>
__global__ void __launch_bounds__(C::kWarps * 32, 1) zs_wselect_kernel(const Args a) {
    static_assert(!(LSE && SPEC), "no speculation with the log-sum-exp");
    extern __shared__ __align__(128) uint8_t smem_raw[];
    WSelSmem<C>& sm = *reinterpret_cast<WSelSmem<C>*>(smem_raw);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    WarpSel<C>& ws = sm.w[warp];
    grid_dep_trigger();  // the merge may be scheduled; it waits for this grid to end
    // Warp slots are dealt across the CTAs first (slot `warp` of CTA b takes share
    // warp * gridDim.x + b), so a layout with fewer warps than the grid's slots still
    // has warps on every SM of the grid instead of filling the first CTAs.
    const int32_t gw = warp * (int32_t)gridDim.x + (int32_t)blockIdx.x;
    if (gw >= a.wl_NW) return;  // the whole warp; nothing in this kernel syncs the block
    WShare sh;
    sh.b0 = wl_bound(a.wl_E, a.wl_NW, gw);
    sh.b1 = wl_bound(a.wl_E, a.wl_NW, gw + 1);
    if (sh.b0 >= sh.b1) return;
    sh.r0 = (int32_t)(sh.b0 / a.wl_Vn);
    sh.np = (int32_t)((sh.b1 - 1) / a.wl_Vn) - sh.r0 + 1;
    if (lane == 0) {
        for (int s = 0; s < kWStages; ++s) mbar_init(&ws.full[s], 1);
        mbar_fence_init();
    }
    __syncwarp();
    const uint64_t pol = l2_evict_first_policy();
    const unsigned below = lanemask_lt();

    WIssue is;
    is.j = 0;
    is.t = 0;
    is.pc = wl_piece(a, sh.b0, sh.b1, sh.r0, 0);
    int32_t issued = 0, consumed = 0;
    for (int s = 0; s < kWStages; ++s) {
        if (!wl_issue(a, ws, s, is, sh, pol, lane)) break;
        ++issued;
    }
    bool ok = true;
    for (int32_t j = 0; j < sh.np && ok; ++j) {
        const WPiece pc = wl_piece(a, sh.b0, sh.b1, sh.r0, j);
        if (!pc.active) continue;
        const RowPlan rp = plan_row(load_params(a.row_params, a.shared, pc.row), a.V_total, a.hist,
                                    a.hist_len, a.hist_ld, pc.row);
        const bool greedy_np = rp.greedy && !rp.penal;
        // A piece keeps its top (ksel + n) raw keys, n the window entries that fall in
        // its own columns: a key that is not penalised and has ksel + n raw keys above
        // it has at least ksel unpenalised keys above it after the penalty, so it
        // cannot be in the row's shortlist; penalised ids are added back at the end.
        uint32_t keff = (uint32_t)rp.keff;
        if (rp.penal) {
            const int32_t* window = a.hist + (int64_t)pc.row * a.hist_ld + (rp.hist_len - rp.win);
            const int32_t lo = a.id_offset + pc.c0, hi = a.id_offset + pc.c1;
            uint32_t n_in = 0;
            for (int base = 0; base < rp.win; base += 32) {
                const int jw = base + lane;
                const int32_t gid = jw < rp.win ? window[jw] : -1;
                n_in += __popc(__ballot_sync(kFull, gid >= lo && gid < hi));
            }
            keff = min(keff, (uint32_t)rp.ksel + n_in);
        }
        const uint32_t compact_at =
            min((uint32_t)(C::kCap - kWStepElems), keff + (keff > 128u ? keff : 128u));
        const float lc = (rp.greedy ? 1.0f : 1.0f / rp.p.temp) * 1.4426950408889634f;
        const float* row_logits = a.logits + (int64_t)pc.row * a.ld;
        const int32_t id_col0 = a.id_offset;  // global id of local column 0
        WState w;
        w.count = 0u;
        w.tau_key = 0ull;
        w.tau_f = -INFINITY;
        w.tau_id = 0;
        w.mode = kWAll;
        w.kb = 0ull;
        w.vb = -INFINITY;
        w.lm = -INFINITY;
        w.ls = 0.0f;
        // A long piece of a long shortlist starts from a sampled threshold instead of
        // ramping up from its first tile (see wspec_threshold; the merge certifies it).
        uint32_t spec_ord = 0u;
        if (SPEC && a.spec && !rp.greedy && !rp.penal && keff >= kSpecMinKeff &&
            pc.c1 - pc.c0 >= kSpecMinCols) {
            spec_ord = (pc.c1 - pc.c0 >= 2 * kSpecMinCols)
                           ? wspec_threshold<32>(row_logits, pc, keff, lane)
                           : wspec_threshold<16>(row_logits, pc, keff, lane);
            if (spec_ord != 0u) {
                w.mode = kWFast;
                w.tau_f = value_of_ord(spec_ord);
                w.tau_id = INT32_MAX;  // every element of that value passes
                w.tau_key = (uint64_t)spec_ord << 32;
            }
        }
        // head: the columns before the first 16-byte boundary (at most 3)
        {
            const int nh = pc.e0 - pc.c0;
            const bool okh = lane < nh;
            const float x = okh ? row_logits[pc.c0 + lane] : 0.0f;
            wfilter1<C, LSE>(ws, w, okh, x, id_col0 + pc.c0 + lane, greedy_np, keff, lc, below, lane);
        }
        for (int t = 0; t < pc.ntiles; ++t) {
            const int stage = consumed % kWStages;
            const uint32_t parity = (uint32_t)(consumed / kWStages) & 1u;
            const bool got = mbar_wait_bounded(&ws.full[stage], parity);
            if (!__all_sync(kFull, got)) {
                ok = false;
                break;
            }
            const int start = pc.e0 + t * kWTile;
            const int n = min(kWTile, pc.e1 - start);
            const float4* t4 = reinterpret_cast<const float4*>(ws.ring[stage]);
            if (t == 0 && !greedy_np && w.mode == kWAll && keff <= (uint32_t)(kWTile / 4) &&
                (uint32_t)(n >> 2) >= keff) {
                // start from a threshold instead of taking every element
                const uint32_t T = wfirst_threshold(t4, n >> 2, keff, lane);
                if (T != 0u) {
                    w.mode = kWFast;
                    w.tau_f = value_of_ord(T);
                    w.tau_id = INT32_MAX;  // every element of that value passes
                    w.tau_key = (uint64_t)T << 32;
                }
            }
            if (greedy_np || w.mode != kWFast) {
                wfilter_tile<C, LSE>(ws, w, t4, n >> 2, id_col0 + start, greedy_np, keff, lc, below,
                                  lane);
            } else if (!wfilter_tile_fast<C, LSE>(ws, w, ws.ring[stage], n >> 2, id_col0 + start,
                                               keff, lc, lane)) {
                // too many survivors for one batch: the per-step path (log-sum-exp done)
                wfilter_tile<C, false>(ws, w, t4, n >> 2, id_col0 + start, false, keff, lc, below,
                                    lane);
            }
            // Raise the threshold early: fewer elements reach it afterwards.
            if (!greedy_np && w.count > compact_at) wcompact(ws, w, keff, lane);
            ++consumed;
            __syncwarp();
            if (wl_issue(a, ws, stage, is, sh, pol, lane)) ++issued;
        }
        if (!ok) break;
        // tail: the columns after the last 16-byte boundary (at most 3)
        {
            const int nt = pc.c1 - pc.e1;
            const bool okt = lane < nt;
            const float x = okt ? row_logits[pc.e1 + lane] : 0.0f;
            wfilter1<C, LSE>(ws, w, okt, x, id_col0 + pc.e1 + lane, greedy_np, keff, lc, below, lane);
        }
        wend_piece<C, LSE>(a, ws, w, pc, rp, greedy_np, lc, gw, j, spec_ord, below, lane);
    }
    if (!ok) {
        if (lane == 0) set_status(a.status, kStatusTimeout);
        // leave no copy in flight into this warp's stages
        for (int32_t g = consumed; g < issued; ++g)
            mbar_wait_bounded(&ws.full[g % kWStages], (uint32_t)(g / kWStages) & 1u);
    }
}

// One step of zeninfer's generate loop after the sampler (src/main.cpp:626-632):
// a row that was already stopped keeps its Rng state (the loop drew nothing for
// it) and reports -1; a row that sampled `eos` stops without appending it; any
// other row appends its id to its on-device history.  A full history keeps its
// last `keep` entries (the penalty window, repeat_last_n) before the append, so
// the window the next step reads is unchanged.  One thread per row.
struct DecodeArgs {
    int32_t B;
    int32_t eos;
    const uint64_t* rng_prev;  // [B] states before this step's draws
    uint64_t* rng;             // [B]
    int32_t* done;             // [B] 0 running, 1 stopped
    int32_t* out_ids;          // [B]
    int32_t* hist;             // [B][hist_ld] or null
    int64_t hist_ld;
    int32_t* hist_len;         // [B] or null
    const Params* row_params;  // [B] or null (then `shared`)
    Params shared;
    int32_t* tokens;           // [B][tokens_ld] or null
    int64_t tokens_ld;
    int64_t step;
};

__global__ void zs_decode_append_kernel(const DecodeArgs a) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= a.B) return;
    int32_t* tok = a.tokens ? a.tokens + (int64_t)r * a.tokens_ld + a.step : nullptr;
    if (a.done[r]) {
        a.rng[r] = a.rng_prev[r];
        a.out_ids[r] = -1;
        if (tok) *tok = -1;
        return;
    }
    const int32_t id = a.out_ids[r];
    if (tok) *tok = id;
    if (id == a.eos) {
        a.done[r] = 1;
        return;
    }
    if (!a.hist) return;
    int32_t* h = a.hist + (int64_t)r * a.hist_ld;
    int64_t n = a.hist_len[r];
    if (n >= a.hist_ld) {
        const int32_t rln = a.row_params ? a.row_params[r].repeat_last_n : a.shared.repeat_last_n;
        const int64_t keep = min((int64_t)max(rln, 0), a.hist_ld - 1);
        for (int64_t i = 0; i < keep; ++i) h[i] = h[n - keep + i];
        n = keep;
    }
    h[n] = id;
    a.hist_len[r] = (int32_t)(n + 1);
}

// Failure-path check: one thread waits, with the same bounded wait as the select
// kernels, on an mbarrier phase that nothing completes (no arrival is ever made),
// so the wait runs out after kWaitLimitNs and the kernel reports
// ZS_ERR_DEVICE_TIMEOUT in `status` and returns.  Nothing is in flight.
__global__ void zs_wait_selftest_kernel(int* status) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
        if (!mbar_wait_bounded(&bar, 0u)) set_status(status, kStatusTimeout);
    }
}

// ---------------------------------------------------------------------------
// Large-shortlist path: rows whose top-k + penalty window exceeds the shared
// candidate buffer (top_k > 2048, or very long penalty windows).  One CTA per
// row at a time with global scratch per CTA: keys[V], tmp[V] (u64) and
// prob[V] (f64).  Exact: penalised keys -> radix-select threshold -> ordered
// compaction -> stable LSD radix sort (8-bit digits, descending) -> f64 tail.
// ---------------------------------------------------------------------------

// k-th largest of src[0..n) (n > kk >= 1), radix select over 8-bit digits.
__device__ uint64_t select_threshold_global(CandState& st, const uint64_t* src, uint32_t n,
                                            uint32_t kk, int ctid) {
    uint64_t prefix = 0, mask = 0;
    uint32_t need = kk;
    for (int shift = 56; shift >= 0; shift -= 8) {
        st.hist[ctid] = 0u;
        csync();
        for (uint32_t c0 = 0; c0 < n; c0 += 4 * kNC) {  // four loads in flight per thread
            uint64_t k[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t i = c0 + j * kNC + ctid;
                k[j] = i < n ? src[i] : 0ull;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (c0 + j * kNC + ctid < n && (k[j] & mask) == prefix)
                    atomicAdd(&st.hist[(uint32_t)(k[j] >> shift) & 255u], 1u);
        }
        csync();
        const uint32_t h = st.hist[255 - ctid];
        uint32_t tot;
        const uint32_t cum = block_incl_scan(h, st.scan, ctid, tot);
        if (cum >= need && cum - h < need) {
            st.sel_digit = 255u - (uint32_t)ctid;
            st.sel_above = cum - h;
            st.sel_cnt = h;
        }
        csync();
        const uint32_t digit = st.sel_digit, above = st.sel_above, cnt = st.sel_cnt;
        prefix |= (uint64_t)digit << shift;
        mask |= 0xffull << shift;
        need -= above;
        csync();
        if (cnt == need) break;
    }
    uint64_t mn = ~0ull;
    for (uint32_t i = ctid; i < n; i += kNC) {
        const uint64_t k = src[i];
        if ((k & mask) == prefix && k < mn) mn = k;
    }
    mn = warp_min_u64(mn);
    if ((ctid & 31) == 0) st.red64[ctid >> 5] = mn;
    csync();
    if (ctid == 0) {
        uint64_t t = st.red64[0];
        for (int w = 1; w < kConsumerWarps; ++w) t = st.red64[w] < t ? st.red64[w] : t;
        st.thr = t;
    }
    csync();
    return st.thr;
}

// Stable LSD radix sort of a[0..n) descending; b is scratch of n keys.  The keys
// arrive in ascending id order, that is already descending in their low 32 bits
// (~id), so a stable sort on the upper 32 bits (the value order) alone orders them
// completely: four passes, so the result ends in a.  Per-warp digit counters live
// in wcnt.
__device__ void radix_sort_desc_global(CandState& st, uint32_t* wcnt, uint64_t* a, uint64_t* b,
                                       uint32_t n, int ctid) {
    const int lane = ctid & 31, warp = ctid >> 5;
    const uint32_t seg = ((n + kConsumerWarps - 1) / kConsumerWarps + 31) & ~31u;
    const uint32_t w0 = min(n, (uint32_t)warp * seg), w1 = min(n, w0 + seg);
    uint64_t* src = a;
    uint64_t* dst = b;
    for (int pass = 4; pass < 8; ++pass) {
        const int shift = 8 * pass;
        for (int i = ctid; i < kConsumerWarps * 256; i += kNC) wcnt[i] = 0u;
        csync();
        // four 32-key groups per round: their loads are in flight together
        for (uint32_t c0 = w0; c0 < w1; c0 += 128) {
            uint64_t k[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t i = c0 + 32 * j + lane;
                k[j] = i < w1 ? src[i] : 0ull;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (c0 + 32 * j + lane < w1)
                    atomicAdd(&wcnt[warp * 256 + (255u - ((uint32_t)(k[j] >> shift) & 255u))], 1u);
        }
        csync();
        uint32_t tot_d = 0;
        for (int w = 0; w < kConsumerWarps; ++w) tot_d += wcnt[w * 256 + ctid];
        uint32_t all;
        uint32_t base = block_incl_scan(tot_d, st.scan, ctid, all) - tot_d;
        for (int w = 0; w < kConsumerWarps; ++w) {
            const uint32_t c = wcnt[w * 256 + ctid];
            wcnt[w * 256 + ctid] = base;
            base += c;
        }
        csync();
        for (uint32_t c0 = w0; c0 < w1; c0 += 128) {
            uint64_t kb[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t i = c0 + 32 * j + lane;
                kb[j] = i < w1 ? src[i] : 0ull;
            }
            // the groups in order, so equal digits keep their order (stable)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const bool valid = c0 + 32 * j + lane < w1;
                const uint64_t k = kb[j];
                const uint32_t d = 255u - ((uint32_t)(k >> shift) & 255u);
                // lanes holding the same digit: one ballot per digit bit
                unsigned peers = __ballot_sync(kFull, valid);
#pragma unroll
                for (int b = 0; b < 8; ++b) {
                    const unsigned bb = __ballot_sync(kFull, (d >> b) & 1u);
                    peers &= ((d >> b) & 1u) ? bb : ~bb;
                }
                const uint32_t rank = __popc(peers & lanemask_lt());
                if (valid) dst[wcnt[warp * 256 + d] + rank] = k;
                __syncwarp();
                if (valid && rank == 0) wcnt[warp * 256 + d] += __popc(peers);
                __syncwarp();
            }
        }
        csync();
        uint64_t* t = src;
        src = dst;
        dst = t;
    }
}

// Copies the keys of src[0..n) that are >= T to dst, in their order; returns how
// many.  Each warp owns a contiguous segment: it counts its keys first, the warp
// counts are scanned, then it writes them at its offset (ballot prefix per 32).
__device__ uint32_t ordered_compact_ge(CandState& st, const uint64_t* src, uint32_t n, uint64_t T,
                                       uint64_t* dst, int ctid) {
    const int lane = ctid & 31, warp = ctid >> 5;
    const uint32_t seg = ((n + kConsumerWarps - 1) / kConsumerWarps + 31) & ~31u;
    const uint32_t w0 = min(n, (uint32_t)warp * seg), w1 = min(n, w0 + seg);
    uint32_t cnt = 0;
    for (uint32_t c0 = w0; c0 < w1; c0 += 128) {
        uint64_t k[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t i = c0 + 32 * j + lane;
            k[j] = i < w1 ? src[i] : 0ull;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j)
            cnt += __popc(__ballot_sync(kFull, c0 + 32 * j + lane < w1 && k[j] >= T));
    }
    if (lane == 0) st.scan[warp] = cnt;
    csync();
    uint32_t base = 0, total = 0;
    for (int w = 0; w < kConsumerWarps; ++w) {
        const uint32_t c = st.scan[w];
        if (w < warp) base += c;
        total += c;
    }
    const unsigned below = lanemask_lt();
    for (uint32_t c0 = w0; c0 < w1; c0 += 128) {
        uint64_t k[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t i = c0 + 32 * j + lane;
            k[j] = i < w1 ? src[i] : 0ull;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const bool f = c0 + 32 * j + lane < w1 && k[j] >= T;
            const unsigned b = __ballot_sync(kFull, f);
            if (f) dst[base + __popc(b & below)] = k[j];
            base += __popc(b);
        }
    }
    csync();  // st.scan is free again, dst is written
    return total;
}

template <bool LSE>
__global__ void __launch_bounds__(kNC) zs_large_kernel(const Args a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    CandState& st = *reinterpret_cast<CandState*>(smem_raw);
    uint32_t* wcnt = reinterpret_cast<uint32_t*>(st.cand);  // 8 KB, cand is unused here
    const int ctid = threadIdx.x;
    uint8_t* ws = a.large_ws + (int64_t)blockIdx.x * a.large_ws_per_cta;
    uint64_t* keys = reinterpret_cast<uint64_t*>(ws);
    uint64_t* tmp = keys + a.V;
    double* prob = reinterpret_cast<double*>(tmp + a.V);
    // Either the large-path rows of the batch, or (spec_count set) the rows a merge
    // could not certify after speculative thresholds, whatever their path.
    const int n_work = a.spec_count ? (int)*(volatile const unsigned*)a.spec_count : a.B;
    for (int wi = blockIdx.x; wi < n_work; wi += gridDim.x) {
        const int row = a.spec_count ? a.spec_rows[wi] : wi;
        const RowPlan rp = plan_row(load_params(a.row_params, a.shared, row), a.V_total, a.hist,
                                    a.hist_len, a.hist_ld, row);
        if (!rp.large && !a.spec_count) continue;
        const float* x = a.logits + (int64_t)row * a.ld;
        for (int c0 = 0; c0 < a.V; c0 += 4 * kNC) {  // four loads in flight, then the stores
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int i = c0 + j * kNC + ctid;
                v[j] = i < a.V ? x[i] : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int i = c0 + j * kNC + ctid;
                if (i < a.V) keys[i] = make_key(v[j], a.id_offset + i);
            }
        }
        __threadfence_block();
        csync();
        if (rp.penal && ctid == 0) {
            // Sequential, in window order, exactly as src/sample.cpp:43-49.
            const int32_t* w = a.hist + (int64_t)row * a.hist_ld + (rp.hist_len - rp.win);
            const float pen = rp.p.repeat_penalty;
            for (int j = 0; j < rp.win; ++j) {
                const int32_t gid = w[j];
                if (gid < 0 || gid >= a.V_total) continue;
                const int32_t li = gid - a.id_offset;
                if (li < 0 || li >= a.V) continue;
                float v = key_value(keys[li]);
                v = (v > 0.0f) ? v / pen : v * pen;
                keys[li] = make_key(v, gid);
            }
        }
        __threadfence_block();
        csync();
        const bool x0n = (a.id_offset == 0 && a.V > 0) ? ((uint32_t)(keys[0] >> 32) == 0u) : false;
        const float lc = (rp.greedy ? 1.0f : 1.0f / rp.p.temp) * 1.4426950408889634f;
        float M = -INFINITY, Sx = 0.0f;
        if (LSE) {
            float lm = -INFINITY, ls = 0.0f;
            for (int i = ctid; i < a.V; i += kNC) lse_add1(lm, ls, key_value(keys[i]), lc);
            block_lse(st, lm, ls, lc, ctid);
            M = st.lse_m;
            Sx = st.lse_s;
        }
        const uint32_t n = (uint32_t)a.V;
        const uint32_t kk = (uint32_t)rp.ksel < n ? (uint32_t)rp.ksel : n;
        uint64_t T = 0ull;
        if (kk < n) T = select_threshold_global(st, keys, n, kk, ctid);
        uint32_t base = 0;
        if (kk == n) {  // every key is kept: copy, the sort orders them
            for (uint32_t c0 = 0; c0 < n; c0 += 4 * kNC) {
                uint64_t k4[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t i = c0 + j * kNC + ctid;
                    k4[j] = i < n ? keys[i] : 0ull;
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t i = c0 + j * kNC + ctid;
                    if (i < n) tmp[i] = k4[j];
                }
            }
            base = n;
        }
        if (kk < n) base = ordered_compact_ge(st, keys, n, T, tmp, ctid);
        ZS_CHECK(base == kk, 22, base);  // unique keys: exactly kk are >= the kk-th
        __threadfence_block();
        csync();
        radix_sort_desc_global(st, wcnt, tmp, keys, kk, ctid);
        __threadfence_block();
        csync();
        finalize_row(st, tmp, prob, kk, rp, x0n, LSE, M, Sx, row, a.rng, a.out_ids, a.info,
                     a.cand_ids, a.cand_probs, a.cand_ld, ctid);
        __threadfence_block();
        csync();
    }
}

// ---------------------------------------------------------------------------
// zs_small_kernel: a small batch (decode-sized, a few rows) in ONE launch.
// One thread block cluster of kSmallCl CTAs per row.  CTA r copies the r-th slice
// of the row's columns into its shared memory with 1-D bulk copies (the at most
// three columns after the last 16-byte boundary by plain loads), so every later
// step is a short loop over shared memory: a one-row call is latency-bound, and
// much of that latency was fetching the long unrolled code of a register-resident
// slice.  A repeat penalty (window up to kSmallWinMax) is written over the
// slice's values in place (src/sample.cpp:40-50: one thread per distinct window
// id, compounding once per occurrence).  Each thread proposes its largest key (or
// its four largest, for shortlists above 64), and warp 0 finds the ksel-th
// largest proposal with a register radix walk: ksel different keys of the slice
// reach it.  After a cluster barrier every CTA reads the 16 thresholds through
// distributed shared memory and takes the largest, T: its CTA has ksel keys at
// or above T, so the row's shortlist is at or above T.  Each CTA publishes its
// keys at or above T (a float4 whose largest component is below T's value is
// skipped without making keys); after a second barrier CTA 0 reads every CTA's
// keys, selects and sorts the exact top-ksel, and after a third (which keeps the
// other CTAs' shared memory alive until CTA 0 has read it) runs the f64 tail of
// sample_token (finalize_row).  Greedy rows publish each slice's largest key and
// need no threshold.  The cluster barriers are hardware barriers every CTA of the
// cluster reaches alike; the bulk copies' wait is bounded (it reports
// ZS_ERR_DEVICE_TIMEOUT and the CTA goes on with an empty slice, so the cluster
// still meets at every barrier).  Serves shortlists up to kGroupMaxK, no log Z,
// 16-byte aligned rows of kSmallMinCols to kSmallMaxCols columns (the host
// checks).
// ---------------------------------------------------------------------------
constexpr int kSmallCl = 16;  // CTAs per row (a non-portable cluster size)
constexpr int kSmallNJ = 12;  // float4s per thread
constexpr int kSmallMaxCols = kSmallCl * kNC * 4 * kSmallNJ;  // 196,608
constexpr int kSmallMinCols = kSmallCl * kNC * 4;             // every thread holds a float4
constexpr int kSmallWinMax = kNC;                             // one thread per window entry
constexpr int kSmallChunk = 4096;                             // bytes per bulk copy

struct SmallSmem {
    CandState st;             // this CTA's candidates; on CTA 0 also the row's merge
    uint64_t pub[kCandCap];   // this CTA's published keys
    float4 vals[kSmallNJ * kNC];  // the slice (penalised in place)
    float tail[4];            // its columns after the last 16-byte boundary
    uint64_t bar;             // the bulk copies' completion
    uint64_t pub_tau;         // at least ksel of this slice's keys are >= pub_tau
    uint32_t pub_n;
    int32_t x0_nan;
    int32_t lost;              // the bulk copies' wait ran out: the slice is not there
    uint32_t g_off[kSmallCl];  // CTA 0: first key of each CTA in the concatenated list
    uint32_t g_all;            // CTA 0: keys published in all
    int32_t win[kSmallWinMax];  // the penalty window
};

__global__ void __launch_bounds__(kNC, 1) zs_small_kernel(const Args a) {
    namespace cg = cooperative_groups;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    SmallSmem& sm = *reinterpret_cast<SmallSmem*>(smem_raw);
    CandState& st = sm.st;
    cg::cluster_group cluster = cg::this_cluster();
    const int crank = (int)cluster.block_rank();
    const int row = (int)blockIdx.x / kSmallCl;
    const int ctid = (int)threadIdx.x, lane = ctid & 31;
    const RowPlan rp = plan_row(load_params(a.row_params, a.shared, row), a.V_total, a.hist,
                                a.hist_len, a.hist_ld, row);
    const uint32_t ksel = (uint32_t)rp.ksel;
    const int per = ((a.V + kSmallCl - 1) / kSmallCl + 3) & ~3;
    const int c0 = min(a.V, crank * per), c1 = min(a.V, c0 + per);
    const float* x = a.logits + (int64_t)row * a.ld;
    int n4 = (c1 - c0) >> 2;
    const int tail0 = c0 + 4 * n4;  // at most 3 columns after the last float4
    const int nt = c1 - tail0;
    const uint32_t bytes = (uint32_t)n4 * 16u;
    if (ctid == 0) {
        mbar_init(&sm.bar, 1);
        mbar_fence_init();
        mbar_arrive_expect_tx(&sm.bar, bytes);
        const uint64_t pol = l2_evict_first_policy();
        for (uint32_t off = 0; off < bytes; off += kSmallChunk)
            bulk_load(reinterpret_cast<uint8_t*>(sm.vals) + off,
                      reinterpret_cast<const uint8_t*>(x + c0) + off,
                      min((uint32_t)kSmallChunk, bytes - off), &sm.bar, pol);
    }
    if (ctid < nt) sm.tail[ctid] = x[tail0 + ctid];
    if (rp.penal && ctid < rp.win)
        sm.win[ctid] = a.hist[(int64_t)row * a.hist_ld + (rp.hist_len - rp.win) + ctid];
    if (ctid == 0) {
        sm.pub_n = 0u;
        sm.lost = mbar_wait_bounded(&sm.bar, 0u) ? 0 : 1;
        if (sm.lost) set_status(a.status, kStatusTimeout);
    }
    csync();
    const bool lost = sm.lost != 0;
    if (lost) n4 = 0;  // go on with an empty slice, so every barrier is still met
    float* sv = reinterpret_cast<float*>(sm.vals);
    // Repetition penalty (src/sample.cpp:40-50) on this slice's values, in place:
    // the thread of a window id's first occurrence compounds the penalty once per
    // occurrence on the raw logit.  rp.penal is the same on every thread of the row.
    if (rp.penal && !lost) {
        if (ctid < rp.win) {
            const int32_t gid = sm.win[ctid];
            const int32_t lo = a.id_offset + c0, hi = a.id_offset + c1;
            if (gid >= 0 && gid < a.V_total && gid >= lo && gid < hi) {
                bool first = true;
                for (int q = 0; q < ctid; ++q)
                    if (sm.win[q] == gid) {
                        first = false;
                        break;
                    }
                if (first) {
                    int mult = 1;
                    for (int q = ctid + 1; q < rp.win; ++q) mult += sm.win[q] == gid ? 1 : 0;
                    const float pen = rp.p.repeat_penalty;
                    float val = x[gid - a.id_offset];
                    for (int c = 0; c < mult; ++c) val = (val > 0.0f) ? val / pen : val * pen;
                    const int l = gid - lo;  // column within the slice
                    if (l < 4 * n4) sv[l] = val;
                    else sm.tail[l - 4 * n4] = val;
                }
            }
        }
        csync();
    }
    // the NaN test of logits[0] sees its penalised value (column 0 of CTA 0)
    if (crank == 0 && ctid == 0) sm.x0_nan = (a.V > 0 && !lost && sv[0] != sv[0]) ? 1 : 0;
    const bool has_t = !lost && ctid < nt;
    const float xt = has_t ? sm.tail[ctid] : 0.0f;
    const int32_t tid_t = a.id_offset + tail0 + ctid;  // the tail column's id
    // This thread's largest key (short shortlists) or its four largest keys
    // (descending; longer ones): its proposals.
    uint64_t t0 = 0ull, t1 = 0ull, t2 = 0ull, t3 = 0ull;
    const bool four = ksel > 64u;  // the same on every thread of the row
    if (!four) {
        // the largest value first (fmaxf skips NaN), then the smallest id holding it
        float M = has_t ? xt : __int_as_float(0x7fc00000);
        for (int i = ctid; i < n4; i += kNC) {
            const float4 w = sm.vals[i];
            M = fmaxf(M, fmaxf(fmaxf(w.x, w.y), fmaxf(w.z, w.w)));
        }
        const bool all_nan = M != M;
        for (int i = ctid; i < n4; i += kNC) {
            const float4 w = sm.vals[i];
            if (all_nan || w.x == M || w.y == M || w.z == M || w.w == M) {
                const int32_t id = a.id_offset + c0 + 4 * i;
                uint64_t k = make_key(w.x, id);
                k = max(k, make_key(w.y, id + 1));
                k = max(k, make_key(w.z, id + 2));
                k = max(k, make_key(w.w, id + 3));
                t0 = k > t0 ? k : t0;
            }
        }
        if (has_t) {
            const uint64_t k = make_key(xt, tid_t);
            t0 = k > t0 ? k : t0;
        }
    } else {
        auto propose = [&](uint64_t k) {
            if (k > t3) {
                t3 = k;
                if (t3 > t2) { const uint64_t u = t2; t2 = t3; t3 = u; }
                if (t2 > t1) { const uint64_t u = t1; t1 = t2; t2 = u; }
                if (t1 > t0) { const uint64_t u = t0; t0 = t1; t1 = u; }
            }
        };
        for (int i = ctid; i < n4; i += kNC) {
            const float4 w = sm.vals[i];
            const int32_t id = a.id_offset + c0 + 4 * i;
            propose(make_key(w.x, id));
            propose(make_key(w.y, id + 1));
            propose(make_key(w.z, id + 2));
            propose(make_key(w.w, id + 3));
        }
        if (has_t) propose(make_key(xt, tid_t));
    }
    uint64_t T = 0ull;  // sampled rows: every published key is at or above it
    if (ksel == 1u) {
        // greedy: the slice's largest key is all it publishes
        const uint64_t wm = warp_max_u64(t0);
        if (lane == 0) st.red64[ctid >> 5] = wm;
        csync();
        if (ctid == 0) {
            uint64_t m = 0ull;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) m = st.red64[w] > m ? st.red64[w] : m;
            sm.pub[0] = m;
            sm.pub_n = m != 0ull ? 1u : 0u;
        }
    } else {
        // This CTA's threshold: the ksel-th largest proposal (each is a different key
        // of the slice, and every thread holds at least four elements, so ksel keys
        // of the slice reach it), by warp 0's register radix walk.  An empty slice
        // (a lost copy) proposes nothing and publishes threshold 0.
        if (!four) {
            st.cand[ctid] = t0;
        } else {
            st.cand[4 * ctid] = t0;
            st.cand[4 * ctid + 1] = t1;
            st.cand[4 * ctid + 2] = t2;
            st.cand[4 * ctid + 3] = t3;
        }
        csync();
        if (ctid < 32) {
            uint64_t t = 0ull;
            if (!lost)
                t = four ? warp_topk_keep<4 * kNC / 32>(st.cand, 4 * kNC, ksel, lane)
                         : warp_topk_keep<kNC / 32>(st.cand, kNC, ksel, lane);
            if (lane == 0) sm.pub_tau = t;
        }
        cluster.sync();  // every CTA's threshold is published
        // The largest of them: its CTA has ksel keys at or above it, so the row's
        // shortlist is at or above it, and each CTA publishes only its keys there.
        if (ctid < 32) {
            const uint64_t t = ctid < kSmallCl ? cluster.map_shared_rank(&sm, ctid)->pub_tau : 0ull;
            const uint64_t tm = warp_max_u64(t);
            if (ctid == 0) st.thr = tm;
        }
        csync();
        T = st.thr;
        // A float4 whose largest component is below T's value has no key at or
        // above T (fmaxf skips NaN, whose keys are below any T of a non-NaN value);
        // T of a NaN value compares whole keys.
        const uint32_t To = (uint32_t)(T >> 32);
        const float Tv = value_of_ord(To);
        auto reaches = [&](const float4& w) {
            return To == 0u || fmaxf(fmaxf(w.x, w.y), fmaxf(w.z, w.w)) >= Tv;
        };
        uint32_t c = 0u;
        for (int i = ctid; i < n4; i += kNC) {
            const float4 w = sm.vals[i];
            if (reaches(w)) {
                const int32_t id = a.id_offset + c0 + 4 * i;
                c += (uint32_t)(make_key(w.x, id) >= T) + (uint32_t)(make_key(w.y, id + 1) >= T) +
                     (uint32_t)(make_key(w.z, id + 2) >= T) + (uint32_t)(make_key(w.w, id + 3) >= T);
            }
        }
        if (has_t && make_key(xt, tid_t) >= T) ++c;
        uint32_t total;
        block_incl_scan(c, st.scan, ctid, total);
        if (total + kCandMargin <= (uint32_t)kCandCap) {  // the same on every thread
            // published in any order (CTA 0 sorts): a slot per key from a counter
            if (c) {
                for (int i = ctid; i < n4; i += kNC) {
                    const float4 w = sm.vals[i];
                    if (reaches(w)) {
                        const int32_t id = a.id_offset + c0 + 4 * i;
                        const float xs[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                        for (int r = 0; r < 4; ++r) {
                            const uint64_t k = make_key(xs[r], id + r);
                            if (k >= T) sm.pub[atomicAdd(&sm.pub_n, 1u)] = k;
                        }
                    }
                }
                if (has_t && make_key(xt, tid_t) >= T) sm.pub[atomicAdd(&sm.pub_n, 1u)] = make_key(xt, tid_t);
            }
        } else {
            // More keys reach T than the buffer holds (heavy ties at T): append in
            // rounds, compacting to the top ksel when full.
            if (ctid == 0) st.count = 0u;
            csync();
            uint64_t tau = T - 1ull;  // keys > tau are the keys >= T
            bool full = false;
            for (int j = 0; j <= kSmallNJ; ++j) {  // rounds of one float4 a thread, then the tail
                const int i = j * kNC + ctid;
                uint64_t ks[4] = {0ull, 0ull, 0ull, 0ull};
                if (j < kSmallNJ && i < n4) {
                    const float4 w = sm.vals[i];
                    const int32_t id = a.id_offset + c0 + 4 * i;
                    ks[0] = make_key(w.x, id);
                    ks[1] = make_key(w.y, id + 1);
                    ks[2] = make_key(w.z, id + 2);
                    ks[3] = make_key(w.w, id + 3);
                } else if (j == kSmallNJ && has_t) {
                    ks[0] = make_key(xt, tid_t);
                }
                for (int r = 0; r < 4; ++r) {
                    if (full) tau = compact_select(st, st.count, ksel, ctid);
                    warp_append(st, ks[r] > tau, ks[r], lane);
                    full = csync_or(st.count + kNC + kCandMargin > (uint32_t)kCandCap);
                }
            }
            uint32_t n = st.count;
            if (n > ksel) {
                compact_select(st, n, ksel, ctid);
                n = st.count;
            }
            for (uint32_t i = ctid; i < n; i += kNC) sm.pub[i] = st.cand[i];
            if (ctid == 0) sm.pub_n = n;
        }
    }
    cluster.sync();  // every CTA's keys are published
    uint32_t kk = 0u;
    if (crank == 0) {
        // Counts and offsets of all CTAs first (one remote read each), then every
        // published key in parallel, four loads in flight a thread, in rounds of
        // 4 x kNC keys; before a round that might not fit, the candidates are cut to
        // the top ksel.  The loop bound is the same on every thread (warp_append
        // needs all lanes).
        if (ctid < 32) {
            const uint32_t nr = ctid < kSmallCl ? cluster.map_shared_rank(&sm, ctid)->pub_n : 0u;
            uint32_t inc = nr;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t u = __shfl_up_sync(kFull, inc, o);
                if (lane >= o) inc += u;
            }
            if (ctid < kSmallCl) sm.g_off[ctid] = inc - nr;  // first key of CTA ctid
            if (ctid == 31) sm.g_all = inc;                  // all published keys
            if (ctid == 0) st.count = 0u;
        }
        csync();
        uint64_t tau = T ? T - 1ull : 0ull;  // every published key passes
        const uint32_t all = sm.g_all;
        bool full = false;
        for (uint32_t b = 0; b < all; b += 4 * kNC) {
            if (full) tau = compact_select(st, st.count, ksel, ctid);
            const uint32_t i0 = b + (uint32_t)ctid;
            uint64_t kv[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const uint32_t i = i0 + j * kNC;
                kv[j] = 0ull;
                if (i < all) {
                    int lo = 0, hi = kSmallCl - 1;  // the last CTA starting at or before i
                    while (lo < hi) {
                        const int mid = (lo + hi + 1) >> 1;
                        if (sm.g_off[mid] <= i) lo = mid;
                        else hi = mid - 1;
                    }
                    kv[j] = cluster.map_shared_rank(&sm, lo)->pub[i - sm.g_off[lo]];
                }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) warp_append(st, kv[j] > tau, kv[j], lane);
            full = csync_or(st.count + 4 * kNC + kCandMargin > (uint32_t)kCandCap);
        }
        uint32_t m = st.count;
        if (m > (uint32_t)kNC && m > ksel) {  // up to kNC keys are sorted whole
            compact_select(st, m, ksel, ctid);
            m = st.count;
        }
        sort_desc(st, m, ctid);
        kk = m < ksel ? m : ksel;
    }
    cluster.sync();  // CTA 0 has read every CTA's keys
    if (crank == 0)
        finalize_row(st, st.cand, reinterpret_cast<double*>(st.cand + kProbOffset), kk, rp,
                     sm.x0_nan != 0, false, -INFINITY, 0.0f, row, a.rng, a.out_ids, a.info,
                     a.cand_ids, a.cand_probs, a.cand_ld, ctid);
}

}  // namespace zs

