/*
 * zs_sampler.h -- C ABI of the B200 token sampler (libzs_sampler.so).
 *
 * This is the boundary a host program binds.  It replaces the two entry points
 * of zeninfer's sampler, namespace zen in src/sample.h:
 *
 *   int32_t argmax_token(const float* logits, int n);              src/sample.h:28
 *   int32_t sample_token(const float* logits, int n,
 *                        const SamplingParams& p,
 *                        const std::vector<int32_t>& history,
 *                        Rng& rng);                                src/sample.h:36-37
 *
 * with batched, stream-ordered device entry points.  The C++ API of sample.h
 * itself (host pointers, one row per call) is served on top of this ABI by
 * include/zen/sample.h + libzen_sample.so.
 *
 * Semantics per row are those of sample_token (src/sample.cpp:32-102):
 * repetition penalty over the last repeat_last_n history ids (compounding on
 * duplicates) -> greedy argmax when temp <= 0 -> top-k shortlist (k = top_k, or
 * 256 when top_k == 0) -> f64 softmax over the shortlist -> nucleus prefix
 * (top_p < 1) -> inverse-CDF draw from the row's xorshift64* state, one draw per
 * non-greedy row.  The shortlist order is value descending, then token id
 * ascending (the reference leaves equal values in libstdc++'s introselect order).
 *
 * Conventions: every pointer argument documented "device" is CUDA device memory
 * of the handle's device; "host" is ordinary host memory.  `stream` is a
 * cudaStream_t (NULL = legacy default stream).  All entry points return a
 * zs_status; nothing throws across the ABI.  Calls are asynchronous with
 * respect to the host unless documented otherwise; errors detected on the
 * device (a wait that ran out) are reported by zs_check_device_status().
 */
#ifndef ZS_SAMPLER_H_
#define ZS_SAMPLER_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ZS_ABI_VERSION 4

typedef enum zs_status {
    ZS_OK = 0,
    ZS_ERR_INVALID_ARGUMENT = 1, /* bad size, null pointer, misaligned logits */
    ZS_ERR_CUDA = 2,             /* a CUDA runtime call failed; see zs_last_error() */
    ZS_ERR_NO_DEVICE = 3,        /* no CUDA device, or not an sm_100 device */
    ZS_ERR_DEVICE_TIMEOUT = 4,   /* a kernel's bounded wait ran out; the results are invalid */
    ZS_ERR_NCCL = 5,             /* NCCL missing or a NCCL call failed */
    ZS_ERR_OUT_OF_MEMORY = 6
} zs_status;

/* Same field order, types and meaning as zen::SamplingParams (src/sample.h:9-15). */
typedef struct zs_params {
    float temp;            /* <= 0 means greedy argmax */
    int32_t top_k;         /* 0 = disabled: shortlist of 256 */
    float top_p;           /* 1.0 = disabled (nucleus over the shortlist) */
    float repeat_penalty;  /* 1.0 = disabled */
    int32_t repeat_last_n; /* penalty window over the tail of the history */
} zs_params;

/* Optional per-row diagnostics (48 bytes). */
typedef struct zs_row_info {
    float max_logit; /* max_l of sample_token: f32 max over the penalised row (NaN if
                        logits[0] is NaN); for greedy rows the chosen logit */
    int32_t k;       /* shortlist size (0 for greedy rows) */
    int32_t m;       /* nucleus size */
    int32_t pos;     /* shortlist position of the drawn token (-1 for greedy rows) */
    double r;        /* the uniform draw */
    double sum;      /* sum of exp((x_i - max_l) * inv_temp) over the shortlist */
    double boundary; /* |r - nearest CDF boundary| */
    double log_z;    /* log sum_{all V} exp((x - max_l) * inv_temp) when requested
                        (inv_temp = 1 for greedy rows), NaN otherwise */
} zs_row_info;

/* Optional outputs of zs_sample; any member may be NULL / 0. */
typedef struct zs_extras {
    zs_row_info* row_info; /* device [batch] */
    int32_t* cand_ids;     /* device [batch][cand_ld]: sorted shortlist ids */
    double* cand_probs;    /* device [batch][cand_ld]: shortlist softmax before the nucleus rescale */
    int32_t cand_ld;       /* row stride of cand_ids / cand_probs; entries >= k are untouched */
    int32_t want_log_z;    /* nonzero: fill row_info->log_z (costs one exp per logit) */
} zs_extras;

typedef struct zs_context* zs_handle;

/* One handle per device; it owns the scratch and the kernel configuration.
 * The handle is not thread-safe: use one per host thread, or serialise.  Calls on
 * one handle share its scratch, so issue them on one stream (or order the streams):
 * two calls of one handle running on the GPU at the same time race. */
zs_status zs_create(int device, zs_handle* out);
zs_status zs_destroy(zs_handle h);

/* Message of the last failing call on this host thread ("" if none). */
const char* zs_last_error(void);
const char* zs_status_string(zs_status s);
int zs_abi_version(void);

/* zen::Rng(seed): the xorshift64* state a seed maps to (0 -> 0x9E3779B97F4A7C15). */
uint64_t zs_rng_seed(uint64_t seed);

/*
 * Batched sample_token (src/sample.cpp:32-102) for `batch` rows of n_vocab f32
 * logits, row r at logits + r * ld (device, 4-byte aligned, never modified).
 *
 *   params          host; 1 struct shared by every row, or `batch` structs when
 *                   params_per_row != 0
 *   history         device [batch][history_ld] token ids; row r's history is its
 *                   first history_len[r] entries (history_len: device [batch]).
 *                   Both may be NULL when no row has repeat_penalty != 1.
 *   rng_state       device [batch] xorshift64* states, advanced in place by one
 *                   draw for every non-greedy row (zen::Rng& semantics)
 *   out_ids         device [batch]
 *   extras          host pointer to optional outputs, or NULL
 *
 * n_vocab <= 0 writes 0 to every out_ids entry and draws nothing (sample.cpp:34).
 */
zs_status zs_sample(zs_handle h, const float* logits, int64_t ld, int32_t batch, int32_t n_vocab,
                    const zs_params* params, int32_t params_per_row, const int32_t* history,
                    int64_t history_ld, const int32_t* history_len, uint64_t* rng_state,
                    int32_t* out_ids, const zs_extras* extras, void* stream);

/*
 * One step of the generate loop (src/main.cpp:626-632) with the history, the Rng
 * states and the stop flags on the device, so a decode loop needs no host copy:
 *   next = sample_token(logits, V, params, history, rng); if (next == eos) stop;
 *   history.push_back(next)
 * for every row whose done[r] is 0 on entry.  Rows with done[r] != 0 draw nothing
 * (their rng_state is left as it was) and get out_ids[r] = -1.  A row that samples
 * eos_id sets done[r] = 1 and does not append it (the reference breaks before the
 * push).  Other rows append to history (device [batch][history_ld], lengths in
 * history_len); a full row keeps its last repeat_last_n entries first, so
 * history_ld must exceed repeat_last_n for every row with repeat_penalty != 1.
 * history and history_len may both be NULL (no penalty, nothing appended).
 * tokens (device [batch][tokens_ld], may be NULL) receives out_ids at column `step`.
 * No counterpart function in the reference: cmd_generate inlines this loop.
 */
zs_status zs_decode_step(zs_handle h, const float* logits, int64_t ld, int32_t batch,
                         int32_t n_vocab, const zs_params* params, int32_t params_per_row,
                         int32_t* history, int64_t history_ld, int32_t* history_len,
                         uint64_t* rng_state, int32_t* done, int32_t eos_id, int32_t* out_ids,
                         int32_t* tokens, int64_t tokens_ld, int64_t step, void* stream);

/*
 * The lm_head of Model::eval (src/model.cpp:401-403) fused with sample_token: for
 * each of `batch` rows,
 *   xn     = rmsnorm(hidden_r, norm_w, eps)      (src/model.cpp:31-38)
 *   logits = matvec(xn, weight)                  (src/model.cpp:40-42, 403)
 *   out_ids[r] = sample_token(logits, n_vocab, params, history_r, rng_r)
 * on the tensor cores: xn is rounded to bfloat16 and `weight` is bfloat16
 * [n_vocab][n_embd] (row-major, 16-byte aligned; the reference's output.weight
 * after dequantisation, stored as bfloat16), products accumulate in f32.  The
 * logits differ from the reference's f32 matvec by the bfloat16 rounding of xn and
 * the accumulation order; the sampling on those logits is zs_sample's exactly.
 *   hidden     device f32 [batch][hidden_ld], the last position's hidden state
 *   norm_w     device f32 [n_embd], output_norm.weight
 *   n_embd     a multiple of 8, from 64 to 12288
 *   out_logits optional device f32 [batch][logits_ld] (logits_ld >= n_vocab, a
 *              multiple of 4): the logits the sampling used
 * Rows whose shortlist (top_k, or 256 when top_k is 0; 1 for greedy) is at most 88
 * and that have no repeat penalty can be selected inside the GEMM's epilogue and never
 * leave the chip as logits; zs_set_lmhead_route says when they are (by default above
 * 1024 rows).  Any other batch is written as logits (to out_logits or handle scratch)
 * and sampled by zs_sample.  Other arguments as zs_sample.
 * Replaces, for one step of cmd_generate, model.eval's last two lines and the
 * sample_token call (src/main.cpp:628).
 */
zs_status zs_lmhead_sample(zs_handle h, const float* hidden, int64_t hidden_ld,
                           const float* norm_w, float eps, const void* weight, int32_t batch,
                           int32_t n_embd, int32_t n_vocab, const zs_params* params,
                           int32_t params_per_row, const int32_t* history, int64_t history_ld,
                           const int32_t* history_len, uint64_t* rng_state, int32_t* out_ids,
                           float* out_logits, int64_t logits_ld, void* stream);

/* The lm_head alone: the last two lines of Model::eval (src/model.cpp:401-403),
 *   out_logits[r] = matvec(rmsnorm(hidden_r, norm_w, eps), weight)
 * for `batch` rows on the tensor cores, with the same arithmetic (bf16 xn and
 * weight, f32 accumulation) and the same argument rules as zs_lmhead_sample;
 * out_logits (device f32 [batch][logits_ld]) is required.  Sample the result with
 * zs_sample when the shortlist cannot be taken in the GEMM's epilogue. */
zs_status zs_lmhead_logits(zs_handle h, const float* hidden, int64_t hidden_ld,
                           const float* norm_w, float eps, const void* weight, int32_t batch,
                           int32_t n_embd, int32_t n_vocab, float* out_logits, int64_t logits_ld,
                           void* stream);

/* Batched argmax_token (src/sample.cpp:24-30): first index of the maximum; a NaN at
 * index 0 yields 0.  No penalty, no draw. */
zs_status zs_argmax(zs_handle h, const float* logits, int64_t ld, int32_t batch, int32_t n_vocab,
                    int32_t* out_ids, void* stream);

/* Waits for `stream` and reports ZS_ERR_DEVICE_TIMEOUT if any kernel of this handle
 * gave up on a bounded wait since the last check (the flag is then cleared). */
zs_status zs_check_device_status(zs_handle h, void* stream);

/* Exercises the failure path of the device waits: launches one thread that waits,
 * with the select kernels' bounded wait, on a barrier nothing ever completes; after
 * the limit (1 s) it records ZS_ERR_DEVICE_TIMEOUT for this handle and returns, so
 * the next zs_check_device_status reports it.  No GPU fault, nothing left running.
 * No counterpart in the reference (its sampler has no device code). */
zs_status zs_selftest_wait_timeout(zs_handle h, void* stream);

/* Per-kernel device time, for measurement.  While timing is on, every kernel this
 * handle launches is bracketed by CUDA events on its stream.  zs_get_timing waits
 * for those events, returns the sums since the previous zs_get_timing (or since
 * timing was switched on) and starts over.  `launches` counts every kernel launch
 * of the handle in that span, timed or not.  No counterpart in the reference. */
typedef struct zs_timing {
    double select_ms, merge_ms, large_ms;              /* summed event time per kernel */
    int64_t select_launches, merge_launches, large_launches;
    int64_t launches;
    double lmhead_ms;                                  /* zs_lmhead_kernel */
    int64_t lmhead_launches;
    double lmnorm_ms;                                  /* its rmsnorm prologue */
    int64_t lmnorm_launches;
} zs_timing;
zs_status zs_set_timing(zs_handle h, int32_t enable);
zs_status zs_get_timing(zs_handle h, zs_timing* out);

/* How zs_lmhead_sample takes the shortlist (and zs_lmhead_logits computes its
 * logits), for this handle.  No counterpart in the reference (its lm_head and sampler
 * are separate CPU calls).
 *   ZS_LMHEAD_ROUTE_AUTO      (default) exact up to 8 rows (while it fits: below),
 *                             two passes below 1024 rows, fused from 1024
 *   ZS_LMHEAD_ROUTE_FUSED     in the GEMM's epilogue whenever the rows allow it (no
 *                             logits buffer: for callers that cannot spare one)
 *   ZS_LMHEAD_ROUTE_TWO_PASS  always write tensor-core logits, then zs_sample
 *   ZS_LMHEAD_ROUTE_EXACT     f32 logits bit-exact with the reference's default lm_head
 *                             (src/model.cpp:401-403 with src/kernels.cpp:52-78: f32
 *                             xn, its AVX2 summation order) on the same weights (the
 *                             weight argument is bf16, so a reference whose f32
 *                             weights are bf16 values), then zs_sample; up to 8
 *                             rows, hidden sizes up to 2048 and rows x hidden size
 *                             up to 8192, else ZS_ERR_INVALID_ARGUMENT
 * The tensor-core routes (fused, two passes) round xn to bf16 and give the same ids
 * and Rng states as each other.  The routes that write logits write them to out_logits
 * when given, else to handle scratch of batch x n_vocab floats. */
#define ZS_LMHEAD_ROUTE_AUTO 0
#define ZS_LMHEAD_ROUTE_FUSED 1
#define ZS_LMHEAD_ROUTE_TWO_PASS 2
#define ZS_LMHEAD_ROUTE_EXACT 3
zs_status zs_set_lmhead_route(zs_handle h, int32_t route);

/* The tiles of the lm_head GEMM (zs_lmhead_sample, zs_lmhead_logits), for this
 * handle.  No counterpart in the reference.
 *   ZS_LMHEAD_TILES_AUTO    (default) CTA pairs from 512 rows up, one CTA below
 *   ZS_LMHEAD_TILES_SINGLE  one CTA per 128-row x 128-column tile
 *   ZS_LMHEAD_TILES_PAIR    two CTAs (a cluster of two SMs) per 256 x 256 tile
 *                           whenever the device can hold them
 * A pair's MMAs read half the operand bytes per product of one CTA's.  Logits, ids
 * and Rng states are the same either way. */
#define ZS_LMHEAD_TILES_AUTO 0
#define ZS_LMHEAD_TILES_SINGLE 1
#define ZS_LMHEAD_TILES_PAIR 2
zs_status zs_set_lmhead_tiles(zs_handle h, int32_t mode);

/* Speculative opening thresholds of zs_sample (and zs_decode_step), per handle.  No
 * counterpart in the reference.  A long row slice of a long shortlist (top_k or the
 * default 256 at least 128, no repeat penalty, no log Z) can start its streaming
 * filter from a threshold sampled from about 3% of its columns instead of ramping up
 * from its first tile; the merge certifies every such row (its shortlist's last key
 * is at or above every threshold its slices used, so nothing dropped could rank) and
 * redoes the rest exactly with the large-shortlist kernel before drawing.  Results
 * are identical in every mode; only the time differs.
 *   ZS_SPECULATION_ON        (default)
 *   ZS_SPECULATION_OFF       every slice ramps up from its first tile
 *   ZS_SPECULATION_REDO_ALL  speculate, then redo every speculated row (a test of
 *                            the redo path; slow) */
#define ZS_SPECULATION_OFF 0
#define ZS_SPECULATION_ON 1
#define ZS_SPECULATION_REDO_ALL 2
zs_status zs_set_speculation(zs_handle h, int32_t mode);

/* Batches of at most max_rows rows (default 8; 0 turns it off) run as ONE launch:
 * a cluster of 16 CTAs per row holds the row in registers, and the row's shortlist
 * is merged through distributed shared memory, for penalty windows (repeat_last_n)
 * up to 256, shortlists up to 256, no log Z, 16-byte aligned rows (logits and ld * 4) of 16,384
 * to 196,608 columns, where the GPU can keep that many 16-CTA clusters resident.
 * Other batches take the select and merge launches.  Results are identical either
 * way.  No counterpart in the reference. */
zs_status zs_set_small_batch(zs_handle h, int32_t max_rows);

/* The display numbers of zeninfer's `logits` command (src/main.cpp:473-503) for each
 * of `batch` rows of n_vocab f32 logits (device, row r at logits + r * ld):
 *   out_min, out_max  device double [batch]: the row's smallest and largest value,
 *                     from starts of 1e30 and -1e30 as there (NaN ignored)
 *   out_z             device double [batch]: sum over the row of exp(x - max), f64
 *   top_ids           device int32 [batch][topn]: the k = clamp(topn, 1, n_vocab)
 *                     largest ids, value descending then id ascending (the reference's
 *                     partial_sort leaves equal values in libstdc++'s order)
 *   top_p             device double [batch][topn]: exp(x - max) / Z of those ids
 * Entries k..topn-1 of a row are left as they were. */
zs_status zs_logits_stats(zs_handle h, const float* logits, int64_t ld, int32_t batch,
                          int32_t n_vocab, int32_t topn, double* out_min, double* out_max,
                          double* out_z, int32_t* top_ids, double* top_p, void* stream);

/* ---------------------------------------------------------------------------------
 * Vocab-sharded sampling (tensor-parallel lm_head layout).  Rank g of n_ranks
 * holds columns [vocab_offset, vocab_offset + n_local) of every row.  No
 * counterpart function in the reference (its sampler sees whole rows); per row the
 * result is sample_token's (src/sample.cpp:32-102) on the whole row.  Each rank
 *   1. zs_shard_partials: selects its local candidates -> a partial block area
 *      (per row: local top-k keys, local max, local sum-exp, flags);
 *   2. exchanges blocks (any transport: NCCL, torch.distributed), either
 *      a. all of them to every rank (all-gather), then zs_shard_merge merges every
 *         row on every rank; or
 *      b. row-owner: rank o owns rows zs_shard_owner_rows(o); every rank sends the
 *         zs_shard_row_spans of o's rows to o, o merges only its rows
 *         (zs_shard_merge_rows), then the owners' ids and Rng states are
 *         all-gathered.  The merge work per rank shrinks with n_ranks.
 * Every rank ends with identical ids and rng states.  zs_sample_sharded does the
 * whole step with NCCL itself (route b).  All ranks must pass the same batch,
 * n_vocab_total, n_ranks and params.
 * --------------------------------------------------------------------------------- */

/* Bytes of one rank's partial block area (the all-gather send size), for this batch. */
zs_status zs_shard_partial_bytes(int32_t batch, int32_t n_vocab_total, int32_t n_ranks,
                                 const zs_params* params, int32_t params_per_row,
                                 int64_t* out_bytes);

zs_status zs_shard_partials(zs_handle h, const float* logits_local, int64_t ld, int32_t batch,
                            int32_t n_local, int32_t vocab_offset, int32_t n_vocab_total,
                            int32_t n_ranks, const zs_params* params, int32_t params_per_row,
                            const int32_t* history, int64_t history_ld,
                            const int32_t* history_len, void* partial_out, int32_t want_log_z,
                            void* stream);

/* gathered: device, n_ranks partial block areas back to back (rank order). */
zs_status zs_shard_merge(zs_handle h, const void* gathered, int32_t n_ranks, int32_t batch,
                         int32_t n_vocab_total, const zs_params* params, int32_t params_per_row,
                         uint64_t* rng_state, int32_t* out_ids, const zs_extras* extras,
                         void* stream);

/* The rows rank `rank` owns in the row-owner exchange: [*row_begin, *row_begin +
 * *row_count), R = ceil(batch / n_ranks) rows per rank in rank order, so the owners'
 * shares sit back to back in an array of n_ranks * R entries (the last ranks may own
 * fewer rows, or none). */
zs_status zs_shard_owner_rows(int32_t batch, int32_t n_ranks, int32_t rank, int32_t* row_begin,
                              int32_t* row_count);

/* Byte ranges of one rank's partial block area that hold every block the merge of
 * rows [row_begin, row_begin + row_count) reads: *n_spans (at most 3) pairs
 * (offset, length) in spans[0 .. 2 * *n_spans).  The owner of those rows needs these
 * ranges of every rank's area, each at the same offsets inside that rank's slot of
 * its gathered buffer. */
zs_status zs_shard_row_spans(int32_t batch, int32_t n_vocab_total, int32_t n_ranks,
                             const zs_params* params, int32_t params_per_row, int32_t row_begin,
                             int32_t row_count, int64_t* spans, int32_t* n_spans);

/* zs_shard_merge for rows [row_begin, row_begin + row_count) only.  `gathered` has
 * the layout of zs_shard_merge's, but only the zs_shard_row_spans of these rows need
 * to be filled; only these rows' entries of rng_state, out_ids and extras are read
 * or written (indexed by row, 0 .. batch - 1). */
zs_status zs_shard_merge_rows(zs_handle h, const void* gathered, int32_t n_ranks, int32_t batch,
                              int32_t row_begin, int32_t row_count, int32_t n_vocab_total,
                              const zs_params* params, int32_t params_per_row,
                              uint64_t* rng_state, int32_t* out_ids, const zs_extras* extras,
                              void* stream);

/* The whole sharded step with an ncclComm_t (passed as void*) created by the caller
 * against the NCCL that this process has loaded (libnccl.so.2 is resolved at run
 * time); n_ranks must equal the communicator's size.  Without extras it takes the
 * row-owner route (grouped ncclSend/ncclRecv of the owners' block spans, the owner's
 * merge, an in-place ncclAllGather of ids and Rng states); with extras (row info or
 * candidate lists for every row) every rank merges every row after one all-gather.
 *
 * Failure handling: with a collective timeout (zs_set_collective_timeout, default
 * 30000 ms) the call waits, before it returns, until its work on `stream` is done,
 * polling ncclCommGetAsyncError.  If NCCL reports an error, or the deadline passes
 * (a rank stopped taking part, so the collective cannot complete), it calls
 * ncclCommAbort on the communicator, which ends the waiting NCCL kernels, and returns
 * ZS_ERR_NCCL; the communicator is then freed and must not be used or destroyed
 * again (create a new one), and out_ids / rng_state hold no valid result.  The
 * handle stays usable.  A timeout of 0 makes the call asynchronous (no wait, no
 * abort: the caller watches the communicator).  Non-blocking communicators
 * (ncclInProgress) are polled within the same deadline.
 * The reference has no failure path but exiting with "error:" (src/main.cpp:815-818). */
zs_status zs_sample_sharded(zs_handle h, const float* logits_local, int64_t ld, int32_t batch,
                            int32_t n_local, int32_t vocab_offset, int32_t n_vocab_total,
                            int32_t n_ranks, const zs_params* params, int32_t params_per_row,
                            const int32_t* history, int64_t history_ld,
                            const int32_t* history_len, uint64_t* rng_state, int32_t* out_ids,
                            const zs_extras* extras, void* nccl_comm, void* stream);

/* zs_sample_sharded's bound, per handle, in milliseconds (0 = do not wait). */
zs_status zs_set_collective_timeout(zs_handle h, int32_t timeout_ms);

/* ---------------------------------------------------------------------------------
 * zs_sample_noalloc: zs_sample without any memory allocation.  No counterpart in
 * the reference (sample_token needs no device scratch).
 *
 * For callers that must not allocate while they sample: a serving loop that gave
 * nearly all device memory to its KV-cache pool at start-up has nothing left for
 * a library's cudaMalloc in mid-run, and a cudaFree in a decode step waits for the
 * whole device.  This call uses a fixed scratch of ZS_NOALLOC_SCRATCH_BYTES in
 * static device memory of the library instead, and calls no allocating routine.
 *
 * Same kernels and results as zs_sample with one shared zs_params, on the CURRENT
 * device (no handle).  Differences:
 *   - a row's candidate blocks must fit the scratch: a small batch is cut into
 *     fewer vocabulary slices than zs_sample would use when needed, and a batch
 *     that does not fit even at one slice per row is rejected with
 *     ZS_ERR_INVALID_ARGUMENT before anything is launched.  Without a repeat
 *     penalty, over 151,936 columns, the most rows one call takes are 2,072 at
 *     top_k 321 to 1280 (e.g. 1024), 14,208 at the default shortlist of 256 and
 *     about 78,000 at top_k 50: the blocks take about (batch + 2 w) x (16 + 8 k)
 *     bytes, w = 1,776 warps for k <= 320 and 1,036 above;
 *   - rows whose top_k + repeat window exceed 2048, or whose window exceeds 512,
 *     are rejected (that path needs a workspace sized by the vocabulary);
 *   - no extras (row info, candidate lists).
 * device_status: NULL, or a device int32 the caller zeroes before first use; a
 *   kernel that gives up on a bounded wait stores ZS_ERR_DEVICE_TIMEOUT there.
 * Each call clears the scratch's fail counter itself (cudaMemsetAsync on `stream`);
 *   nothing else in the scratch needs to start at zero.
 * The first call on a device does a one-time set-up (kernel attributes, the
 *   scratch address); when that happens lazily, make the first call before any
 *   stream capture starts.
 * There is ONE scratch per device: calls in flight at the same time on one device
 *   (other streams, other threads) race on it and corrupt each other's results.
 *   Order them, e.g. by issuing them all on one stream.
 * --------------------------------------------------------------------------------- */
#define ZS_NOALLOC_SCRATCH_BYTES (32u << 20)

zs_status zs_sample_noalloc(const float* logits, int64_t ld, int32_t batch, int32_t n_vocab,
                            const zs_params* params, const int32_t* history,
                            int64_t history_ld, const int32_t* history_len,
                            uint64_t* rng_state, int32_t* out_ids, int32_t* device_status,
                            void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ZS_SAMPLER_H_ */
