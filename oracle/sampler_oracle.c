/*
 * sampler_oracle.c -- CPU restatement of zeninfer's token sampler.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA sampler in
 * zeninfer_b200/csrc; nothing in the product links, loads or calls it.  Only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg use it.
 *
 * It restates src/sample.cpp of the reference step by step (same f32 / f64
 * expressions, same summation order) with one deliberate change: the shortlist
 * order is total -- value descending, then token id ascending -- where the
 * reference's std::nth_element / std::sort (src/sample.cpp:62-67) order equal
 * values in whatever way libstdc++'s introselect leaves them.  NaN logits rank
 * below every number (the reference's comparator is not a strict weak order
 * with NaNs, so its output there is unspecified).  On rows without ties at the
 * shortlist boundary it must agree bit for bit with the reference compiled
 * unchanged (oracle/_ref); tests/test_oracle.py checks exactly that.
 *
 * Besides the sampled id it exposes what the reference keeps internal: the
 * sorted shortlist (ids, values), the shortlist softmax p_i, the nucleus size m,
 * the uniform draw r and the distance of r to the nearest CDF boundary.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* Same field order and meaning as zen::SamplingParams (src/sample.h:9-15). */
typedef struct zo_params {
    float temp;
    int32_t top_k;
    float top_p;
    float repeat_penalty;
    int32_t repeat_last_n;
} zo_params;

/* Per-row diagnostics; same layout as zs_row_info in include/zs_sampler.h. */
typedef struct zo_row_info {
    float max_logit;
    int32_t k;
    int32_t m;
    int32_t pos;
    double r;
    double sum;
    double boundary;
    double log_z;
} zo_row_info;

#define ZO_TOPP_SHORTLIST 256 /* kTopPShortlist, src/sample.cpp:12 */

/* xorshift64*  (src/sample.h:18-26, src/sample.cpp:15-22). */
uint64_t zo_rng_seed(uint64_t seed) { return seed ? seed : 0x9E3779B97F4A7C15ull; }

uint64_t zo_rng_next(uint64_t* s) {
    uint64_t x = *s;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *s = x;
    return x * 2685821657736338717ull;
}

double zo_rng_uniform(uint64_t* s) {
    return (double)(zo_rng_next(s) >> 11) * (1.0 / 9007199254740992.0);
}

/* argmax_token, src/sample.cpp:24-30: strict '>' so the first maximum wins. */
int32_t zo_argmax(const float* x, int n) {
    int32_t best = 0;
    for (int i = 1; i < n; ++i)
        if (x[i] > x[best]) best = i;
    return best;
}

/* Total order key: value descending (NaN lowest, -0 == +0), then id ascending. */
static inline uint32_t ord_of(float v) {
    if (v != v) return 0u;
    if (v == 0.0f) v = 0.0f;
    uint32_t u;
    memcpy(&u, &v, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

static inline uint64_t key_of(float v, int32_t id) {
    return ((uint64_t)ord_of(v) << 32) | (uint64_t)(uint32_t)(~(uint32_t)id);
}

static inline int32_t id_of(uint64_t key) { return (int32_t)(~(uint32_t)(key & 0xffffffffu)); }

/* Rearranges a[0..n) so that a[0..k) hold the k largest keys (keys are unique). */
static void select_largest(uint64_t* a, size_t n, size_t k) {
    size_t lo = 0, hi = n;
    if (k == 0 || k >= n) return;
    while (hi - lo > 1) {
        size_t mid = lo + (hi - lo) / 2;
        uint64_t x = a[lo], y = a[mid], z = a[hi - 1];
        size_t pidx;
        if ((x < y) == (y < z)) pidx = mid;
        else if ((y < x) == (x < z)) pidx = lo;
        else pidx = hi - 1;
        uint64_t piv = a[pidx];
        a[pidx] = a[hi - 1];
        a[hi - 1] = piv;
        size_t store = lo;
        for (size_t i = lo; i < hi - 1; ++i) {
            if (a[i] > piv) {
                uint64_t t = a[i];
                a[i] = a[store];
                a[store] = t;
                ++store;
            }
        }
        a[hi - 1] = a[store];
        a[store] = piv;
        if (store == k || store + 1 == k) return;
        if (store > k) hi = store;
        else lo = store + 1;
    }
}

static int cmp_desc(const void* pa, const void* pb) {
    uint64_t a = *(const uint64_t*)pa, b = *(const uint64_t*)pb;
    return (a < b) - (a > b);
}

/* Applies the repetition penalty in place (src/sample.cpp:40-50): compounds per
 * history entry, skips out-of-range ids, only over the last repeat_last_n. */
static void apply_penalty(float* x, int n, const zo_params* p, const int32_t* hist, int hist_len) {
    if (!(p->repeat_penalty != 1.0f) || hist_len <= 0 || hist == NULL) return;
    size_t keep = (size_t)(p->repeat_last_n > 0 ? p->repeat_last_n : 0);
    size_t len = (size_t)hist_len;
    size_t begin = len > keep ? len - keep : 0;
    for (size_t i = begin; i < len; ++i) {
        int32_t id = hist[i];
        if (id < 0 || id >= n) continue;
        float v = x[id];
        x[id] = (v > 0.0f) ? v / p->repeat_penalty : v * p->repeat_penalty;
    }
}

/*
 * One row, following sample_token (src/sample.cpp:32-102).
 *   work: n floats + n uint64 of scratch, or NULL to allocate.
 *   cand_ids/cand_vals/cand_probs (nullable, capacity cand_cap): sorted shortlist
 *   and its softmax p_i (before the nucleus rescale).
 *   full_z: when nonzero, info->log_z = log(sum_i exp((x_i - max_l) * inv_t)) over
 *   the whole penalised row in f64 (inv_t = 1 for greedy rows).
 */
int32_t zo_sample_row(const float* logits, int n, const zo_params* p, const int32_t* hist,
                      int hist_len, uint64_t* state, int32_t* cand_ids, float* cand_vals,
                      double* cand_probs, int cand_cap, zo_row_info* info, int full_z,
                      void* work) {
    zo_row_info local;
    if (info == NULL) info = &local;
    info->max_logit = 0.0f;
    info->k = 0;
    info->m = 0;
    info->pos = -1;
    info->r = 0.0;
    info->sum = 0.0;
    info->boundary = 0.0;
    info->log_z = NAN;
    if (n <= 0) return 0;

    int own = (work == NULL);
    if (own) work = malloc((size_t)n * (sizeof(float) + sizeof(uint64_t)));
    uint64_t* keys = (uint64_t*)work;
    float* x = (float*)(keys + n);
    memcpy(x, logits, (size_t)n * sizeof(float));
    apply_penalty(x, n, p, hist, hist_len);

    if (full_z) {
        float inv_t = (p->temp > 0.0f) ? 1.0f / p->temp : 1.0f;
        float mx = x[0];
        for (int i = 1; i < n; ++i) mx = (mx < x[i]) ? x[i] : mx;
        double z = 0.0;
        for (int i = 0; i < n; ++i) z += exp(((double)x[i] - (double)mx) * (double)inv_t);
        info->log_z = log(z);
    }

    if (p->temp <= 0.0f) {
        int32_t id = zo_argmax(x, n);
        info->max_logit = x[id];
        if (own) free(work);
        return id;
    }

    const float inv_temp = 1.0f / p->temp;
    float max_l = x[0];
    for (int i = 1; i < n; ++i) max_l = (max_l < x[i]) ? x[i] : max_l; /* std::max */
    info->max_logit = max_l;

    int k = (p->top_k > 0) ? (p->top_k < n ? p->top_k : n)
                           : (ZO_TOPP_SHORTLIST < n ? ZO_TOPP_SHORTLIST : n);
    for (int i = 0; i < n; ++i) keys[i] = key_of(x[i], i);
    select_largest(keys, (size_t)n, (size_t)k);
    qsort(keys, (size_t)k, sizeof(uint64_t), cmp_desc);

    double* prob = (double*)malloc((size_t)k * sizeof(double));
    double sum = 0.0;
    for (int i = 0; i < k; ++i) {
        const double e = exp(((double)x[id_of(keys[i])] - (double)max_l) * (double)inv_temp);
        prob[i] = e;
        sum += e;
    }
    for (int i = 0; i < k; ++i) prob[i] /= sum;
    for (int i = 0; i < k && i < cand_cap; ++i) {
        int32_t id = id_of(keys[i]);
        if (cand_ids) cand_ids[i] = id;
        if (cand_vals) cand_vals[i] = x[id];
        if (cand_probs) cand_probs[i] = prob[i];
    }

    int m = k;
    if (p->top_p < 1.0f) {
        double acc = 0.0;
        m = 0;
        while (m < k && acc < (double)p->top_p) {
            acc += prob[m];
            ++m;
        }
        if (m == 0) m = 1;
        double rescale = 0.0;
        for (int i = 0; i < m; ++i) rescale += prob[i];
        for (int i = 0; i < m; ++i) prob[i] /= rescale;
    }

    const double r = zo_rng_uniform(state);
    double acc = 0.0, prev = 0.0;
    int pos = m - 1;
    int hit = 0;
    for (int i = 0; i < m; ++i) {
        prev = acc;
        acc += prob[i];
        if (r < acc) {
            pos = i;
            hit = 1;
            break;
        }
    }
    double d;
    if (hit) {
        double a = r - prev, b = acc - r;
        d = a < b ? a : b;
    } else {
        d = r - acc;
    }
    int32_t out = id_of(keys[pos]);
    info->k = k;
    info->m = m;
    info->pos = pos;
    info->r = r;
    info->sum = sum;
    info->boundary = d;
    free(prob);
    if (own) free(work);
    return out;
}

/* ---- batched, multithreaded driver (rows are independent) ---- */

typedef struct {
    const float* logits;
    int64_t ld;
    int B, n;
    const zo_params* params;
    int params_per_row;
    const int32_t* hist;
    int64_t hist_ld;
    const int32_t* hist_len;
    uint64_t* states;
    int32_t* out_ids;
    int32_t* cand_ids;
    float* cand_vals;
    double* cand_probs;
    int cand_ld;
    zo_row_info* infos;
    int full_z;
    int next_row;
    pthread_mutex_t mu;
} zo_batch;

static void* zo_worker(void* arg) {
    zo_batch* b = (zo_batch*)arg;
    void* work = malloc((size_t)b->n * (sizeof(float) + sizeof(uint64_t)) + 64);
    for (;;) {
        pthread_mutex_lock(&b->mu);
        int r = b->next_row++;
        pthread_mutex_unlock(&b->mu);
        if (r >= b->B) break;
        const zo_params* p = b->params + (b->params_per_row ? r : 0);
        const int32_t* h = b->hist ? b->hist + (int64_t)r * b->hist_ld : NULL;
        int hl = b->hist_len ? b->hist_len[r] : 0;
        size_t co = (size_t)r * (size_t)(b->cand_ld > 0 ? b->cand_ld : 0);
        b->out_ids[r] = zo_sample_row(b->logits + (int64_t)r * b->ld, b->n, p, h, hl,
                                      &b->states[r], b->cand_ids ? b->cand_ids + co : NULL,
                                      b->cand_vals ? b->cand_vals + co : NULL,
                                      b->cand_probs ? b->cand_probs + co : NULL, b->cand_ld,
                                      b->infos ? &b->infos[r] : NULL, b->full_z, work);
    }
    free(work);
    return NULL;
}

int zo_sample_rows(const float* logits, int64_t ld, int B, int n, const zo_params* params,
                   int params_per_row, const int32_t* hist, int64_t hist_ld,
                   const int32_t* hist_len, uint64_t* states, int32_t* out_ids, int32_t* cand_ids,
                   float* cand_vals, double* cand_probs, int cand_ld, zo_row_info* infos,
                   int full_z, int nthreads) {
    zo_batch b;
    b.logits = logits;
    b.ld = ld;
    b.B = B;
    b.n = n;
    b.params = params;
    b.params_per_row = params_per_row;
    b.hist = hist;
    b.hist_ld = hist_ld;
    b.hist_len = hist_len;
    b.states = states;
    b.out_ids = out_ids;
    b.cand_ids = cand_ids;
    b.cand_vals = cand_vals;
    b.cand_probs = cand_probs;
    b.cand_ld = cand_ld;
    b.infos = infos;
    b.full_z = full_z;
    b.next_row = 0;
    pthread_mutex_init(&b.mu, NULL);
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    for (int t = 1; t < nthreads; ++t) pthread_create(&th[t], NULL, zo_worker, &b);
    zo_worker(&b);
    for (int t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
    pthread_mutex_destroy(&b.mu);
    return 0;
}

/*
 * The display numbers of the `logits` command, src/main.cpp:473-503, one row at a
 * time (test infrastructure, like everything here): min and max as double from
 * starts of 1e30 / -1e30 (std::min / std::max ignore a NaN the way these compares
 * do), Z = sum of exp((double)x - max) in index order, the top-k ids with k =
 * clamp(topn, 1, n) in the total order (value descending, id ascending; the
 * reference's partial_sort leaves ties in libstdc++'s order) and p = exp(x - max)/Z.
 * top_ids / top_p rows are top_ld apart.
 */
int zo_logits_stats(const float* logits, int64_t ld, int B, int n, int topn, double* out_min,
                    double* out_max, double* out_z, int32_t* top_ids, double* top_p,
                    int64_t top_ld) {
    if (n <= 0) return -1;
    const int k = topn < 1 ? 1 : (topn > n ? n : topn);
    uint64_t* keys = (uint64_t*)malloc((size_t)n * sizeof(uint64_t));
    if (!keys) return -1;
    for (int r = 0; r < B; ++r) {
        const float* x = logits + (int64_t)r * ld;
        double mx = -1e30, mn = 1e30;
        for (int i = 0; i < n; ++i) {
            const double v = (double)x[i];
            mx = (mx < v) ? v : mx; /* std::max<double>(max_l, v) */
            mn = (v < mn) ? v : mn; /* std::min<double>(min_l, v) */
        }
        double z = 0.0;
        for (int i = 0; i < n; ++i) z += exp((double)x[i] - mx);
        for (int i = 0; i < n; ++i) keys[i] = key_of(x[i], i);
        select_largest(keys, (size_t)n, (size_t)k);
        qsort(keys, (size_t)k, sizeof(uint64_t), cmp_desc);
        out_min[r] = mn;
        out_max[r] = mx;
        out_z[r] = z;
        for (int i = 0; i < k; ++i) {
            const int32_t id = id_of(keys[i]);
            top_ids[(int64_t)r * top_ld + i] = id;
            top_p[(int64_t)r * top_ld + i] = exp((double)x[id] - mx) / z;
        }
    }
    free(keys);
    return 0;
}

/* ---- lm_head of Model::eval (src/model.cpp:401-403) as the B200 path computes it --
 * rmsnorm (src/model.cpp:31-38): sum of x^2 in double, in order; scale =
 * 1/sqrt(sum/n + eps); xn_i = (float)((double)x_i * scale * (double)w_i).  Every
 * product is of two floats, so exact in double: contraction cannot change it.
 * The device path rounds xn to bfloat16 (nearest even) for the tensor cores and
 * takes the weights as bfloat16; the logits here are then the reference's
 * dot_f32_scalar (src/kernels.cpp: double accumulation in order, one rounding
 * to float at the end) over those bfloat16 values, which the tensor cores'
 * f32 accumulation approximates. */
static inline float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static inline uint16_t f32_to_bf16_rne(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u); /* NaN */
    const uint32_t lsb = (u >> 16) & 1u;
    return (uint16_t)((u + 0x7fffu + lsb) >> 16);
}

void zo_rmsnorm_bf16(const float* x, const float* w, int n, float eps, float* out_f32,
                     uint16_t* out_bf16) {
    double sum = 0.0;
    for (int i = 0; i < n; ++i) sum += (double)x[i] * (double)x[i];
    const double scale = 1.0 / sqrt(sum / (double)n + (double)eps);
    for (int i = 0; i < n; ++i) {
        const float v = (float)((double)x[i] * scale * (double)w[i]);
        if (out_f32) out_f32[i] = v;
        if (out_bf16) out_bf16[i] = f32_to_bf16_rne(v);
    }
}

typedef struct {
    const float* hidden;
    int64_t hld;
    int B, E, V;
    const float* norm_w;
    float eps;
    const uint16_t* w;
    uint16_t* out_xn;
    float* logits;
    int64_t lld;
    int next;
    pthread_mutex_t mu;
} zo_lm_batch;

static void* zo_lm_worker(void* arg) {
    zo_lm_batch* b = (zo_lm_batch*)arg;
    float* xf = (float*)malloc((size_t)b->E * sizeof(float));
    uint16_t* xb = (uint16_t*)malloc((size_t)b->E * sizeof(uint16_t));
    for (;;) {
        pthread_mutex_lock(&b->mu);
        const int r = b->next++;
        pthread_mutex_unlock(&b->mu);
        if (r >= b->B) break;
        zo_rmsnorm_bf16(b->hidden + (int64_t)r * b->hld, b->norm_w, b->E, b->eps, xf, xb);
        if (b->out_xn) memcpy(b->out_xn + (int64_t)r * b->E, xb, (size_t)b->E * 2);
        for (int i = 0; i < b->E; ++i) xf[i] = bf16_to_f32(xb[i]);
        for (int v = 0; v < b->V; ++v) {
            const uint16_t* wr = b->w + (int64_t)v * b->E;
            double acc = 0.0;
            for (int i = 0; i < b->E; ++i) acc += (double)xf[i] * (double)bf16_to_f32(wr[i]);
            b->logits[(int64_t)r * b->lld + v] = (float)acc;
        }
    }
    free(xf);
    free(xb);
    return NULL;
}

/* hidden [B][hld] f32, norm_w [E], w [V][E] bfloat16 bits; out_xn (nullable)
 * [B][E] bfloat16 bits; logits [B][lld]. */
int zo_lmhead_rows(const float* hidden, int64_t hld, int B, int E, const float* norm_w, float eps,
                   const uint16_t* w, int V, uint16_t* out_xn, float* logits, int64_t lld,
                   int nthreads) {
    zo_lm_batch b = {hidden, hld, B, E, V, norm_w, eps, w, out_xn, logits, lld, 0,
                     PTHREAD_MUTEX_INITIALIZER};
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    for (int t = 1; t < nthreads; ++t) pthread_create(&th[t], NULL, zo_lm_worker, &b);
    zo_lm_worker(&b);
    for (int t = 1; t < nthreads; ++t) pthread_join(th[t], NULL);
    return 0;
}

/* ---- the lm_head as the reference computes it by default (f32 throughout) ----
 * src/kernels.cpp:52-78 dot_f32_avx2: 32 float accumulators (four vectors of 8),
 * accumulator l takes a[i] * b[i] for i = l, l + 32, ... by fused multiply-add in
 * order; then (acc0 + acc1) + (acc2 + acc3) per vector lane, the upper half of the
 * 8 added to the lower, [0] + [2] and [1] + [3], and those two; the result in double
 * plus the terms past the last multiple of 32 in double, in order; one float
 * rounding.  a is the weight row, b the normalised row (src/kernels.cpp:85). */
float zo_dot_avx2_order(const float* a, const float* b, int64_t n) {
    float acc[32];
    for (int l = 0; l < 32; ++l) acc[l] = 0.0f;
    int64_t i = 0;
    for (; i + 32 <= n; i += 32)
        for (int l = 0; l < 32; ++l) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
    float s[8], t[4];
    for (int e = 0; e < 8; ++e) s[e] = (acc[e] + acc[8 + e]) + (acc[16 + e] + acc[24 + e]);
    for (int m = 0; m < 4; ++m) t[m] = s[m] + s[m + 4];
    const float t20 = t[0] + t[2], t21 = t[1] + t[3];
    const float t3 = t20 + t21;
    double total = (double)t3;
    for (; i < n; ++i) total += (double)a[i] * (double)b[i];
    return (float)total;
}

/* hidden [B][hld] f32, norm_w [E], w [V][E] bfloat16 bits; out_xn (nullable) [B][E]
 * f32; logits [B][lld]: src/model.cpp:31-38 rmsnorm (f32 out) then the dot above. */
int zo_lmhead_f32_rows(const float* hidden, int64_t hld, int B, int E, const float* norm_w,
                       float eps, const uint16_t* w, int V, float* out_xn, float* logits,
                       int64_t lld) {
    float* xf = (float*)malloc((size_t)E * sizeof(float));
    float* wf = (float*)malloc((size_t)E * sizeof(float));
    for (int r = 0; r < B; ++r) {
        zo_rmsnorm_bf16(hidden + (int64_t)r * hld, norm_w, E, eps, xf, NULL);
        if (out_xn) memcpy(out_xn + (int64_t)r * E, xf, (size_t)E * sizeof(float));
        for (int v = 0; v < V; ++v) {
            const uint16_t* wr = w + (int64_t)v * E;
            for (int i = 0; i < E; ++i) wf[i] = bf16_to_f32(wr[i]);
            logits[(int64_t)r * lld + v] = zo_dot_avx2_order(wf, xf, E);
        }
    }
    free(xf);
    free(wf);
    return 0;
}
