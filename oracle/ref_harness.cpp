// ref_harness.cpp -- batch driver around the reference sampler, compiled unchanged.
//
// TEST INFRASTRUCTURE ONLY (the checker and the timed CPU baseline).  The
// Makefile in this directory compiles the reference's own src/sample.cpp
// together with this file into oracle/_ref/libzen_ref.so; nothing of the
// reference's source is copied.  The functions here only loop over rows and
// call zen::sample_token / zen::argmax_token / zen::Rng exactly as
// cmd_generate does (src/main.cpp:615-628): one Rng per row, one call per row.
#include <atomic>
#include <cstdint>
#include <thread>
#include <vector>

#include "kernels.h"
#include "model.h"
#include "sample.h"

namespace {
struct RefParams {  // same layout as zen::SamplingParams
    float temp;
    int32_t top_k;
    float top_p;
    float repeat_penalty;
    int32_t repeat_last_n;
};
}  // namespace

extern "C" {

// Samples B rows with the reference sampler on `nthreads` host threads.
//   seeds[r]        seed given to zen::Rng for row r (the Rng is built per row)
//   out_next[r]     (nullable) the Rng's next() output *after* the call, which
//                   shows how many draws sample_token consumed
int zref_sample_rows(const float* logits, int64_t ld, int B, int n, const RefParams* params,
                     int params_per_row, const int32_t* hist, int64_t hist_ld,
                     const int32_t* hist_len, const uint64_t* seeds, int32_t* out_ids,
                     uint64_t* out_next, int nthreads) {
    std::atomic<int> next_row{0};
    auto work = [&]() {
        for (;;) {
            const int r = next_row.fetch_add(1);
            if (r >= B) break;
            const RefParams& rp = params[params_per_row ? r : 0];
            zen::SamplingParams sp;
            sp.temp = rp.temp;
            sp.top_k = rp.top_k;
            sp.top_p = rp.top_p;
            sp.repeat_penalty = rp.repeat_penalty;
            sp.repeat_last_n = rp.repeat_last_n;
            std::vector<int32_t> h;
            if (hist && hist_len && hist_len[r] > 0)
                h.assign(hist + r * hist_ld, hist + r * hist_ld + hist_len[r]);
            zen::Rng rng(seeds[r]);
            out_ids[r] = zen::sample_token(logits + r * ld, n, sp, h, rng);
            if (out_next) out_next[r] = rng.next();
        }
    };
    if (nthreads < 1) nthreads = 1;
    std::vector<std::thread> pool;
    for (int t = 1; t < nthreads; ++t) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
    return 0;
}

int32_t zref_argmax(const float* logits, int n) { return zen::argmax_token(logits, n); }

// The lm_head of Model::eval (src/model.cpp:401-403) for B independent rows:
// zen::rmsnorm of the row's hidden state with output_norm, then
// zen::matvec_f32_impl over output_ ([V][E] f32, row-major) with the chosen
// implementation (0 scalar, 1 AVX2), rows spread over `nthreads` host threads.
//   out_xn   (nullable) [B][E] the normalised row
//   logits   [B][lld]
int zref_lmhead_rows(const float* hidden, int64_t hld, int B, int E, const float* norm_w,
                     float eps, const float* w, int V, float* out_xn, float* logits, int64_t lld,
                     int impl, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    std::atomic<int> next{0};
    auto work = [&]() {
        std::vector<float> xn((size_t)E);
        for (int r; (r = next.fetch_add(1)) < B;) {
            zen::rmsnorm(xn.data(), hidden + (int64_t)r * hld, norm_w, E, eps);
            if (out_xn)
                for (int i = 0; i < E; ++i) out_xn[(int64_t)r * E + i] = xn[(size_t)i];
            zen::matvec_f32_impl(logits + (int64_t)r * lld, xn.data(), w, V, E,
                                 impl ? zen::Impl::Avx2 : zen::Impl::Scalar);
        }
    };
    std::vector<std::thread> pool;
    for (int t = 1; t < nthreads; ++t) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
    return 0;
}

// zen::matvec_f32_impl alone over caller-supplied normalised rows xn [B][E].
int zref_matvec_rows(const float* xn, int B, int E, const float* w, int V, float* logits,
                     int64_t lld, int impl, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    std::atomic<int> next{0};
    auto work = [&]() {
        for (int r; (r = next.fetch_add(1)) < B;)
            zen::matvec_f32_impl(logits + (int64_t)r * lld, xn + (int64_t)r * E, w, V, E,
                                 impl ? zen::Impl::Avx2 : zen::Impl::Scalar);
    };
    std::vector<std::thread> pool;
    for (int t = 1; t < nthreads; ++t) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
    return 0;
}

// First `count` outputs of zen::Rng(seed).next() and the first uniform().
void zref_rng_stream(uint64_t seed, int count, uint64_t* out_next, double* out_uniform) {
    zen::Rng a(seed);
    for (int i = 0; i < count; ++i) out_next[i] = a.next();
    zen::Rng b(seed);
    *out_uniform = b.uniform();
}

}  // extern "C"
