// zen/sample.h -- zeninfer's sampler API (src/sample.h of the reference),
// served by the B200 sampler in libzs_sampler.so.
//
// Drop-in for the reference header: same namespace, types, defaults and
// signatures, so cmd_generate (src/main.cpp:615-628) compiles unchanged against
// it.  Two members are added to Rng (state / set_state) so the device can carry
// the generator state; next() and uniform() are the reference's xorshift64*.
//
// The functions copy the host logits row to the current CUDA device, run the
// sampler kernels there and copy the id back (one row per call, synchronous).
// For batched, stream-ordered device use see zs_sampler.h.  Errors a CUDA call
// reports are thrown as std::runtime_error (the reference's CLI prints any
// std::exception as "error: ..." and exits 1, src/main.cpp:815-818).
#pragma once

#include <cstdint>
#include <vector>

namespace zen {

struct SamplingParams {
    float temp = 0.0f;            // <= 0 means greedy
    int top_k = 0;                // 0 = disabled (256-token shortlist)
    float top_p = 1.0f;           // 1.0 = disabled (nucleus over the shortlist)
    float repeat_penalty = 1.0f;  // 1.0 = disabled
    int repeat_last_n = 64;
};

// xorshift64*; seed 0 is replaced by 0x9E3779B97F4A7C15.
class Rng {
  public:
    explicit Rng(uint64_t seed) : s_(seed ? seed : 0x9E3779B97F4A7C15ull) {}
    uint64_t next();
    double uniform();  // [0, 1)

    uint64_t state() const { return s_; }
    void set_state(uint64_t s) { s_ = s; }

  private:
    uint64_t s_;
};

// First index of the maximum (a NaN at index 0 yields 0).
int32_t argmax_token(const float* logits, int n);

// Samples one token id from `logits` (not modified).  `history` is the tokens
// generated so far, used only for the repetition penalty.  top-p acts on the
// top-K shortlist (K = top_k, or 256 when top_k is 0).  One rng draw per
// non-greedy call.
int32_t sample_token(const float* logits, int n, const SamplingParams& p,
                     const std::vector<int32_t>& history, Rng& rng);

}  // namespace zen
