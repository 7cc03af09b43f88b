// sample_shim.cpp -- zen::argmax_token / zen::sample_token / zen::Rng
// (include/zen/sample.h) on top of the C ABI.  One host row per call: the row
// goes through a pinned staging buffer to the device, the sampler kernels run
// on a per-thread stream, and the id (and Rng state) come back.
#include <cuda_runtime.h>

#include <cstring>
#include <stdexcept>
#include <string>

#include "zen/sample.h"
#include "zs_sampler.h"

namespace zen {

uint64_t Rng::next() {
    s_ ^= s_ >> 12;
    s_ ^= s_ << 25;
    s_ ^= s_ >> 27;
    return s_ * 2685821657736338717ull;
}

double Rng::uniform() { return static_cast<double>(next() >> 11) * (1.0 / 9007199254740992.0); }

namespace {

[[noreturn]] void raise(const char* what, const std::string& detail) {
    throw std::runtime_error(std::string("zen sampler: ") + what + ": " + detail);
}

void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) raise(what, cudaGetErrorString(e));
}

void check_zs(zs_status s, const char* what) {
    if (s != ZS_OK) raise(what, std::string(zs_status_string(s)) + " (" + zs_last_error() + ")");
}

// Per host thread and device: handle, stream and staging buffers.
struct Session {
    int device = -1;
    zs_handle h = nullptr;
    cudaStream_t stream = nullptr;
    float* h_logits = nullptr;  // pinned
    float* d_logits = nullptr;
    size_t cap = 0;
    int32_t* h_hist = nullptr;  // pinned
    int32_t* d_hist = nullptr;
    size_t hist_cap = 0;
    struct Io {
        uint64_t state;
        int32_t id;
        int32_t hist_len;
    };
    Io* h_io = nullptr;  // pinned
    Io* d_io = nullptr;

    ~Session() {
        if (device < 0) return;
        cudaSetDevice(device);
        if (stream) cudaStreamDestroy(stream);
        cudaFreeHost(h_logits);
        cudaFree(d_logits);
        cudaFreeHost(h_hist);
        cudaFree(d_hist);
        cudaFreeHost(h_io);
        cudaFree(d_io);
        zs_destroy(h);
    }

    void open() {
        int dev = 0;
        check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
        if (dev == device) return;
        if (device >= 0) raise("session", "the current CUDA device changed between calls on this thread");
        check_zs(zs_create(dev, &h), "zs_create");
        device = dev;
        check_cuda(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
        check_cuda(cudaMallocHost((void**)&h_io, sizeof(Io)), "cudaMallocHost");
        check_cuda(cudaMalloc((void**)&d_io, sizeof(Io)), "cudaMalloc");
    }

    void reserve(size_t n, size_t nh) {
        if (n > cap) {
            cudaFreeHost(h_logits);
            cudaFree(d_logits);
            h_logits = nullptr;
            d_logits = nullptr;
            cap = 0;
            check_cuda(cudaMallocHost((void**)&h_logits, n * sizeof(float)), "cudaMallocHost");
            check_cuda(cudaMalloc((void**)&d_logits, n * sizeof(float)), "cudaMalloc");
            cap = n;
        }
        if (nh > hist_cap) {
            cudaFreeHost(h_hist);
            cudaFree(d_hist);
            h_hist = nullptr;
            d_hist = nullptr;
            hist_cap = 0;
            check_cuda(cudaMallocHost((void**)&h_hist, nh * sizeof(int32_t)), "cudaMallocHost");
            check_cuda(cudaMalloc((void**)&d_hist, nh * sizeof(int32_t)), "cudaMalloc");
            hist_cap = nh;
        }
    }
};

thread_local Session g_session;

int32_t run(const float* logits, int n, const SamplingParams& p,
            const std::vector<int32_t>* history, Rng* rng) {
    Session& s = g_session;
    s.open();
    const bool penal = history && !history->empty() && p.repeat_penalty != 1.0f;
    // Only the penalty window is ever read; ship just that tail.
    size_t keep = 0;
    if (penal) {
        const size_t last_n = static_cast<size_t>(p.repeat_last_n > 0 ? p.repeat_last_n : 0);
        keep = history->size() < last_n ? history->size() : last_n;
    }
    s.reserve(static_cast<size_t>(n), keep > 0 ? keep : 1);
    std::memcpy(s.h_logits, logits, static_cast<size_t>(n) * sizeof(float));
    check_cuda(cudaMemcpyAsync(s.d_logits, s.h_logits, static_cast<size_t>(n) * sizeof(float),
                               cudaMemcpyHostToDevice, s.stream),
               "cudaMemcpyAsync");
    s.h_io->state = rng ? rng->state() : 1;
    s.h_io->id = 0;
    s.h_io->hist_len = static_cast<int32_t>(keep);
    if (keep > 0) {
        std::memcpy(s.h_hist, history->data() + (history->size() - keep), keep * sizeof(int32_t));
        check_cuda(cudaMemcpyAsync(s.d_hist, s.h_hist, keep * sizeof(int32_t),
                                   cudaMemcpyHostToDevice, s.stream),
                   "cudaMemcpyAsync");
    }
    check_cuda(cudaMemcpyAsync(s.d_io, s.h_io, sizeof(Session::Io), cudaMemcpyHostToDevice, s.stream),
               "cudaMemcpyAsync");
    zs_params zp;
    zp.temp = p.temp;
    zp.top_k = p.top_k;
    zp.top_p = p.top_p;
    zp.repeat_penalty = p.repeat_penalty;
    zp.repeat_last_n = p.repeat_last_n;
    check_zs(zs_sample(s.h, s.d_logits, n, 1, n, &zp, 0, keep > 0 ? s.d_hist : nullptr,
                       static_cast<int64_t>(keep), keep > 0 ? &s.d_io->hist_len : nullptr,
                       &s.d_io->state, &s.d_io->id, nullptr, s.stream),
             "zs_sample");
    check_cuda(cudaMemcpyAsync(s.h_io, s.d_io, sizeof(Session::Io), cudaMemcpyDeviceToHost, s.stream),
               "cudaMemcpyAsync");
    check_cuda(cudaStreamSynchronize(s.stream), "cudaStreamSynchronize");
    check_zs(zs_check_device_status(s.h, s.stream), "sampler kernel");
    if (rng) rng->set_state(s.h_io->state);
    return s.h_io->id;
}

}  // namespace

int32_t argmax_token(const float* logits, int n) {
    if (n <= 0) return 0;
    SamplingParams greedy;
    return run(logits, n, greedy, nullptr, nullptr);
}

int32_t sample_token(const float* logits, int n, const SamplingParams& p,
                     const std::vector<int32_t>& history, Rng& rng) {
    if (n <= 0) return 0;
    return run(logits, n, p, &history, &rng);
}

}  // namespace zen
