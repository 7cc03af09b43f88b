// bench_host_api.cpp -- times the drop-in C++ API (include/zen/sample.h) the way
// zeninfer's generate loop calls it (src/main.cpp:628): one host logits row per
// call, the generated ids as a std::vector history, one zen::Rng advanced in
// place.  Every call copies the row to the device, samples, and copies the id
// and the Rng state back (sample_shim.cpp).
//
//   bench_host_api <row.f32> <n> <calls> <temp> <top_k> <top_p> <penalty> <last_n> <hist_len>
//
// Prints one JSON object: mean, min, median and max microseconds per call, and
// the ids' checksum so a caller can compare runs.
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "zen/sample.h"

int main(int argc, char** argv) {
    if (argc != 10) {
        std::fprintf(stderr,
                     "usage: %s row.f32 n calls temp top_k top_p penalty last_n hist_len\n",
                     argv[0]);
        return 2;
    }
    const int n = std::atoi(argv[2]);
    const int calls = std::atoi(argv[3]);
    zen::SamplingParams p;
    p.temp = static_cast<float>(std::atof(argv[4]));
    p.top_k = std::atoi(argv[5]);
    p.top_p = static_cast<float>(std::atof(argv[6]));
    p.repeat_penalty = static_cast<float>(std::atof(argv[7]));
    p.repeat_last_n = std::atoi(argv[8]);
    const int hist_len = std::atoi(argv[9]);
    if (n <= 0 || calls <= 0 || hist_len < 0) return 2;
    std::vector<float> row(static_cast<size_t>(n));
    FILE* f = std::fopen(argv[1], "rb");
    if (!f || std::fread(row.data(), sizeof(float), row.size(), f) != row.size()) {
        std::fprintf(stderr, "cannot read %d floats from %s\n", n, argv[1]);
        return 2;
    }
    std::fclose(f);
    std::vector<int32_t> history;
    for (int i = 0; i < hist_len; ++i) history.push_back((i * 997) % n);
    zen::Rng rng(42);
    try {
        for (int i = 0; i < 20; ++i) zen::sample_token(row.data(), n, p, history, rng);
        std::vector<double> us(static_cast<size_t>(calls));
        uint64_t checksum = 0;
        for (int i = 0; i < calls; ++i) {
            const auto t0 = std::chrono::steady_clock::now();
            const int32_t id = zen::sample_token(row.data(), n, p, history, rng);
            const auto t1 = std::chrono::steady_clock::now();
            us[static_cast<size_t>(i)] = std::chrono::duration<double, std::micro>(t1 - t0).count();
            checksum = checksum * 1000003u + static_cast<uint32_t>(id);
        }
        double sum = 0.0;
        for (double v : us) sum += v;
        std::vector<double> sorted = us;
        std::sort(sorted.begin(), sorted.end());
        std::printf("{\"calls\": %d, \"us_per_call\": %.3f, \"min_us\": %.3f, \"median_us\": %.3f, "
                    "\"max_us\": %.3f, \"checksum\": %llu}\n",
                    calls, sum / calls, sorted.front(), sorted[sorted.size() / 2], sorted.back(),
                    static_cast<unsigned long long>(checksum));
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
    return 0;
}
