// ref_sampler_shim.cpp — TEST INFRASTRUCTURE ONLY.
//
// Compiles chatterbox.cpp's own sample_next_token_ex (src/main.cpp:726-801)
// and chatterbox_sampling_params (src/chatterbox_t3_internal.h:113-118),
// cut out of the reference tree at build time by oracle/Makefile into
// oracle/_ref/ (git-ignored; never committed), and exposes it through a C
// entry point so the tests can compare the oracle and the CUDA sampler with
// the reference itself.  Built with the reference's defaults (C++17 GNU
// dialect, -O3, no -march: no FMA contraction on x86-64).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <random>
#include <set>
#include <vector>

namespace tts_cpp::chatterbox::detail {
#include "chatterbox_sampling_params.inc"
#include "sample_next_token_ex.inc"
}  // namespace tts_cpp::chatterbox::detail

using namespace tts_cpp::chatterbox::detail;

extern "C" {

// One call of the reference sampler with std::mt19937(seed) after
// discard(skip) outputs.  Returns the token; *used receives how many engine
// outputs the call consumed (0 or 2).
int ref_sample_next_token_ex(const float * logits, int n, const int32_t * generated, int n_gen,
                             int32_t top_k, float top_p, float temp, float repeat_penalty,
                             uint32_t seed, uint64_t skip, int * used) {
    std::vector<float> l(logits, logits + n);
    std::vector<int32_t> g(generated, generated + n_gen);
    chatterbox_sampling_params p;
    p.top_k = top_k; p.top_p = top_p; p.temp = temp; p.repeat_penalty = repeat_penalty;
    std::mt19937 rng(seed);
    rng.discard(skip);
    std::mt19937 before = rng;
    const int32_t t = sample_next_token_ex(l, g, p, rng);
    if (used) { int k = 0; while (!(before == rng) && k < 8) { before(); ++k; } *used = k; }
    return t;
}

// A whole decode-loop's worth of draws: steps x n logits, one engine; the
// history grows with every sampled token as in Engine::Impl::run_t3.
void ref_sample_sequence(const float * logits, int n, int steps, int32_t top_k, float top_p, float temp,
                         float repeat_penalty, uint32_t seed, int32_t * out) {
    chatterbox_sampling_params p;
    p.top_k = top_k; p.top_p = top_p; p.temp = temp; p.repeat_penalty = repeat_penalty;
    std::mt19937 rng(seed);
    std::vector<int32_t> gen;
    for (int s = 0; s < steps; ++s) {
        std::vector<float> l(logits + (size_t) s * n, logits + (size_t) (s + 1) * n);
        const int32_t t = sample_next_token_ex(l, gen, p, rng);
        gen.push_back(t);
        out[s] = t;
    }
}

}  // extern "C"
