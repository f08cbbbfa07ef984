// t3_dropin_main.cpp — the T3 half of chatterbox.cpp's Engine::Impl::run_t3
// (src/chatterbox_engine.cpp:304-359), written against the drop-in API in
// include/t3b200_dropin.hpp instead of the ggml one.  Prints the generated
// speech tokens (stop token popped, as run_t3 does) on one line.
//
//   t3_dropin_main MODEL.gguf SEED N_PREDICT N_TEXT TEXT_ID...
#include <cstdio>
#include <cstdlib>
#include <random>
#include <vector>

#include "t3b200_dropin.hpp"

using namespace tts_cpp::chatterbox::b200;

int main(int argc, char ** argv) {
    if (argc < 5) { fprintf(stderr, "usage: %s model.gguf seed n_predict n_text ids...\n", argv[0]); return 2; }
    const unsigned seed = (unsigned) strtoul(argv[2], nullptr, 10);
    const int n_predict = atoi(argv[3]), n_text = atoi(argv[4]);
    if (argc < 5 + n_text) return 2;
    std::vector<int32_t> text_tokens;
    for (int i = 0; i < n_text; ++i) text_tokens.push_back((int32_t) atoi(argv[5 + i]));

    chatterbox_model model;
    if (!load_model_gguf(argv[1], model, 512, 99)) return 1;

    chatterbox_sampling_params sp;   // reference defaults: 1000 / 0.95 / 0.8 / 1.2
    std::mt19937 rng(seed);
    std::vector<float> logits;
    int prompt_len = 0;
    if (!eval_prompt(model, nullptr, 1, text_tokens, logits, prompt_len)) return 1;
    int n_past = prompt_len;
    std::vector<int32_t> generated;
    int32_t current = sample_next_token_ex(logits, generated, sp, rng);
    generated.push_back(current);
    for (int i = 0; i < n_predict; ++i) {
        if (current == model.hparams.stop_speech_token) break;
        if (n_past + 1 > model.hparams.n_ctx) break;
        if (!eval_step(model, nullptr, 1, n_past, current, logits)) return 1;
        ++n_past;
        current = sample_next_token_ex(logits, generated, sp, rng);
        generated.push_back(current);
    }
    if (!generated.empty() && generated.back() == model.hparams.stop_speech_token) generated.pop_back();
    printf("prompt_len %d tokens", prompt_len);
    for (int32_t t : generated) printf(" %d", t);
    printf("\n");
    free_model(model);
    return 0;
}
