// t3b200_dropin.hpp — chatterbox.cpp's T3 internal API served by libt3b200.so.
//
// Same names, argument meaning and error behaviour as
// src/chatterbox_t3_internal.h:120-148 (load_model_gguf, eval_prompt,
// eval_step, sample_next_token_ex), in namespace tts_cpp::chatterbox::b200,
// so the reference's Engine / CLI call sites can switch by namespace under a
// build option.  Functions return false (or token 0) and print the reason
// to stderr on failure, as the reference does; nothing throws.
//
// Differences a caller can see:
//   * the ggml_gallocr_t and n_threads arguments are accepted and ignored
//     (the device owns its buffers);
//   * sample_next_token_ex runs on the device of the last model loaded and
//     keeps the caller's std::mt19937 in lockstep with the device copy, so a
//     sequence of calls draws the same tokens as the reference's sampler.
#pragma once

#include <cstdint>
#include <random>
#include <string>
#include <vector>

#include "t3b200.h"

namespace tts_cpp::chatterbox::b200 {

struct chatterbox_hparams {   // chatterbox_t3_internal.h:44-56
    int32_t n_text_vocab       = 0;
    int32_t n_speech_vocab     = 0;
    int32_t start_speech_token = 0;
    int32_t stop_speech_token  = 0;
    int32_t n_ctx              = 0;
    int32_t n_embd             = 0;
    int32_t n_head             = 0;
    int32_t n_layer            = 0;
    int32_t speaker_embed_size = 0;
    int32_t cond_prompt_len    = 0;
    float   eps                = 1e-5f;
};

struct chatterbox_sampling_params {   // chatterbox_t3_internal.h:113-118
    int32_t top_k          = 1000;
    float   top_p          = 0.95f;
    float   temp           = 0.8f;
    float   repeat_penalty = 1.2f;
};

struct chatterbox_model {
    chatterbox_hparams hparams;
    t3b_ctx *          ctx = nullptr;
    std::vector<std::string> tok_tokens;
    std::vector<std::string> tok_merges;
    void *             mapping = nullptr;   // mmap of the GGUF (released by free_model)
    size_t             mapping_size = 0;
};

bool load_model_gguf(const std::string & path, chatterbox_model & model, int requested_ctx, int n_gpu_layers);

bool eval_prompt(const chatterbox_model & model, void * allocr, int n_threads,
                 const std::vector<int32_t> & text_tokens, std::vector<float> & logits_out, int & prompt_len);

bool eval_step(const chatterbox_model & model, void * allocr, int n_threads, int n_past, int32_t token,
               std::vector<float> & logits_out);

int32_t sample_next_token_ex(const std::vector<float> & logits, const std::vector<int32_t> & generated,
                             const chatterbox_sampling_params & params, std::mt19937 & rng);

void free_model(chatterbox_model & model);

}  // namespace tts_cpp::chatterbox::b200
