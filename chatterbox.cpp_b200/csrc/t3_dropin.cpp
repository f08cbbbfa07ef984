// t3_dropin.cpp — chatterbox.cpp's T3 internal API over the C ABI of
// libt3b200.so (include/t3b200_dropin.hpp).  Host code only: it parses the
// GGUF file (a minimal reader of the GGUF v2/v3 container), hands the tensors
// to t3b_create, and forwards eval_prompt / eval_step / sample_next_token_ex.
#include "t3b200_dropin.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <sstream>
#include <stdexcept>

namespace tts_cpp::chatterbox::b200 {

namespace {

// ---------------------------------------------------------------- GGUF ----
// Container layout (GGUF v2/v3): magic "GGUF", u32 version, u64 n_tensors,
// u64 n_kv, then n_kv (key, type, value) records, n_tensors tensor infos
// (name, n_dims, ne[n_dims], ggml type, offset), then the data section at
// the next multiple of general.alignment (default 32).
enum { G_U8 = 0, G_I8, G_U16, G_I16, G_U32, G_I32, G_F32, G_BOOL, G_STR, G_ARR, G_U64, G_I64, G_F64 };

struct Reader {
    const uint8_t * p;
    const uint8_t * end;
    template <class T> T get() {
        if (p + sizeof(T) > end) throw std::runtime_error("truncated GGUF");
        T v; std::memcpy(&v, p, sizeof(T)); p += sizeof(T); return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (p + n > end) throw std::runtime_error("truncated GGUF string");
        std::string s((const char *) p, (size_t) n); p += n; return s;
    }
    void skip_value(uint32_t t) {
        static const int sz[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        if (t == G_STR) { str(); return; }
        if (t == G_ARR) {
            const uint32_t et = get<uint32_t>();
            const uint64_t n = get<uint64_t>();
            for (uint64_t i = 0; i < n; ++i) skip_value(et);
            return;
        }
        if (t > G_F64) throw std::runtime_error("bad GGUF value type");
        p += sz[t];
    }
};

struct KV { uint32_t type; const uint8_t * at; };
struct TInfo { std::string name; uint32_t n_dims; int64_t ne[4]; uint32_t type; uint64_t offset; };

size_t type_row_bytes(uint32_t type, int64_t ne0) {
    switch (type) {
        case 0: return (size_t) ne0 * 4;          // F32
        case 1: return (size_t) ne0 * 2;          // F16
        case 2: return (size_t) ne0 / 32 * 18;    // Q4_0
        case 8: return (size_t) ne0 / 32 * 34;    // Q8_0
        case 26: return (size_t) ne0 * 4;         // I32
    }
    return 0;
}

t3b_ctx * g_last_ctx = nullptr;   // device of the last loaded model (sampler)

}  // namespace

bool load_model_gguf(const std::string & path, chatterbox_model & model, int requested_ctx, int n_gpu_layers) {
    (void) n_gpu_layers;   // the whole model always runs on the GPU
    const int fd = open(path.c_str(), O_RDONLY);
    if (fd < 0) { fprintf(stderr, "%s: failed to open '%s'\n", __func__, path.c_str()); return false; }
    struct stat st;
    if (fstat(fd, &st) != 0) { close(fd); fprintf(stderr, "%s: cannot stat '%s'\n", __func__, path.c_str()); return false; }
    void * map = mmap(nullptr, (size_t) st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (map == MAP_FAILED) { fprintf(stderr, "%s: mmap failed for '%s'\n", __func__, path.c_str()); return false; }
    model.mapping = map;
    model.mapping_size = (size_t) st.st_size;
    try {
        Reader r{(const uint8_t *) map, (const uint8_t *) map + st.st_size};
        if (r.get<uint32_t>() != 0x46554747u) throw std::runtime_error("not a GGUF file");
        const uint32_t version = r.get<uint32_t>();
        if (version < 2) throw std::runtime_error("GGUF v1 is not supported");
        const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
        std::map<std::string, KV> kv;
        for (uint64_t i = 0; i < n_kv; ++i) {
            std::string key = r.str();
            const uint32_t t = r.get<uint32_t>();
            kv[key] = KV{t, r.p};
            r.skip_value(t);
        }
        auto u32 = [&](const char * key) -> uint32_t {   // require_key (main.cpp:269-273)
            auto it = kv.find(key);
            if (it == kv.end()) throw std::runtime_error(std::string("missing GGUF key: ") + key);
            uint32_t v; std::memcpy(&v, it->second.at, 4); return v;
        };
        auto& hp = model.hparams;
        hp.n_text_vocab = (int32_t) u32("chatterbox.text_vocab_size");
        hp.n_speech_vocab = (int32_t) u32("chatterbox.speech_vocab_size");
        hp.start_speech_token = (int32_t) u32("chatterbox.start_speech_token");
        hp.stop_speech_token = (int32_t) u32("chatterbox.stop_speech_token");
        hp.speaker_embed_size = (int32_t) u32("chatterbox.speaker_embed_size");
        hp.cond_prompt_len = (int32_t) u32("chatterbox.cond_prompt_length");
        { const uint32_t b = u32("chatterbox.layer_norm_eps"); std::memcpy(&hp.eps, &b, 4); }
        hp.n_ctx = (int32_t) u32("chatterbox.n_ctx");
        hp.n_embd = (int32_t) u32("chatterbox.n_embd");
        hp.n_head = (int32_t) u32("chatterbox.n_head");
        hp.n_layer = (int32_t) u32("chatterbox.n_layer");
        const int32_t model_ctx = hp.n_ctx;
        if (requested_ctx > 0) hp.n_ctx = std::min(hp.n_ctx, requested_ctx);
        uint32_t align = 32;
        if (kv.count("general.alignment")) align = u32("general.alignment");
        // embedded tokenizer arrays (main.cpp:433-454)
        auto strings = [&](const char * key, std::vector<std::string> & out) {
            auto it = kv.find(key);
            if (it == kv.end() || it->second.type != G_ARR) return false;
            Reader a{it->second.at, r.end};
            if (a.get<uint32_t>() != G_STR) return false;
            const uint64_t n = a.get<uint64_t>();
            out.reserve(n);
            for (uint64_t i = 0; i < n; ++i) out.push_back(a.str());
            return true;
        };
        if (!(strings("tokenizer.ggml.tokens", model.tok_tokens) && strings("tokenizer.ggml.merges", model.tok_merges)))
            fprintf(stderr, "%s: no embedded tokenizer; --tokenizer-dir will be required for --text\n", __func__);
        std::vector<TInfo> infos((size_t) n_tensors);
        for (auto & ti : infos) {
            ti.name = r.str();
            ti.n_dims = r.get<uint32_t>();
            if (ti.n_dims > 4) throw std::runtime_error("tensor with more than 4 dims");
            for (int d = 0; d < 4; ++d) ti.ne[d] = d < (int) ti.n_dims ? (int64_t) r.get<uint64_t>() : 1;
            ti.type = r.get<uint32_t>();
            ti.offset = r.get<uint64_t>();
        }
        const size_t hdr = (size_t) (r.p - (const uint8_t *) map);
        const size_t data = (hdr + align - 1) / align * align;
        std::vector<t3b_tensor> desc;
        desc.reserve(infos.size());
        for (const auto & ti : infos) {
            size_t bytes = type_row_bytes(ti.type, ti.ne[0]);
            for (int d = 1; d < 4; ++d) bytes *= (size_t) ti.ne[d];
            if (data + ti.offset + bytes > model.mapping_size) throw std::runtime_error("tensor data past end: " + ti.name);
            t3b_tensor t{};
            t.name = ti.name.c_str();
            t.type = (int32_t) ti.type;
            t.n_dims = (int32_t) ti.n_dims;
            for (int d = 0; d < 4; ++d) t.ne[d] = ti.ne[d];
            t.data = (const uint8_t *) map + data + ti.offset;
            desc.push_back(t);
        }
        t3b_model_desc md{};
        md.hp = {hp.n_text_vocab, hp.n_speech_vocab, hp.start_speech_token, hp.stop_speech_token, model_ctx,
                 hp.n_embd, hp.n_head, hp.n_layer, hp.speaker_embed_size, hp.cond_prompt_len, hp.eps};
        md.n_tensors = (int32_t) desc.size();
        md.tensors = desc.data();
        model.ctx = t3b_create(0, &md);
        if (!model.ctx) throw std::runtime_error(t3b_last_error(nullptr));
        // one utterance at a time, as the reference's single KV cache
        if (t3b_stream_alloc(model.ctx, 1, hp.n_ctx, 0) != T3B_OK) throw std::runtime_error(t3b_last_error(model.ctx));
        g_last_ctx = model.ctx;
    } catch (const std::exception & e) {
        fprintf(stderr, "%s: %s\n", __func__, e.what());
        free_model(model);
        return false;
    }
    return true;
}

bool eval_prompt(const chatterbox_model & model, void * allocr, int n_threads,
                 const std::vector<int32_t> & text_tokens, std::vector<float> & logits_out, int & prompt_len) {
    (void) allocr; (void) n_threads;
    prompt_len = 1 + model.hparams.cond_prompt_len + (int) text_tokens.size() + 1;
    if (prompt_len > model.hparams.n_ctx) {
        fprintf(stderr, "%s: prompt %d exceeds context %d\n", __func__, prompt_len, model.hparams.n_ctx);
        return false;
    }
    logits_out.resize(model.hparams.n_speech_vocab);
    int32_t P = 0;
    if (t3b_prefill(model.ctx, 0, text_tokens.data(), (int) text_tokens.size(), nullptr, 0, nullptr,
                    logits_out.data(), &P) != T3B_OK) {
        fprintf(stderr, "%s: %s\n", __func__, t3b_last_error(model.ctx));
        return false;
    }
    return true;
}

bool eval_step(const chatterbox_model & model, void * allocr, int n_threads, int n_past, int32_t token,
               std::vector<float> & logits_out) {
    (void) allocr; (void) n_threads;
    logits_out.resize(model.hparams.n_speech_vocab);
    const int32_t np = n_past;
    if (t3b_step(model.ctx, 1, nullptr, &token, &np, logits_out.data()) != T3B_OK) {
        fprintf(stderr, "%s: %s\n", __func__, t3b_last_error(model.ctx));
        return false;
    }
    return true;
}

int32_t sample_next_token_ex(const std::vector<float> & logits, const std::vector<int32_t> & generated,
                             const chatterbox_sampling_params & params, std::mt19937 & rng) {
    t3b_ctx * ctx = g_last_ctx;
    if (!ctx) { fprintf(stderr, "%s: no model loaded\n", __func__); return 0; }
    // the device engine takes the caller's std::mt19937 state (its stream
    // format: 624 words then the index) and hands it back after the draw
    std::vector<uint32_t> w(625);
    {
        std::stringstream ss;
        ss << rng;
        for (auto & x : w) { unsigned long v = 0; ss >> v; x = (uint32_t) v; }
    }
    if (t3b_set_rng_state(ctx, 0, w.data()) != T3B_OK ||
        t3b_set_history(ctx, 0, generated.empty() ? nullptr : generated.data(), (int) generated.size()) != T3B_OK) {
        fprintf(stderr, "%s: %s\n", __func__, t3b_last_error(ctx));
        return 0;
    }
    t3b_sample_params p{params.top_k, params.top_p, params.temp, params.repeat_penalty, 0.0f, 0.0f};
    int32_t tok = 0;
    if (t3b_sample(ctx, 1, nullptr, &p, logits.data(), &tok) != T3B_OK ||
        t3b_get_rng_state(ctx, 0, w.data()) != T3B_OK) {
        fprintf(stderr, "%s: %s\n", __func__, t3b_last_error(ctx));
        return 0;
    }
    std::stringstream ss;
    for (int i = 0; i < 625; ++i) ss << w[i] << ' ';
    ss >> rng;
    return tok;
}

void free_model(chatterbox_model & model) {
    if (model.ctx) {
        if (g_last_ctx == model.ctx) g_last_ctx = nullptr;
        t3b_destroy(model.ctx);
        model.ctx = nullptr;
    }
    if (model.mapping) { munmap(model.mapping, model.mapping_size); model.mapping = nullptr; }
}

}  // namespace tts_cpp::chatterbox::b200
