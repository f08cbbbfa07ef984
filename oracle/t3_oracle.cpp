// t3_oracle.cpp — CPU restatement of chatterbox.cpp's T3 decode path.
//
// TEST INFRASTRUCTURE ONLY.  This file is the checker that the CUDA path is
// compared against, and the timed CPU baseline in bench.py.  Nothing in the
// product (chatterbox.cpp_b200/) links, loads or calls it.
//
// What it restates (paths relative to the chatterbox.cpp source tree):
//   * src/main.cpp:469-582  build_transformer_core  (LN -> QKV -> KV append ->
//     attention -> proj + residual -> LN -> fc -> GELU -> proj + residual,
//     then ln_f and speech_head)
//   * src/main.cpp:588-637  build_prompt_graph / build_step_graph (input
//     assembly: speaker projection, cond tokens, text tokens, start token,
//     learned positions)
//   * src/main.cpp:643-710  eval_prompt / eval_step (which logits row is
//     returned, causal mask in the prompt pass)
//   * src/main.cpp:726-801  sample_next_token_ex (exact operation order)
//   * libstdc++ 13 bits/random.tcc:2657-2715 (discrete_distribution) and
//     :3349-3381 (generate_canonical) for the multinomial draw.
//   * GGUF block formats as in gguf-py quants.py (Q4_0, Q8_0) and the
//     activation re-quantisation ggml's CPU backend performs before a
//     quantised dot product (ggml vec_dot_type = Q8_0).
//
// ggml itself (pinned 58c38058 by scripts/setup-ggml.sh:16) is not available
// in this build environment, so the ggml arithmetic cannot be executed here:
// the GEMV / norm / GELU / attention semantics below are a restatement of
// ggml's published CPU algorithms and are "parity unpinned".  The sampler is
// pinned: tests compare it with the reference's own sample_next_token_ex
// compiled from its source (oracle/Makefile, target ref).
//
// Numeric modes (orc_model_config):
//   gemv_mode 0 = EXACT  dequantise weights, accumulate in double.
//   gemv_mode 1 = GGML   activations re-quantised to Q8_0 (for Q4_0/Q8_0
//                        weights) or rounded to f16 (for F16 weights), per
//                        32-block integer dot, float block accumulation.
//   gelu_f16   1 = ggml CPU GELU lookup-table semantics (input and output
//                  rounded through f16), 0 = plain f32 tanh approximation.
//   kv_f16     1 = K/V cache entries rounded to f16 (the CUDA path's cache
//                  format), 0 = f32 cache as in src/main.cpp:419-424.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>
#include <immintrin.h>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

enum { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8 };  // ggml type ids

inline float h2f(uint16_t h) { return _cvtsh_ss(h); }
inline uint16_t f2h(float f) { return _cvtss_sh(f, _MM_FROUND_TO_NEAREST_INT); }

size_t row_bytes(int type, int K) {
    switch (type) {
        case T_F32: return (size_t) K * 4;
        case T_F16: return (size_t) K * 2;
        case T_Q4_0: return (size_t) (K / 32) * 18;
        case T_Q8_0: return (size_t) (K / 32) * 34;
    }
    return 0;
}

void dequant_row(int type, const uint8_t * src, int K, float * dst) {
    switch (type) {
        case T_F32: std::memcpy(dst, src, (size_t) K * 4); break;
        case T_F16: {
            const uint16_t * s = (const uint16_t *) src;
            for (int k = 0; k < K; ++k) dst[k] = h2f(s[k]);
        } break;
        case T_Q4_0: {
            for (int b = 0; b < K / 32; ++b) {
                const uint8_t * blk = src + (size_t) b * 18;
                uint16_t dh; std::memcpy(&dh, blk, 2);
                const float d = h2f(dh);
                for (int j = 0; j < 16; ++j) {
                    dst[b * 32 + j]      = (float) ((int) (blk[2 + j] & 0x0F) - 8) * d;
                    dst[b * 32 + j + 16] = (float) ((int) (blk[2 + j] >> 4) - 8) * d;
                }
            }
        } break;
        case T_Q8_0: {
            for (int b = 0; b < K / 32; ++b) {
                const uint8_t * blk = src + (size_t) b * 34;
                uint16_t dh; std::memcpy(&dh, blk, 2);
                const float d = h2f(dh);
                for (int j = 0; j < 32; ++j) dst[b * 32 + j] = (float) (int8_t) blk[2 + j] * d;
            }
        } break;
    }
}

// One activation row re-quantised to Q8_0 blocks (gguf-py quants.py Q8_0
// semantics: d = amax/127, q = round-half-away(x/d), d stored as f16).
struct QRow {
    std::vector<int8_t> q;
    std::vector<float>  d;   // f16-rounded scale, as the dot product sees it
};

void quantize_q8(const float * x, int K, QRow & out) {
    out.q.resize(K);
    out.d.resize(K / 32);
    for (int b = 0; b < K / 32; ++b) {
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) amax = std::max(amax, std::fabs(x[b * 32 + j]));
        const float d  = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        for (int j = 0; j < 32; ++j) out.q[b * 32 + j] = (int8_t) std::roundf(x[b * 32 + j] * id);
        out.d[b] = h2f(f2h(d));
    }
}

float dot_q4_q8(const uint8_t * w, const QRow & xq, int K) {
    float sumf = 0.0f;
    for (int b = 0; b < K / 32; ++b) {
        const uint8_t * blk = w + (size_t) b * 18;
        uint16_t dh; std::memcpy(&dh, blk, 2);
        const int8_t * xqb = xq.q.data() + b * 32;
        int sumi = 0;
        for (int j = 0; j < 16; ++j) {
            sumi += ((int) (blk[2 + j] & 0x0F) - 8) * xqb[j];
            sumi += ((int) (blk[2 + j] >> 4) - 8) * xqb[j + 16];
        }
        sumf += (float) sumi * h2f(dh) * xq.d[b];
    }
    return sumf;
}

float dot_q8_q8(const uint8_t * w, const QRow & xq, int K) {
    float sumf = 0.0f;
    for (int b = 0; b < K / 32; ++b) {
        const uint8_t * blk = w + (size_t) b * 34;
        uint16_t dh; std::memcpy(&dh, blk, 2);
        const int8_t * wq = (const int8_t *) (blk + 2);
        const int8_t * xqb = xq.q.data() + b * 32;
        int sumi = 0;
        for (int j = 0; j < 32; ++j) sumi += (int) wq[j] * xqb[j];
        sumf += (float) sumi * h2f(dh) * xq.d[b];
    }
    return sumf;
}

int g_threads = 1;

// y[m*N + n] = W[n,:] . x[m*K : (m+1)*K] (+ bias[n]).  W rows are K
// contiguous elements of `type` (GGUF layout: ne0 = K, ne1 = N).
void matvec(int type, const void * W, int N, int K, const float * x, int M,
            const float * bias, float * y, int mode) {
    const uint8_t * wb = (const uint8_t *) W;
    const size_t rb = row_bytes(type, K);
    for (int m = 0; m < M; ++m) {
        const float * xm = x + (size_t) m * K;
        float * ym = y + (size_t) m * N;
        if (mode == 1 && (type == T_Q4_0 || type == T_Q8_0)) {
            QRow xq;
            quantize_q8(xm, K, xq);
#pragma omp parallel for schedule(static) num_threads(g_threads)
            for (int n = 0; n < N; ++n) {
                const uint8_t * wr = wb + (size_t) n * rb;
                float v = type == T_Q4_0 ? dot_q4_q8(wr, xq, K) : dot_q8_q8(wr, xq, K);
                ym[n] = bias ? v + bias[n] : v;
            }
        } else if (mode == 1 && type == T_F16) {
            std::vector<float> xh(K);
            for (int k = 0; k < K; ++k) xh[k] = h2f(f2h(xm[k]));
#pragma omp parallel for schedule(static) num_threads(g_threads)
            for (int n = 0; n < N; ++n) {
                const uint16_t * wr = (const uint16_t *) (wb + (size_t) n * rb);
                double acc = 0.0;
                for (int k = 0; k < K; ++k) acc += (double) (h2f(wr[k]) * xh[k]);
                float v = (float) acc;
                ym[n] = bias ? v + bias[n] : v;
            }
        } else {
#pragma omp parallel for schedule(static) num_threads(g_threads)
            for (int n = 0; n < N; ++n) {
                std::vector<float> wrow(K);
                dequant_row(type, wb + (size_t) n * rb, K, wrow.data());
                double acc = 0.0;
                for (int k = 0; k < K; ++k) acc += (double) wrow[k] * (double) xm[k];
                float v = (float) acc;
                ym[n] = bias ? v + bias[n] : v;
            }
        }
    }
}

// ggml_norm followed by ggml_mul(g) and ggml_add(b) (src/main.cpp:503-504).
void layernorm(const float * x, int n, const float * g, const float * b, float eps, float * y) {
    double sum = 0.0;
    for (int i = 0; i < n; ++i) sum += (double) x[i];
    const float mean = (float) (sum / n);
    double sum2 = 0.0;
    for (int i = 0; i < n; ++i) {
        const float v = x[i] - mean;
        y[i] = v;
        sum2 += (double) (v * v);
    }
    const float var = (float) (sum2 / n);
    const float scale = 1.0f / std::sqrt(var + eps);
    for (int i = 0; i < n; ++i) {
        const float t = y[i] * scale;
        const float u = t * g[i];
        y[i] = u + b[i];
    }
}

// ggml GELU, tanh approximation (ggml_gelu).  With f16_table the input and
// output pass through f16 and |x| >= 10 short-cuts, as ggml's CPU lookup
// table does.
float gelu_f32(float x) {
    const float c = 0.79788456080286535587989211986876f;
    const float a = 0.044715f;
    return 0.5f * x * (1.0f + std::tanh(c * x * (1.0f + a * x * x)));
}
float gelu(float x, int f16_table) {
    if (!f16_table) return gelu_f32(x);
    if (x <= -10.0f) return 0.0f;
    if (x >= 10.0f) return x;
    return h2f(f2h(gelu_f32(h2f(f2h(x)))));
}

// ---------------------------------------------------------------------------
// Model
// ---------------------------------------------------------------------------

struct Wt { int type = -1; const void * data = nullptr; };

struct Layer {
    const float * ln1_g = nullptr, * ln1_b = nullptr, * ln2_g = nullptr, * ln2_b = nullptr;
    Wt attn_w, proj_w, fc_w, fc2_w;
    const float * attn_b = nullptr, * proj_b = nullptr, * fc_b = nullptr, * fc2_b = nullptr;
};

struct Model {
    int n_layer, n_embd, n_head, max_ctx, n_vocab, n_text_vocab, spk_size;
    float eps;
    int gemv_mode = 1, gelu_f16 = 1, kv_f16 = 0;
    const float * wpe = nullptr, * lnf_g = nullptr, * lnf_b = nullptr;
    const uint16_t * text_emb = nullptr, * speech_emb = nullptr;
    Wt head; const float * head_b = nullptr;
    const float * spkr_w = nullptr, * spkr_b = nullptr;
    const float * builtin_spk = nullptr; const int32_t * builtin_cond = nullptr; int n_builtin_cond = 0;
    std::vector<Layer> layers;
    std::vector<float> kc, vc;   // [layer][head][pos][hd]
    float * trace = nullptr;     // nullable: [n_layer + 1][n_embd] residual stream of the last row (tests)
    size_t kv_index(int l, int h, int pos) const {
        const int hd = n_embd / n_head;
        return (((size_t) l * n_head + h) * max_ctx + pos) * hd;
    }
};

// Transformer over N rows at positions n_past .. n_past+N-1, causal.  x is
// [N, n_embd] input embeddings; writes logits for the last row (or all rows
// when all_logits) into `logits`.
void forward(Model & m, std::vector<float> & x, int n_past, int N, float * logits, bool all_logits) {
    const int D = m.n_embd, H = m.n_head, HD = D / H;
    const float scale = 1.0f / std::sqrt((float) HD);
    std::vector<float> cur((size_t) N * D), qkv((size_t) N * 3 * D), attn((size_t) N * D);
    std::vector<float> h4((size_t) N * 4 * D), tmp((size_t) N * D);
    for (int il = 0; il < m.n_layer; ++il) {
        const Layer & L = m.layers[il];
        for (int r = 0; r < N; ++r)
            layernorm(&x[(size_t) r * D], D, L.ln1_g, L.ln1_b, m.eps, &cur[(size_t) r * D]);
        matvec(L.attn_w.type, L.attn_w.data, 3 * D, D, cur.data(), N, L.attn_b, qkv.data(), m.gemv_mode);
        // KV append (src/main.cpp:528-546)
        for (int r = 0; r < N; ++r)
            for (int h = 0; h < H; ++h)
                for (int d = 0; d < HD; ++d) {
                    float kk = qkv[(size_t) r * 3 * D + D + h * HD + d];
                    float vv = qkv[(size_t) r * 3 * D + 2 * D + h * HD + d];
                    if (m.kv_f16) { kk = h2f(f2h(kk)); vv = h2f(f2h(vv)); }
                    m.kc[m.kv_index(il, h, n_past + r) + d] = kk;
                    m.vc[m.kv_index(il, h, n_past + r) + d] = vv;
                }
        // attention, causal (src/main.cpp:548-560)
#pragma omp parallel for collapse(2) schedule(static) num_threads(g_threads)
        for (int r = 0; r < N; ++r)
            for (int h = 0; h < H; ++h) {
                const int Lk = n_past + r + 1;
                const float * q = &qkv[(size_t) r * 3 * D + h * HD];
                std::vector<float> s(Lk);
                float mx = -INFINITY;
                for (int j = 0; j < Lk; ++j) {
                    const float * kr = &m.kc[m.kv_index(il, h, j)];
                    double acc = 0.0;
                    for (int d = 0; d < HD; ++d) acc += (double) q[d] * (double) kr[d];
                    s[j] = (float) acc * scale;
                    mx = std::max(mx, s[j]);
                }
                double den = 0.0;
                std::vector<double> o(HD, 0.0);
                for (int j = 0; j < Lk; ++j) {
                    const double w = std::exp((double) s[j] - (double) mx);
                    den += w;
                    const float * vr = &m.vc[m.kv_index(il, h, j)];
                    for (int d = 0; d < HD; ++d) o[d] += w * (double) vr[d];
                }
                for (int d = 0; d < HD; ++d) attn[(size_t) r * D + h * HD + d] = (float) (o[d] / den);
            }
        // proj + bias + residual: (W a + b) + x
        matvec(L.proj_w.type, L.proj_w.data, D, D, attn.data(), N, L.proj_b, tmp.data(), m.gemv_mode);
        for (size_t i = 0; i < (size_t) N * D; ++i) x[i] = tmp[i] + x[i];
        for (int r = 0; r < N; ++r)
            layernorm(&x[(size_t) r * D], D, L.ln2_g, L.ln2_b, m.eps, &cur[(size_t) r * D]);
        matvec(L.fc_w.type, L.fc_w.data, 4 * D, D, cur.data(), N, L.fc_b, h4.data(), m.gemv_mode);
        for (size_t i = 0; i < (size_t) N * 4 * D; ++i) h4[i] = gelu(h4[i], m.gelu_f16);
        matvec(L.fc2_w.type, L.fc2_w.data, D, 4 * D, h4.data(), N, L.fc2_b, tmp.data(), m.gemv_mode);
        for (size_t i = 0; i < (size_t) N * D; ++i) x[i] = tmp[i] + x[i];
        if (m.trace) std::memcpy(m.trace + (size_t) (il + 1) * D, &x[(size_t) (N - 1) * D], sizeof(float) * D);
    }
    const int r0 = all_logits ? 0 : N - 1;
    for (int r = r0; r < N; ++r) {
        layernorm(&x[(size_t) r * D], D, m.lnf_g, m.lnf_b, m.eps, &cur[0]);
        float * out = logits + (size_t) (all_logits ? r : 0) * m.n_vocab;
        matvec(m.head.type, m.head.data, m.n_vocab, D, cur.data(), 1, m.head_b, out, m.gemv_mode);
    }
}

// ---------------------------------------------------------------------------
// Sampler
// ---------------------------------------------------------------------------

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as
// easy as 1, 2, 3", SC'11).  counter = {c0,c1,c2,c3}, key = {k0,k1}.
void philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
    uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int r = 0; r < 10; ++r) {
        const uint64_t p0 = (uint64_t) 0xD2511F53u * c0;
        const uint64_t p1 = (uint64_t) 0xCD9E8D57u * c2;
        const uint32_t n0 = (uint32_t) (p1 >> 32) ^ c1 ^ k0;
        const uint32_t n1 = (uint32_t) p1;
        const uint32_t n2 = (uint32_t) (p0 >> 32) ^ c3 ^ k1;
        const uint32_t n3 = (uint32_t) p0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

// generate_canonical<double, 53> over a 32-bit engine: two draws.
double canonical53(uint32_t x1, uint32_t x2) {
    double sum = (double) x1;
    sum += (double) x2 * 4294967296.0;
    double r = sum / 18446744073709551616.0;
    if (r >= 1.0) r = std::nextafter(1.0, 0.0);
    return r;
}

struct SampleParams {
    int32_t top_k;
    float   top_p;
    float   temp;
    float   repeat_penalty;
    float   min_p;        // extension: 0 = off
    float   cfg_weight;   // extension: 0 = off (uncond ignored)
};

// Returns the token; *aux receives stage statistics for tests:
// aux[0] = survivors after top-k, aux[1] = survivors after top-p,
// aux[2] = 1 when the top-p cut fell inside a group of equal scores
// (where std::sort's tie order is unspecified).
int sample_row(const float * cond, const float * uncond, int n, const int32_t * hist, int n_hist,
               const SampleParams & p, uint32_t x1, uint32_t x2, int32_t * aux) {
    std::vector<float> s(n);
    const bool cfg = uncond != nullptr && p.cfg_weight != 0.0f;
    for (int i = 0; i < n; ++i) {
        if (cfg) {
            const float diff = cond[i] - uncond[i];
            const float scaled = p.cfg_weight * diff;
            s[i] = cond[i] + scaled;
        } else {
            s[i] = cond[i];
        }
    }
    // (1) temperature (main.cpp:735-738)
    if (p.temp > 0.0f && p.temp != 1.0f) {
        const float inv_t = 1.0f / p.temp;
        for (int i = 0; i < n; ++i) s[i] *= inv_t;
    }
    // (1b) min-p extension: drop p_i < min_p * p_max  <=>  exp(s_i - max) < min_p
    if (p.min_p > 0.0f) {
        float mx = -INFINITY;
        for (int i = 0; i < n; ++i) if (s[i] != -INFINITY) mx = std::max(mx, s[i]);
        for (int i = 0; i < n; ++i)
            if (s[i] != -INFINITY && std::exp(s[i] - mx) < p.min_p) s[i] = -INFINITY;
    }
    // (2) top-k (main.cpp:740-748): threshold = value at descending rank k
    if (p.top_k > 0 && p.top_k < n) {
        std::vector<float> desc(s);
        std::sort(desc.begin(), desc.end(), [](float a, float b) { return a > b; });
        float thr = desc[p.top_k];
        int above = 0;
        for (int i = 0; i < n; ++i) if (s[i] > thr) ++above;
        if (above < p.top_k) thr -= 1e-10f;
        for (int i = 0; i < n; ++i) if (s[i] <= thr) s[i] = -INFINITY;
    }
    int surv_k = 0;
    for (int i = 0; i < n; ++i) if (s[i] != -INFINITY) ++surv_k;
    // (3) top-p (main.cpp:750-772): descending order, sequential float sums
    int tie_at_cut = 0;
    if (p.top_p < 1.0f) {
        std::vector<int> ord;
        for (int i = 0; i < n; ++i) if (s[i] != -INFINITY) ord.push_back(i);
        std::stable_sort(ord.begin(), ord.end(), [&](int a, int b) { return s[a] > s[b]; });
        if (!ord.empty()) {
            const float mx = s[ord[0]];
            std::vector<float> e(ord.size());
            float psum = 0.0f;
            for (size_t j = 0; j < ord.size(); ++j) { e[j] = std::exp(s[ord[j]] - mx); psum += e[j]; }
            float cum = 0.0f;
            size_t cut = ord.size();
            for (size_t j = 0; j < ord.size(); ++j) {
                cum += e[j] / psum;
                if (cum >= p.top_p) { cut = j + 1; break; }
            }
            if (cut < ord.size() && s[ord[cut]] == s[ord[cut - 1]]) tie_at_cut = 1;
            for (size_t j = cut; j < ord.size(); ++j) s[ord[j]] = -INFINITY;
        }
    }
    int surv_p = 0;
    for (int i = 0; i < n; ++i) if (s[i] != -INFINITY) ++surv_p;
    // (4) repetition penalty over the distinct history ids (main.cpp:774-781)
    if (p.repeat_penalty != 1.0f && n_hist > 0) {
        std::vector<char> seen(n, 0);
        for (int j = 0; j < n_hist; ++j) {
            const int t = hist[j];
            if (t < 0 || t >= n || seen[t]) continue;
            seen[t] = 1;
            if (s[t] == -INFINITY) continue;
            s[t] = s[t] > 0 ? s[t] / p.repeat_penalty : s[t] * p.repeat_penalty;
        }
    }
    if (aux) { aux[0] = surv_k; aux[1] = surv_p; aux[2] = tie_at_cut; }
    // (5) softmax over survivors, index order (main.cpp:783-793)
    float mx = -INFINITY;
    for (int i = 0; i < n; ++i) if (s[i] != -INFINITY) mx = std::max(mx, s[i]);
    std::vector<float> pr(n);
    float psum = 0.0f;
    for (int i = 0; i < n; ++i) {
        pr[i] = s[i] == -INFINITY ? 0.0f : std::exp(s[i] - mx);
        psum += pr[i];
    }
    if (psum == 0.0f) return 0;
    for (int i = 0; i < n; ++i) pr[i] /= psum;
    // (6) greedy
    if (p.temp <= 0.0f) {
        int best = 0;
        for (int i = 1; i < n; ++i) if (pr[i] > pr[best]) best = i;
        return best;
    }
    // (7) discrete_distribution: double normalisation, cumulative sums,
    // last entry forced to 1, lower_bound of the canonical draw.
    if (n < 2) return 0;
    double dsum = 0.0;
    for (int i = 0; i < n; ++i) dsum += (double) pr[i];
    const double u = canonical53(x1, x2);
    double c = 0.0;
    for (int i = 0; i < n; ++i) {
        c = (i == 0) ? (double) pr[0] / dsum : c + (double) pr[i] / dsum;
        const double ci = (i == n - 1) ? 1.0 : c;
        if (!(ci < u)) return i;
    }
    return n - 1;
}

}  // namespace

// ===========================================================================
// C API (ctypes)
// ===========================================================================
extern "C" {

void orc_set_threads(int n) { g_threads = n > 0 ? n : 1; }

// The host C library's expf over a batch (what std::exp(float) in the
// reference sampler returns), for checking the device exp.
void orc_expf_batch(const float * in, float * out, int64_t n) {
#pragma omp parallel for schedule(static) num_threads(g_threads)
    for (int64_t i = 0; i < n; ++i) out[i] = std::exp(in[i]);
}

float orc_f16_to_f32(uint16_t h) { return h2f(h); }
uint16_t orc_f32_to_f16(float f) { return f2h(f); }

void orc_dequant_rows(int type, const void * src, int n_rows, int K, float * dst) {
    const size_t rb = row_bytes(type, K);
    for (int r = 0; r < n_rows; ++r)
        dequant_row(type, (const uint8_t *) src + rb * r, K, dst + (size_t) r * K);
}

void orc_quantize_q8_row(const float * x, int K, int8_t * q, float * d) {
    QRow r; quantize_q8(x, K, r);
    std::memcpy(q, r.q.data(), (size_t) K);
    std::memcpy(d, r.d.data(), sizeof(float) * (K / 32));
}

void orc_matvec(int type, const void * W, int N, int K, const float * x, int M,
                const float * bias, float * y, int mode) {
    matvec(type, W, N, K, x, M, bias, y, mode);
}

void orc_layernorm(const float * x, int n, const float * g, const float * b, float eps, float * y) {
    layernorm(x, n, g, b, eps, y);
}

float orc_gelu(float x, int f16_table) { return gelu(x, f16_table); }

void orc_philox4x32_10(const uint32_t * ctr, const uint32_t * key, uint32_t * out) {
    philox4x32_10(ctr, key, out);
}

double orc_canonical53(uint32_t x1, uint32_t x2) { return canonical53(x1, x2); }

// n words from std::mt19937(seed) after discarding `skip` outputs.
void orc_mt19937_words(uint32_t seed, uint64_t skip, int n, uint32_t * out) {
    std::mt19937 g(seed);
    g.discard(skip);
    for (int i = 0; i < n; ++i) out[i] = (uint32_t) g();
}

int orc_sample(const float * cond, const float * uncond, int n, const int32_t * hist, int n_hist,
               int32_t top_k, float top_p, float temp, float repeat_penalty, float min_p,
               float cfg_weight, uint32_t x1, uint32_t x2, int32_t * aux) {
    SampleParams p{top_k, top_p, temp, repeat_penalty, min_p, cfg_weight};
    return sample_row(cond, uncond, n, hist, n_hist, p, x1, x2, aux);
}

void * orc_model_new(int n_layer, int n_embd, int n_head, int max_ctx, int n_vocab,
                     int n_text_vocab, int spk_size, float eps) {
    Model * m = new Model();
    m->n_layer = n_layer; m->n_embd = n_embd; m->n_head = n_head; m->max_ctx = max_ctx;
    m->n_vocab = n_vocab; m->n_text_vocab = n_text_vocab; m->spk_size = spk_size; m->eps = eps;
    m->layers.resize(n_layer);
    m->kc.assign((size_t) n_layer * n_embd * max_ctx, 0.0f);
    m->vc.assign((size_t) n_layer * n_embd * max_ctx, 0.0f);
    return m;
}

void orc_model_free(void * h) { delete (Model *) h; }

void orc_model_config(void * h, int gemv_mode, int gelu_f16, int kv_f16) {
    Model * m = (Model *) h;
    m->gemv_mode = gemv_mode; m->gelu_f16 = gelu_f16; m->kv_f16 = kv_f16;
}

// Bind a GGUF tensor by its name (convert-t3-turbo-to-gguf.py naming).
int orc_model_set(void * h, const char * name, int type, const void * data, int64_t n_elems) {
    Model * m = (Model *) h;
    std::string s(name);
    auto F = [&](const float *& dst) { if (type != T_F32) return -2; dst = (const float *) data; return 0; };
    if (s == "model/wpe") return F(m->wpe);
    if (s == "model/ln_f/g") return F(m->lnf_g);
    if (s == "model/ln_f/b") return F(m->lnf_b);
    if (s == "chatterbox/text_emb") { if (type != T_F16) return -2; m->text_emb = (const uint16_t *) data; return 0; }
    if (s == "chatterbox/speech_emb") { if (type != T_F16) return -2; m->speech_emb = (const uint16_t *) data; return 0; }
    if (s == "chatterbox/speech_head") { m->head = {type, data}; return 0; }
    if (s == "chatterbox/speech_head_bias") return F(m->head_b);
    if (s == "chatterbox/cond_spkr/w") return F(m->spkr_w);
    if (s == "chatterbox/cond_spkr/b") return F(m->spkr_b);
    if (s == "chatterbox/builtin/speaker_emb") return F(m->builtin_spk);
    if (s == "chatterbox/builtin/cond_prompt_speech_tokens") {
        m->builtin_cond = (const int32_t *) data; m->n_builtin_cond = (int) n_elems; return 0;
    }
    int il = -1; char rest[128] = {0};
    if (std::sscanf(name, "model/h%d/%127s", &il, rest) == 2 && il >= 0 && il < m->n_layer) {
        Layer & L = m->layers[il];
        std::string r(rest);
        if (r == "ln_1/g") return F(L.ln1_g);
        if (r == "ln_1/b") return F(L.ln1_b);
        if (r == "ln_2/g") return F(L.ln2_g);
        if (r == "ln_2/b") return F(L.ln2_b);
        if (r == "attn/c_attn/w") { L.attn_w = {type, data}; return 0; }
        if (r == "attn/c_attn/b") return F(L.attn_b);
        if (r == "attn/c_proj/w") { L.proj_w = {type, data}; return 0; }
        if (r == "attn/c_proj/b") return F(L.proj_b);
        if (r == "mlp/c_fc/w") { L.fc_w = {type, data}; return 0; }
        if (r == "mlp/c_fc/b") return F(L.fc_b);
        if (r == "mlp/c_proj/w") { L.fc2_w = {type, data}; return 0; }
        if (r == "mlp/c_proj/b") return F(L.fc2_b);
    }
    return -1;  // unknown tensor: ignored by the caller
}

// Prompt pass (src/main.cpp:588-616, 643-689).  Rows: speaker projection,
// cond speech tokens, text tokens (zeroed when uncond != 0: the CFG
// unconditional row), start token; plus learned positions.  cond/spk may be
// null to use the GGUF's builtin voice.  Returns prompt_len, or -1.
int orc_prompt(void * h, const int32_t * text, int n_text, const int32_t * cond, int n_cond,
               const float * spk, int start_tok, int uncond, float * logits_out) {
    Model * m = (Model *) h;
    if (!cond) { cond = m->builtin_cond; n_cond = m->n_builtin_cond; }
    if (!spk) spk = m->builtin_spk;
    const int D = m->n_embd;
    const int P = 1 + n_cond + n_text + 1;
    if (P > m->max_ctx) return -1;
    std::vector<float> x((size_t) P * D);
    // speaker row: cond_spkr_w [K=spk, N=D] f32 . spk + b
    matvec(T_F32, m->spkr_w, D, m->spk_size, spk, 1, m->spkr_b, &x[0], 0);
    for (int i = 0; i < n_cond; ++i)
        for (int d = 0; d < D; ++d) x[(size_t) (1 + i) * D + d] = h2f(m->speech_emb[(size_t) cond[i] * D + d]);
    for (int i = 0; i < n_text; ++i)
        for (int d = 0; d < D; ++d)
            x[(size_t) (1 + n_cond + i) * D + d] = uncond ? 0.0f : h2f(m->text_emb[(size_t) text[i] * D + d]);
    for (int d = 0; d < D; ++d) x[(size_t) (P - 1) * D + d] = h2f(m->speech_emb[(size_t) start_tok * D + d]);
    for (int r = 0; r < P; ++r)
        for (int d = 0; d < D; ++d) x[(size_t) r * D + d] = x[(size_t) r * D + d] + m->wpe[(size_t) r * D + d];
    forward(*m, x, 0, P, logits_out, false);
    return P;
}

// One decode step (src/main.cpp:618-637, 691-710).
int orc_step(void * h, int n_past, int32_t token, float * logits_out) {
    Model * m = (Model *) h;
    if (n_past + 1 > m->max_ctx || token < 0 || token >= m->n_vocab) return -1;
    const int D = m->n_embd;
    std::vector<float> x(D);
    for (int d = 0; d < D; ++d)
        x[d] = h2f(m->speech_emb[(size_t) token * D + d]) + m->wpe[(size_t) n_past * D + d];
    forward(*m, x, n_past, 1, logits_out, false);
    return 0;
}

// orc_step that also records the residual stream: hidden_out[0] = the
// step embedding, hidden_out[l + 1] = layer l's output ([n_layer + 1][n_embd]).
int orc_step_trace(void * h, int n_past, int32_t token, float * logits_out, float * hidden_out) {
    Model * m = (Model *) h;
    if (n_past + 1 > m->max_ctx || token < 0 || token >= m->n_vocab) return -1;
    const int D = m->n_embd;
    for (int d = 0; d < D; ++d)
        hidden_out[d] = h2f(m->speech_emb[(size_t) token * D + d]) + m->wpe[(size_t) n_past * D + d];
    m->trace = hidden_out;
    const int rc = orc_step(h, n_past, token, logits_out);
    m->trace = nullptr;
    return rc;
}

// Copy of one layer's K or V cache rows [n_head][0..n_pos)[hd] for tests.
void orc_model_kv(void * h, int layer, int which, int n_pos, float * out) {
    Model * m = (Model *) h;
    const int HD = m->n_embd / m->n_head;
    for (int hh = 0; hh < m->n_head; ++hh)
        for (int p = 0; p < n_pos; ++p)
            std::memcpy(out + ((size_t) hh * n_pos + p) * HD,
                        (which ? m->vc : m->kc).data() + m->kv_index(layer, hh, p), sizeof(float) * HD);
}

}  // extern "C"
