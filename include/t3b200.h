/*
 * t3b200.h — C ABI of the B200-native T3 decode path (libt3b200.so).
 *
 * This library replaces the compute behind chatterbox.cpp's T3 internal API
 * (src/chatterbox_t3_internal.h:120-148 in the chatterbox.cpp tree):
 *
 *   load_model_gguf       -> t3b_create        (weights handed over as GGUF
 *                                                tensor views; the caller keeps
 *                                                parsing GGUF)
 *   (KV allocation, main.cpp:419-424)
 *                         -> t3b_stream_alloc  (per-stream f16 caches)
 *   eval_prompt           -> t3b_prefill
 *   eval_step             -> t3b_step
 *   sample_next_token_ex  -> t3b_sample (+ t3b_set_rng / t3b_set_rng_state /
 *                                        t3b_set_history)
 *   decode loop of Engine::Impl::run_t3 (chatterbox_engine.cpp:334-358)
 *                         -> t3b_decode        (whole loop on the device)
 *
 * Conventions: plain C types only; every entry point returns T3B_OK (0) or a
 * negative T3B_ERR_* code and records a message readable with
 * t3b_last_error().  No exceptions cross the ABI.  A context is bound to one
 * CUDA device and is not thread-safe (as chatterbox_model, engine.h:28-30);
 * t3b_cancel() alone may be called from any thread.
 *
 * Kernel-level entry points (t3b_op_*) take DEVICE pointers and a CUDA
 * stream (cudaStream_t passed as void*); they are the ggml ops the T3 graph
 * uses (ggml_mul_mat + bias/GELU/residual epilogues, ggml_flash_attn_ext,
 * the host sampler) exposed for tests and micro-benchmarks.
 */
#ifndef T3B200_H
#define T3B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define T3B_OK             0
#define T3B_ERR_ARG       -1   /* bad argument / shape / missing tensor      */
#define T3B_ERR_CUDA      -2   /* CUDA runtime error                          */
#define T3B_ERR_OOM       -3   /* device allocation failed                    */
#define T3B_ERR_STATE     -4   /* call out of order (e.g. no streams)         */
#define T3B_ERR_DEVICE    -5   /* device-side check failed (error word set)   */
#define T3B_ERR_CANCELLED -6   /* t3b_cancel() observed                       */
#define T3B_ERR_TIMEOUT   -7   /* a bounded device-side wait ran out          */

/* ggml type ids of the tensors the T3 GGUF holds */
enum t3b_dtype { T3B_F32 = 0, T3B_F16 = 1, T3B_Q4_0 = 2, T3B_Q8_0 = 8 };

/* One GGUF tensor view: name as written by convert-t3-turbo-to-gguf.py
 * (map_tensor_name, :147-194), ggml type, ggml shape (ne[0] contiguous),
 * host pointer to the raw GGUF bytes. */
typedef struct t3b_tensor {
    const char * name;
    int32_t      type;
    int32_t      n_dims;
    int64_t      ne[4];
    const void * data;
} t3b_tensor;

/* Mirrors chatterbox_hparams (chatterbox_t3_internal.h:44-56). */
typedef struct t3b_hparams {
    int32_t n_text_vocab;
    int32_t n_speech_vocab;
    int32_t start_speech_token;
    int32_t stop_speech_token;
    int32_t n_ctx;
    int32_t n_embd;
    int32_t n_head;
    int32_t n_layer;
    int32_t speaker_embed_size;
    int32_t cond_prompt_len;
    float   eps;
} t3b_hparams;

typedef struct t3b_model_desc {
    t3b_hparams        hp;
    int32_t            n_tensors;
    const t3b_tensor * tensors;
} t3b_model_desc;

/* chatterbox_sampling_params (chatterbox_t3_internal.h:113-118) plus two
 * extensions that are off at 0: min_p and cfg_weight.  With both 0 the
 * sampler is the reference's sample_next_token_ex (main.cpp:726-801). */
typedef struct t3b_sample_params {
    int32_t top_k;
    float   top_p;
    float   temp;
    float   repeat_penalty;
    float   min_p;
    float   cfg_weight;
} t3b_sample_params;

/* RNG modes.  MT19937: the device mirrors std::mt19937 and libstdc++'s
 * generate_canonical<double,53> + discrete_distribution, so a stream seeded
 * like the reference draws the same tokens.  PHILOX: Philox4x32-10 with
 * key = seed and counter = (draw index, stream), no state to carry. */
enum t3b_rng_mode { T3B_RNG_MT19937 = 0, T3B_RNG_PHILOX = 1 };

typedef struct t3b_ctx t3b_ctx;

/* load_model_gguf (main.cpp:348-463): uploads and repacks every tensor of
 * the T3 GGUF onto `device`.  Returns NULL on failure; the reason is then
 * available from t3b_last_error(NULL). */
t3b_ctx *    t3b_create(int device, const t3b_model_desc * desc);
void         t3b_destroy(t3b_ctx * ctx);
const char * t3b_last_error(const t3b_ctx * ctx);

/* Allocates per-stream f16 KV caches (replaces memory_k/memory_v,
 * main.cpp:419-424).  cfg != 0 gives every stream two rows (cond, uncond).
 * Replaces any previous allocation. */
int t3b_stream_alloc(t3b_ctx * ctx, int n_streams, int max_ctx, int cfg);

/* eval_prompt (main.cpp:643-689) for one stream: rows = [speaker
 * projection; cond speech tokens; text tokens; start token] + positions.
 * cond_tokens/spk_emb NULL = the GGUF's builtin voice.  For a CFG stream the
 * uncond row repeats the prompt with the text embeddings zeroed.
 * logits_out (host, nullable) receives [rows][n_speech_vocab] of the last
 * prompt position.  *prompt_len (nullable) = 1 + n_cond + n_text + 1. */
int t3b_prefill(t3b_ctx * ctx, int stream, const int32_t * text, int n_text,
                const int32_t * cond_tokens, int n_cond, const float * spk_emb,
                float * logits_out, int32_t * prompt_len);

/* eval_step (main.cpp:691-710) for n streams at once.  tokens[i] is fed to
 * stream streams[i] at position n_past[i] (NULL = the stream's own
 * position counter).  logits_out (host, nullable) receives
 * [n][rows_per_stream][n_speech_vocab]; the logits also stay on the device
 * for t3b_sample. */
int t3b_step(t3b_ctx * ctx, int n, const int32_t * streams, const int32_t * tokens,
             const int32_t * n_past, float * logits_out);

/* sample_next_token_ex (main.cpp:726-801) for n streams, on the device.
 * logits (host, nullable): [n][rows_per_stream][V]; NULL = use the logits the
 * last t3b_step/t3b_prefill left on the device for these streams.  The
 * sampled token is appended to each stream's history (the reference's
 * `generated`).  tokens_out: host. */
int t3b_sample(t3b_ctx * ctx, int n, const int32_t * streams, const t3b_sample_params * params,
               const float * logits, int32_t * tokens_out);

int t3b_set_rng(t3b_ctx * ctx, int stream, int mode, uint64_t seed, uint64_t discard);
/* std::mt19937 state as its stream operator prints it: 624 words + index. */
int t3b_set_rng_state(t3b_ctx * ctx, int stream, const uint32_t * words625);
int t3b_get_rng_state(t3b_ctx * ctx, int stream, uint32_t * words625);
/* Replaces a stream's token history (the `generated` vector). */
int t3b_set_history(t3b_ctx * ctx, int stream, const int32_t * tokens, int n);

/* The decode loop of Engine::Impl::run_t3 (chatterbox_engine.cpp:334-358)
 * run on the device for n streams after t3b_prefill: sample from the
 * prefill logits, then up to max_steps x (step, sample), stopping a stream at
 * stop_speech_token or n_ctx.  tokens_out: host [n][max_steps + 1];
 * n_out[i] = tokens written for stream i (stop token included, as the
 * reference's loop leaves it before its pop_back).  ignore_stop != 0 keeps
 * decoding past the stop token (benchmarks). */
int t3b_decode(t3b_ctx * ctx, int n, const int32_t * streams, const t3b_sample_params * params,
               int max_steps, int ignore_stop, int32_t * tokens_out, int32_t * n_out);

/* ---------------- continuous batching (many utterances in flight) -------
 * Replaces the one-utterance-at-a-time loops of chatterbox.cpp's callers
 * (Engine::Impl::run_t3, chatterbox_engine.cpp:330-358; the CLI's segment
 * loop, chatterbox_cli.cpp:1597-1683) for serving: requests queue, each is
 * admitted into a free stream slot of this context (t3b_stream_alloc sets
 * the slot count, context length and CFG), every t3b_serve_run iteration
 * steps all admitted streams as one batch, and a stream that ends (stop
 * token, n_predict steps or a full cache) frees its slot for the next
 * request at once.  Per request the loop is run_t3's; a trailing stop token
 * is popped.  Early-stop retry as the CLI's (chatterbox_cli.cpp:1615-1674):
 * a stop-token ending shorter than min_tokens replays the request (at most
 * max_retries times) with its RNG advanced by attempt * 1009 draws, keeping
 * the longest attempt if all are short (min_tokens 0 = off). */
typedef struct t3b_request {
    const int32_t * text;           /* text token ids (copied at submit) */
    int32_t         n_text;
    const int32_t * cond_tokens;    /* NULL: the GGUF's builtin voice */
    int32_t         n_cond;
    const float *   spk_emb;        /* NULL: builtin speaker embedding */
    t3b_sample_params params;
    int32_t         rng_mode;       /* T3B_RNG_MT19937 (std::mt19937(seed)) or T3B_RNG_PHILOX */
    uint64_t        seed;
    int32_t         n_predict;      /* decode steps after the first token (Engine n_predict) */
    int32_t         min_tokens;     /* the CLI uses max(8, 5 * n_text) */
    int32_t         max_retries;    /* the CLI uses 3 */
} t3b_request;

/* Queues a request; returns its id (>= 0) or a T3B_ERR_* code. */
int t3b_serve_submit(t3b_ctx * ctx, const t3b_request * req);
/* Runs up to max_iters iterations (admit into free slots, one batched
 * step + sample of every admitted stream, retire ended streams); returns
 * early when nothing is admitted or queued.  *n_active / *n_queued
 * (nullable) = streams in slots / requests waiting afterwards.
 * t3b_last_device_ms() = device time of the iterations' batched steps. */
int t3b_serve_run(t3b_ctx * ctx, int max_iters, int32_t * n_active, int32_t * n_queued);
/* 1 when request `id` has finished (min(n, cap) tokens copied to host
 * tokens_out, *n_out = n), 0 while it is pending; *attempts (nullable) =
 * attempts made so far.  A request refused at admission (e.g. a prompt
 * longer than the context) finishes with that error code. */
int t3b_serve_result(t3b_ctx * ctx, int id, int32_t * tokens_out, int cap, int32_t * n_out, int32_t * attempts);

/* Tokens sampled by t3b_serve_run's batched steps since t3b_stream_alloc,
 * and the device time of those steps (ms). */
int t3b_serve_stats(const t3b_ctx * ctx, long long * step_tokens, double * step_ms);

/* Engine::cancel() equivalent (chatterbox_engine.cpp:546-548). */
void t3b_cancel(t3b_ctx * ctx);

/* Device time of the last t3b_decode / t3b_step call, in milliseconds. */
float t3b_last_device_ms(const t3b_ctx * ctx);

/* Logits tracing (debug): with max_steps > 0, every t3b_decode records the
 * logits its first stream samples from (prefill logits, then each step's)
 * into a device buffer of max_steps + 1 rows; t3b_get_logits_trace copies
 * the first n rows to host memory [n][n_speech_vocab].  0 disables. */
int t3b_trace_logits(t3b_ctx * ctx, int max_steps);
int t3b_get_logits_trace(t3b_ctx * ctx, float * out, int n);

/* The cudaStream_t (as void*) every kernel of this context runs on, for
 * callers that order their own work or timing events against it. */
void * t3b_stream_handle(const t3b_ctx * ctx);

/* Residual-stream trace (parity diagnostics; no counterpart in
 * chatterbox.cpp, whose graph keeps intermediate tensors internal).  With
 * on != 0, a t3b_step (and the first step of a persistent-kernel
 * t3b_decode) records the hidden state of its first row: row 0 = the step
 * embedding speech_emb[tok] + wpe[pos] (main.cpp:625-627), row l + 1 = the
 * output of layer l (after the MLP residual, main.cpp:571).
 * t3b_get_hidden_trace copies [n_layer + 1][n_embd] floats to host memory. */
int t3b_trace_hidden(t3b_ctx * ctx, int on);
int t3b_get_hidden_trace(t3b_ctx * ctx, float * out);

/* Polls after which a wait of the persistent decode kernel (for another
 * CTA's hand-off or for a staging copy) gives up and the call returns
 * T3B_ERR_TIMEOUT; 0 restores the default (~2M polls, about a second).  A
 * copy still in flight is always waited for before a CTA exits.  No
 * counterpart in chatterbox.cpp (its CPU graph has no device waits). */
int t3b_set_wait_limit(t3b_ctx * ctx, unsigned polls);

/* Kernels this context launched from t3b_step, t3b_sample and t3b_decode
 * (cumulative; a persistent decode counts one launch). */
unsigned long long t3b_launch_count(const t3b_ctx * ctx);

/* S3Gen hand-off (replaces the host copy of `generated` that
 * chatterbox_engine.cpp:395 passes to s3gen_synthesize_to_wav,
 * src/chatterbox_tts.cpp:1297): writes the stream's speech tokens into the
 * caller's DEVICE buffer tokens_dev with S3Gen's own preprocessing
 * (chatterbox_tts.cpp:1389-1398: ids >= 6561, i.e. start/stop, dropped;
 * append_silence != 0 appends 3 silence tokens 4299), and the count into
 * the device int *n_dev (-1 when it exceeds cap).  Runs after the context's
 * queued work; consumer_stream (cudaStream_t, nullable) is made to wait for
 * it, so a ggml-cuda S3Gen stream can read the buffer without a host sync. */
int t3b_s3gen_tokens(t3b_ctx * ctx, int stream, int32_t * tokens_dev, int cap, int32_t * n_dev, int append_silence,
                     void * consumer_stream);

/* ---------------- kernel-level entry points (device pointers) ----------- */

/* Bytes of one repacked weight row: Q4_0 K*9/16, Q8_0 K*17/16, F16 2K. */
size_t t3b_op_row_bytes(int dtype, int K);

/* Repack N GGUF rows (ne0 = K) from host memory into the device row layout
 * the GEMV kernels read: per row the quants (nibbles / int8 / f16) then the
 * K/32 f16 block scales. */
int t3b_op_repack(int dtype, const void * gguf_rows_host, int N, int K, void * out_dev);

/* ggml_mul_mat(W, x) + bias with an epilogue (main.cpp:505,562-571,577):
 *   epilogue 0: y = W.x + b
 *   epilogue 1: y = gelu(W.x + b)          (ggml_gelu, f16-table semantics)
 *   epilogue 2: y = (W.x + b) + residual   (residual may alias y)
 * ln_g/ln_b non-NULL apply LayerNorm (ggml_norm * g + b, eps) to x first.
 * x: [M][K] f32, y: [M][N] f32. */
int t3b_op_gemv(int dtype, const void * w_dev, int N, int K, const float * x_dev, int M,
                const float * ln_g, const float * ln_b, float eps, const float * bias_dev,
                const float * residual_dev, int epilogue, float * y_dev, void * cuda_stream);

/* Decode attention (ggml_flash_attn_ext at N=1, main.cpp:548-560) for M
 * rows: q [M][n_head*64] f32, caches [M][n_head][max_ctx][64] f16, row m
 * attends positions 0 .. len[m]-1, scale 1/8.  out [M][n_head*64] f32.
 * The K and V caches are read with 16-byte loads: both pointers must be
 * 16-byte aligned (T3B_ERR_ARG otherwise; the same holds for the prompt and
 * allocation-free variants). */
int t3b_op_attention(const float * q_dev, const void * k_dev, const void * v_dev, int M,
                     int n_head, int max_ctx, const int32_t * len_dev, float * out_dev,
                     void * cuda_stream);

/* Causal attention of a prompt chunk (ggml_flash_attn_ext with eval_prompt's
 * causal mask, main.cpp:548-560,663-677): M query rows of ONE cache, row m
 * at position pos[m] attending keys 0 .. pos[m]; q [M][n_head*64] f32,
 * caches [n_head][max_ctx][64] f16 (K and V given separately), scale 1/8,
 * out [M][n_head*64] f32.  Flash-attention tiling (64 queries x 64 keys
 * per step).  Length errors are kept for t3b_op_check. */
int t3b_op_attention_prompt(const float * q_dev, const void * k_dev, const void * v_dev, int M, int n_head,
                            int max_ctx, const int32_t * pos_dev, float * out_dev, void * cuda_stream);

/* The fused sampler on device buffers: cond/uncond logits [rows][V] f32
 * (uncond nullable), history [rows][hist_stride] i32 with hist_len[rows],
 * per-row params, Philox seeds/counters [rows] (u64), tokens_out [rows]. */
int t3b_op_sample_philox(const float * cond_dev, const float * uncond_dev, int rows, int V,
                         const int32_t * hist_dev, const int32_t * hist_len_dev, int hist_stride,
                         const t3b_sample_params * params_dev, const uint64_t * seed_dev,
                         const uint64_t * counter_dev, int32_t * tokens_out_dev,
                         void * cuda_stream);

/* Allocation-free variant of t3b_op_attention (this entry point has no
 * counterpart in chatterbox.cpp).  It is for callers that may not allocate
 * device memory on their decode path: hosts that hand every byte of device
 * memory to their own pool allocator, and real-time callers that cannot
 * afford cudaMalloc, which may take allocator locks or synchronise the
 * device.  The split partials and completion counters live in a fixed
 * static device array that every GPU loading libt3b200.so keeps until the
 * process exits (4 MiB of partials + 16 KiB of counters).  Limits: M x n_head
 * x ceil(max_ctx / 128) <= 15887 partial records (for M < 8; from 8 rows on
 * the kernel needs no partials) and M x n_head <= 4096; larger calls return
 * T3B_ERR_ARG without launching.  The first call on a device resolves the
 * array's address (cudaGetSymbolAddress) and should be made before any
 * stream capture.  All calls share the array: each call clears the counters
 * it uses on `cuda_stream` first, and calls whose kernels overlap on the
 * GPU (two streams, or two threads) race on it.  Length errors are kept for
 * t3b_op_check. */
int t3b_op_attention_noalloc(const float * q_dev, const void * k_dev, const void * v_dev, int M,
                             int n_head, int max_ctx, const int32_t * len_dev, float * out_dev,
                             void * cuda_stream);

/* Synchronises cuda_stream, then reads and clears the device error words of
 * t3b_op_attention and t3b_op_attention_noalloc on the current device: a row
 * whose len is <= 0 or > max_ctx is skipped by the kernel (its output left
 * unwritten) and reported here as T3B_ERR_DEVICE.  Errors stay recorded
 * until this call. */
int t3b_op_check(void * cuda_stream);

/* Host expf fix-up table size (entries where the device exp needed a
 * correction to equal the host libm's expf). */
int t3b_expf_fixup_count(void);
/* Device exp for a batch of floats (test hook): out[i] = expf(in[i]) with
 * the host libm's rounding, computed by the sampler's device routine. */
int t3b_op_expf(const float * in_dev, float * out_dev, int n, void * cuda_stream);

#ifdef __cplusplus
}
#endif

#endif /* T3B200_H */
