// serve.cuh — continuous batching over the context's stream slots (host
// code, included by t3b_abi.cu after the context is defined).
//
// Replaces the per-utterance loops of chatterbox.cpp's callers
// (Engine::Impl::run_t3, src/chatterbox_engine.cpp:330-358, and the CLI's
// per-segment loop with its early-stop retry, src/chatterbox_cli.cpp:
// 1597-1683) by many utterances in flight at once: requests wait in a
// queue, each is admitted into a free stream slot (prefill + first sample),
// every iteration steps all admitted streams in ONE batched step (embedding,
// layers and head over all their rows, one sampler CTA per stream), and a
// stream that ends (stop token, its n_predict steps, or the end of its cache)
// leaves its slot to the next request at once.
//
// Per request the loop is run_t3's: sample from the prompt logits, then
// (stop? / context full? -> end) step + sample, at most n_predict steps; a
// trailing stop token is popped.  Early-stop retry as in the CLI: when the
// stop token ends an utterance shorter than min_tokens, it is replayed (up
// to max_retries times) from the request's seed with the mt19937 stream
// advanced by attempt * 1009 draws; if every attempt is short the longest
// is kept.
#pragma once

#include <deque>

struct ServeReq {
    std::vector<int32_t> text, cond;
    std::vector<float> spk;
    bool has_cond = false, has_spk = false;
    t3b_sample_params params{};
    int rng_mode = T3B_RNG_MT19937;
    uint64_t seed = 0;
    int n_predict = 0, min_tokens = 0, max_retries = 0;
    // progress
    int attempt = 0, steps = 0, slot = -1;
    bool stopped = false, finished = false;
    int failed = T3B_OK;            // admission error (e.g. prompt longer than the context)
    std::vector<int32_t> gen, best, result;
};

struct ServeState {
    std::vector<ServeReq> reqs;
    std::deque<int> queue;          // request ids waiting for a slot (retries go first)
    std::vector<int> slot_req;      // per stream slot: request id or -1
    std::vector<int> active;        // slots stepped together, in list order
    bool dirty = true;              // active list changed since the last upload
    int * tok_pin = nullptr;        // pinned copy of the step's sampled tokens
    int tok_cap = 0;
    long long step_tokens = 0;      // tokens sampled by batched steps since the slots were allocated
    double step_ms = 0.0;           // device time of those steps
};

ServeState * serve_create() { return new ServeState(); }
void serve_destroy(ServeState * s) {
    if (!s) return;
    if (s->tok_pin) cudaFreeHost(s->tok_pin);
    delete s;
}

namespace {

// Ends the current attempt of request r (CLI semantics): pop a trailing stop
// token, keep the longest attempt, replay a short stop-token ending.
void serve_end_attempt(t3b_ctx * ctx, ServeState & S, int r) {
    ServeReq & q = S.reqs[r];
    const int stop = ctx->hp.stop_speech_token;
    if (!q.gen.empty() && q.gen.back() == stop) q.gen.pop_back();
    if (q.gen.size() > q.best.size()) q.best = q.gen;
    const bool plausible = (int) q.gen.size() >= q.min_tokens;
    S.slot_req[q.slot] = -1;
    q.slot = -1;
    S.dirty = true;
    if (!q.stopped || plausible) {
        q.result = q.gen;
        q.finished = true;
    } else if (q.attempt < q.max_retries) {
        q.attempt += 1;
        S.queue.push_front(r);
    } else {
        q.result = q.best;
        q.finished = true;
    }
}

// Prefill + first sample of request r in stream slot `slot`.
int serve_admit(t3b_ctx * ctx, ServeState & S, int r, int slot) {
    ServeReq & q = S.reqs[r];
    q.slot = slot;
    q.steps = 0;
    q.stopped = false;
    q.gen.clear();
    S.slot_req[slot] = r;
    S.dirty = true;
    int32_t P = 0;
    int rc = t3b_prefill(ctx, slot, q.text.data(), (int) q.text.size(), q.has_cond ? q.cond.data() : nullptr,
                         (int) q.cond.size(), q.has_spk ? q.spk.data() : nullptr, nullptr, &P);
    if (rc == T3B_OK) rc = t3b_set_rng(ctx, slot, q.rng_mode, q.seed, (uint64_t) q.attempt * 1009u);
    int32_t tok = 0;
    const int32_t sl = slot;
    if (rc == T3B_OK) rc = t3b_sample(ctx, 1, &sl, &q.params, nullptr, &tok);
    if (rc != T3B_OK) {
        // the request ends with the error; the slot stays free
        S.slot_req[slot] = -1;
        q.slot = -1;
        q.failed = rc;
        q.finished = true;
        return rc == T3B_ERR_ARG ? T3B_OK : rc;   // a bad request does not stop the others
    }
    q.gen.push_back(tok);
    const int stop = ctx->hp.stop_speech_token;
    if (tok == stop) { q.stopped = true; serve_end_attempt(ctx, S, r); }
    else if (q.n_predict <= 0 || P + 1 > ctx->max_ctx) serve_end_attempt(ctx, S, r);
    return T3B_OK;
}

}  // namespace

extern "C" {

int t3b_serve_submit(t3b_ctx * ctx, const t3b_request * req) {
    if (!ctx || !req) return T3B_ERR_ARG;
    if (ctx->S == 0) { set_err(&ctx->err, "t3b_serve_submit: no streams allocated"); return T3B_ERR_STATE; }
    if (req->n_text < 0 || (req->n_text > 0 && !req->text) || req->n_cond < 0 || req->n_predict < 0 ||
        req->min_tokens < 0 || req->max_retries < 0 ||
        (req->rng_mode != T3B_RNG_MT19937 && req->rng_mode != T3B_RNG_PHILOX)) {
        set_err(&ctx->err, "t3b_serve_submit: bad request");
        return T3B_ERR_ARG;
    }
    ServeState & S = *ctx->serve;
    ServeReq q;
    q.text.assign(req->text, req->text + req->n_text);
    if (req->cond_tokens) { q.has_cond = true; q.cond.assign(req->cond_tokens, req->cond_tokens + req->n_cond); }
    if (req->spk_emb) { q.has_spk = true; q.spk.assign(req->spk_emb, req->spk_emb + ctx->hp.speaker_embed_size); }
    q.params = req->params;
    q.rng_mode = req->rng_mode;
    q.seed = req->seed;
    q.n_predict = req->n_predict;
    q.min_tokens = req->min_tokens;
    q.max_retries = req->max_retries;
    S.reqs.push_back(std::move(q));
    const int id = (int) S.reqs.size() - 1;
    S.queue.push_back(id);
    return id;
}

int t3b_serve_run(t3b_ctx * ctx, int max_iters, int32_t * n_active, int32_t * n_queued) {
    if (!ctx || max_iters < 0) return T3B_ERR_ARG;
    if (ctx->S == 0) { set_err(&ctx->err, "t3b_serve_run: no streams allocated"); return T3B_ERR_STATE; }
    CK(cudaSetDevice(ctx->device));
    ServeState & S = *ctx->serve;
    if ((int) S.slot_req.size() != ctx->S) S.slot_req.assign(ctx->S, -1);
    cudaStream_t st = ctx->st;
    const int stop = ctx->hp.stop_speech_token;
    float total_ms = 0.0f;
    for (int it = 0; it < max_iters; ++it) {
        // admit into free slots (retries first, then in submission order)
        for (int s = 0; s < ctx->S && !S.queue.empty(); ++s) {
            if (S.slot_req[s] >= 0) continue;
            const int r = S.queue.front();
            S.queue.pop_front();
            const int rc = serve_admit(ctx, S, r, s);
            if (rc != T3B_OK) return rc;
            if (S.slot_req[s] < 0) --s;   // ended at its first token: the slot is free again
        }
        if (S.dirty) {
            S.active.clear();
            for (int s = 0; s < ctx->S; ++s)
                if (S.slot_req[s] >= 0) S.active.push_back(s);
        }
        const int n = (int) S.active.size();
        if (n == 0) break;
        StepGraph * g = nullptr;
        int rc = ensure_graph(ctx, n, true, &g);
        if (rc != T3B_OK) return rc;
        if (S.dirty) {
            // row maps, per-row positions and per-stream params of the new list
            rc = upload_maps(ctx, S.active);
            if (rc != T3B_OK) return rc;
            std::vector<int> pos(n * ctx->rps);
            std::vector<t3b_sample_params> prm(n);
            for (int i = 0; i < n; ++i) {
                prm[i] = S.reqs[S.slot_req[S.active[i]]].params;
                for (int j = 0; j < ctx->rps; ++j) pos[i * ctx->rps + j] = ctx->pos_host[S.active[i] * ctx->rps + j];
            }
            CK(cudaMemcpyAsync(ctx->pos, pos.data(), sizeof(int) * pos.size(), cudaMemcpyHostToDevice, st));
            CK(cudaMemcpyAsync(ctx->params, prm.data(), sizeof(t3b_sample_params) * n, cudaMemcpyHostToDevice, st));
            ctx->params_last.clear();
            if (S.tok_cap < ctx->S) {
                if (S.tok_pin) CK(cudaFreeHost(S.tok_pin));
                CK(cudaHostAlloc((void **) &S.tok_pin, sizeof(int) * ctx->S, cudaHostAllocDefault));
                S.tok_cap = ctx->S;
            }
            S.dirty = false;
        }
        CK(cudaEventRecord(ctx->ev0, st));
        CK(cudaGraphLaunch(g->ge, st));
        ctx->launches += (unsigned long long) g->n_kernels;
        CK(cudaEventRecord(ctx->ev1, st));
        CK(cudaMemcpyAsync(S.tok_pin, ctx->tok_out, sizeof(int) * n, cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
        float ms = 0.0f;
        cudaEventElapsedTime(&ms, ctx->ev0, ctx->ev1);
        total_ms += ms;
        S.step_ms += ms;
        S.step_tokens += n;
        rc = check_dev_err(ctx);
        if (rc != T3B_OK) return rc;
        for (int i = 0; i < n; ++i) {
            const int s = S.active[i], r = S.slot_req[s];
            ServeReq & q = S.reqs[r];
            for (int j = 0; j < ctx->rps; ++j) ctx->pos_host[s * ctx->rps + j] += 1;
            const int t = S.tok_pin[i];
            q.gen.push_back(t);
            q.steps += 1;
            if (t == stop) { q.stopped = true; serve_end_attempt(ctx, S, r); }
            else if (q.steps >= q.n_predict || ctx->pos_host[s * ctx->rps] + 1 > ctx->max_ctx) serve_end_attempt(ctx, S, r);
        }
    }
    ctx->last_ms = total_ms;
    int act = 0;
    for (int r : S.slot_req) act += r >= 0;
    if (n_active) *n_active = act;
    if (n_queued) *n_queued = (int) S.queue.size();
    return T3B_OK;
}

int t3b_serve_result(t3b_ctx * ctx, int id, int32_t * tokens_out, int cap, int32_t * n_out, int32_t * attempts) {
    if (!ctx) return T3B_ERR_ARG;
    ServeState & S = *ctx->serve;
    if (id < 0 || id >= (int) S.reqs.size() || cap < 0 || (cap > 0 && !tokens_out)) {
        set_err(&ctx->err, "t3b_serve_result: bad request id or buffer");
        return T3B_ERR_ARG;
    }
    const ServeReq & q = S.reqs[id];
    if (attempts) *attempts = q.attempt + 1;
    if (!q.finished) return 0;
    if (q.failed != T3B_OK) { set_err(&ctx->err, "t3b_serve_result: request %d failed at admission", id); return q.failed; }
    const int n = (int) q.result.size();
    if (n_out) *n_out = n;
    if (cap > 0) std::memcpy(tokens_out, q.result.data(), sizeof(int32_t) * (size_t) std::min(n, cap));
    return 1;
}

int t3b_serve_stats(const t3b_ctx * ctx, long long * step_tokens, double * step_ms) {
    if (!ctx || !ctx->serve) return T3B_ERR_ARG;
    if (step_tokens) *step_tokens = ctx->serve->step_tokens;
    if (step_ms) *step_ms = ctx->serve->step_ms;
    return T3B_OK;
}

}  // extern "C"
