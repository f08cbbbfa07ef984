// t3b_abi.cu — libt3b200.so: the C ABI declared in include/t3b200.h.
//
// Owns the device copy of a T3 model (repacked weight rows, f32 norms and
// biases, f16 embeddings), the per-stream f16 KV caches and sampler state,
// and launches the kernels of kernels.cuh / megakernel.cuh on one CUDA
// stream per context.  A decode step for a fixed set of streams is captured
// once as a CUDA graph and replayed (tokens and positions live on the
// device), so the host issues one launch per step.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cudaTypedefs.h>   // PFN_cuTensorMapEncodeTiled

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <random>
#include <sstream>
#include <string>
#include <vector>

#include "kernels.cuh"
#include "megakernel.cuh"

#include "expf_fixup.inc"   // generated at build time by gen_expf_fixup

namespace {

thread_local std::string g_err;   // error of the last failed call without a ctx

void set_err(std::string * dst, const char * fmt, ...) {
    char buf[1024];
    va_list ap; va_start(ap, fmt); vsnprintf(buf, sizeof buf, fmt, ap); va_end(ap);
    if (dst) *dst = buf;
    g_err = buf;
}

#define CK(call) do { cudaError_t e_ = (call); if (e_ != cudaSuccess) { \
    set_err(ERRP, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); return T3B_ERR_CUDA; } } while (0)

// --------------------------------------------------------------------------
// exp fix-up hash table (one per device)
// --------------------------------------------------------------------------
constexpr int kFixBits = 16;   // 2^16 buckets x 4 slots x 8 bytes = 2 MB
struct FixTab { unsigned long long * dev = nullptr; int bits = kFixBits; };
std::mutex g_fix_mu;
std::map<int, FixTab> g_fix;

// Builds the two-choice table: each entry goes to the emptier of its two
// buckets.  Returns false if a bucket pair is full (never for the shipped
// fix-up list at this size; the caller then doubles the table).
bool build_fix_table(int bits, std::vector<unsigned long long> & tab) {
    const uint32_t nb = 1u << bits;
    tab.assign((size_t) nb * T3_EXPF_SLOTS, 0ull);
    std::vector<int> fill(nb, 0);
    for (uint32_t i = 0; i < t3_expf_fixup_n; ++i) {
        const uint32_t key = t3_expf_fixup[i][0];
        const uint32_t h1 = t3_expf_hash1(key, bits), h2 = t3_expf_hash2(key, bits);
        const uint32_t b = fill[h2] < fill[h1] ? h2 : h1;
        if (fill[b] >= T3_EXPF_SLOTS) return false;
        tab[(size_t) b * T3_EXPF_SLOTS + fill[b]++] = ((unsigned long long) key << 32) | t3_expf_fixup[i][1];
    }
    return true;
}

int fix_table(int device, ExpFix * out, std::string * ERRP) {
    std::lock_guard<std::mutex> lk(g_fix_mu);
    auto it = g_fix.find(device);
    if (it == g_fix.end()) {
        std::vector<unsigned long long> tab;
        int bits = kFixBits;
        while (!build_fix_table(bits, tab)) ++bits;
        FixTab ft;
        ft.bits = bits;
        CK(cudaMalloc(&ft.dev, tab.size() * sizeof(unsigned long long)));
        CK(cudaMemcpy(ft.dev, tab.data(), tab.size() * sizeof(unsigned long long), cudaMemcpyHostToDevice));
        it = g_fix.emplace(device, ft).first;
    }
    out->tab = it->second.dev;
    out->bits = it->second.bits;
    out->n = (int) t3_expf_fixup_n;
    return T3B_OK;
}

size_t row_bytes(int type, int K) {
    switch (type) {
        case T3B_Q4_0: return (size_t) K / 2 + (size_t) K / 32 * 2;
        case T3B_Q8_0: return (size_t) K + (size_t) K / 32 * 2;
        case T3B_F16: return (size_t) K * 2;
        case T3B_F32: return (size_t) K * 4;
    }
    return 0;
}
size_t gguf_row_bytes(int type, int K) {
    switch (type) {
        case T3B_Q4_0: return (size_t) K / 32 * 18;
        case T3B_Q8_0: return (size_t) K / 32 * 34;
        case T3B_F16: return (size_t) K * 2;
        case T3B_F32: return (size_t) K * 4;
    }
    return 0;
}

// GGUF rows -> device row layout (quants first, then the block scales).
void repack_rows(int type, const uint8_t * src, int N, int K, uint8_t * dst) {
    const size_t gr = gguf_row_bytes(type, K), rr = row_bytes(type, K);
    for (int n = 0; n < N; ++n) {
        const uint8_t * s = src + gr * n;
        uint8_t * d = dst + rr * n;
        if (type == T3B_Q4_0) {
            for (int b = 0; b < K / 32; ++b) {
                std::memcpy(d + 16 * b, s + 18 * b + 2, 16);
                std::memcpy(d + K / 2 + 2 * b, s + 18 * b, 2);
            }
        } else if (type == T3B_Q8_0) {
            for (int b = 0; b < K / 32; ++b) {
                std::memcpy(d + 32 * b, s + 34 * b + 2, 32);
                std::memcpy(d + K + 2 * b, s + 34 * b, 2);
            }
        } else {
            std::memcpy(d, s, rr);
        }
    }
}

struct Mat { int type = -1, N = 0, K = 0; int rb = 0; uint8_t * p = nullptr; };
struct Layer {
    float * ln1g = nullptr, * ln1b = nullptr, * ln2g = nullptr, * ln2b = nullptr;
    float * attn_b = nullptr, * proj_b = nullptr, * fc_b = nullptr, * fc2_b = nullptr;
    Mat attn, proj, fc, fc2;
};

// Split-K workspace of the tensor-core F16 GEMM: partial tiles and per-tile
// completion counters (zero at allocation; the kernel leaves them zero)
struct GemmWs { float * ws = nullptr; size_t cap = 0; unsigned * cnt = nullptr; int ccap = 0; };
#define TF_CNT 4096

struct StepGraph {
    cudaGraph_t g = nullptr;
    cudaGraphExec_t ge = nullptr;
    int n_kernels = 0;   // kernel nodes per launch (launch accounting)
};

}  // namespace

struct ServeState;                       // serve.cuh: continuous-batching scheduler
ServeState * serve_create();
void serve_destroy(ServeState * s);

struct t3b_ctx {
    int device = 0;
    cudaStream_t st = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    t3b_hparams hp{};
    std::string err;
    std::vector<void *> allocs;     // model allocations
    std::vector<Layer> L;
    float * wpe = nullptr, * lnf_g = nullptr, * lnf_b = nullptr, * head_b = nullptr;
    float * spkr_w = nullptr, * spkr_b = nullptr, * builtin_spk = nullptr;
    __half * semb = nullptr, * temb = nullptr;
    Mat head;
    std::vector<int32_t> builtin_cond;
    ExpFix fx{};
    unsigned * err_word = nullptr;
    unsigned * err_pin = nullptr;   // pinned host copy of err_word (read in the same synchronize as results)
    // pinned staging of the per-step calls' host buffers (logits in/out, tokens): a pageable copy of
    // 26 KB costs a synchronous staging pass of its own
    float * io_pin = nullptr; size_t io_pin_cap = 0;
    std::vector<t3b_sample_params> params_last;   // what t3b_sample last uploaded to params (empty: unknown)
    volatile int cancel = 0;
    float last_ms = 0.0f;
    unsigned wait_limit = 0;            // persistent-kernel wait limit in polls (0: MK_SPIN)
    unsigned long long launches = 0;    // kernels launched by t3b_step / t3b_sample / t3b_decode
    float * htrace = nullptr;           // nullable: [n_layer + 1][n_embd] residual stream of the last traced step
    cudaEvent_t hand_ev = nullptr;      // t3b_s3gen_tokens: consumer streams wait on it
    cudaEvent_t q_ev[2] = {nullptr, nullptr};   // graph decode loop: bounds the steps queued ahead

    // streams
    int S = 0, rps = 1, max_ctx = 0, hist_cap = 0, s_max = 1;
    __half * kv = nullptr; size_t row_elems = 0;
    std::vector<int> pos_host;      // per cache row
    std::vector<void *> sallocs;    // stream allocations
    // per-slot device state
    int * hist = nullptr, * hist_len = nullptr, * rng_mode = nullptr, * done = nullptr, * step_tok = nullptr;
    uint32_t * mt = nullptr;
    unsigned long long * ph_seed = nullptr, * ph_ctr = nullptr;
    t3b_sample_params * params = nullptr;
    int * tok_out = nullptr;
    std::vector<int> rng_mode_host;
    // scratch (R rows)
    int R = 0;
    float * x = nullptr, * qkv = nullptr, * attn = nullptr, * h = nullptr, * logits = nullptr, * part = nullptr;
    float * spk = nullptr;
    int8_t * xq = nullptr; float * xd = nullptr; int * xs = nullptr; __half * xh = nullptr;
    int8_t * xq2 = nullptr; float * xd2 = nullptr; int * xs2 = nullptr;   // fc2 input written by the fc GEMM
    unsigned * cnt = nullptr;
    int * row_slot = nullptr, * pos = nullptr, * row_of = nullptr, * y_row = nullptr;
    int * pk_kind = nullptr, * pk_id = nullptr, * slot_list = nullptr;
    std::vector<int> maps_slots;    // slot list row_slot/row_of/slot_list hold (empty: unknown)
    // captured step graphs keyed by the slot list (+ whether sampling)
    std::map<std::vector<int>, StepGraph> graphs;
    // persistent batch-1 decode kernel state
    MegaState mega{};
    // logits trace (debug)
    float * trace = nullptr; int trace_cap = 0;
    // continuous batching over the stream slots (t3b_serve_*)
    ServeState * serve = nullptr;
    GemmWs gws;                     // split-K workspace of the tensor-core F16 GEMM
};

#undef ERRP
#define ERRP (&ctx->err)

namespace {

template <class T>
int dalloc(t3b_ctx * ctx, std::vector<void *> & list, T ** p, size_t n) {
    void * q = nullptr;
    cudaError_t e = cudaMalloc(&q, std::max<size_t>(n, 1) * sizeof(T));
    if (e != cudaSuccess) {
        set_err(&ctx->err, "cudaMalloc(%zu bytes): %s", n * sizeof(T), cudaGetErrorString(e));
        return T3B_ERR_OOM;
    }
    list.push_back(q);
    *p = (T *) q;
    return T3B_OK;
}

int check_dev_err(t3b_ctx * ctx) {
    unsigned w = 0;
    CK(cudaMemcpyAsync(&w, ctx->err_word, sizeof w, cudaMemcpyDeviceToHost, ctx->st));
    CK(cudaStreamSynchronize(ctx->st));
    if (w) {
        CK(cudaMemsetAsync(ctx->err_word, 0, sizeof(unsigned), ctx->st));
        set_err(&ctx->err, "device check failed (error word 0x%x:%s%s%s)", w,
                (w & T3B_DEVERR_TOKEN) ? " token-out-of-range" : "",
                (w & T3B_DEVERR_POS) ? " position-out-of-range" : "",
                (w & T3B_DEVERR_TIMEOUT) ? " wait-timeout" : "");
        return (w & T3B_DEVERR_TIMEOUT) ? T3B_ERR_TIMEOUT : T3B_ERR_DEVICE;
    }
    return T3B_OK;
}

void free_streams(t3b_ctx * ctx) {
    for (auto & kv : ctx->graphs) {
        if (kv.second.ge) cudaGraphExecDestroy(kv.second.ge);
        if (kv.second.g) cudaGraphDestroy(kv.second.g);
    }
    ctx->graphs.clear();
    ctx->maps_slots.clear();
    for (void * p : ctx->sallocs) cudaFree(p);
    ctx->sallocs.clear();
    ctx->S = 0; ctx->R = 0; ctx->kv = nullptr; ctx->gws = GemmWs();
    mega_free(ctx->mega);
    serve_destroy(ctx->serve);
    ctx->serve = nullptr;
}

// ----- kernel launch helpers (stream = ctx->st) -----

int launch_prep(t3b_ctx * ctx, const float * x, int ldx, int M, int K, const float * g, const float * b, int wtype,
                cudaStream_t st) {
    const int qmode = (wtype == T3B_F16) ? 2 : 1;
    prep_act_kernel<<<M, 256, K * sizeof(float), st>>>(x, ldx, K, g, b, ctx ? ctx->hp.eps : 1e-5f, qmode,
                                                       ctx->xq, ctx->xd, ctx->xs, ctx->xh);
    return T3B_OK;
}

template <int WT, int MT>
void launch_gemv_q_t(const Mat & W, const int8_t * xq, const float * xd, const int * xs, int M, const GemvEpi & e,
                     cudaStream_t st) {
    constexpr int RPW = 2;
    dim3 grid((W.N + 8 * RPW - 1) / (8 * RPW), (M + MT - 1) / MT);
    const size_t smem = (size_t) MT * W.K + (size_t) MT * (W.K / 32) * 8;
    gemv_q_kernel<WT, MT, RPW><<<grid, 256, smem, st>>>(W.p, W.N, W.K, W.rb, xq, xd, xs, M, e);
}
template <int MT, int RPW>
void launch_gemv_h_r(const Mat & W, const __half * xh, int M, const GemvEpi & e, cudaStream_t st) {
    dim3 grid((W.N + 8 * RPW - 1) / (8 * RPW), (M + MT - 1) / MT);
    const size_t smem = (size_t) MT * W.K * 2;
    gemv_f16_kernel<MT, RPW><<<grid, 256, smem, st>>>((const __half *) W.p, W.N, W.K, xh, M, e);
}
template <int MT>
void launch_gemv_h_t(const Mat & W, const __half * xh, int M, const GemvEpi & e, cudaStream_t st) {
    // one row per warp when two would leave SMs idle
    if ((W.N + 15) / 16 * ((M + MT - 1) / MT) < 148) launch_gemv_h_r<MT, 1>(W, xh, M, e, st);
    else launch_gemv_h_r<MT, 2>(W, xh, M, e, st);
}
// activation rows from which quantised weights go through gemm_q_mma_kernel
// (M <= 4 run the one-launch GEMV): at M = 8 the GEMM with 32-row tiles takes
// about half the time of gemv_q_kernel, and it adds the per-block terms in
// block order, as ggml's dot does
#define GQ_MIN_M 5
template <int WT>
void launch_gemv_q(const Mat & W, const int8_t * xq, const float * xd, const int * xs, int M, const GemvEpi & e,
                   cudaStream_t st) {
    if (M >= GQ_MIN_M && W.K % (32 * GQ_KB) == 0) {   // several rows: int8 tensor-core GEMM
        // 32-row tiles when 64-row ones would leave SMs idle (N = 1024: 64 CTAs at M = 128)
        const int tx = (W.N + GQ_BN - 1) / GQ_BN;
        if (tx * ((M + GQ_BM - 1) / GQ_BM) < 148) {
            // eight warps (one 16 x 8 MMA tile each): with one CTA per SM,
            // four warps left the schedulers idle between dependent steps
            gemm_q_mma_kernel<WT, 32, 8><<<dim3(tx, (M + 31) / 32), 256, 0, st>>>(W.p, W.N, W.K, W.rb, xq, xd, xs, M, e);
        } else {
            gemm_q_mma_kernel<WT, GQ_BM, 4><<<dim3(tx, (M + GQ_BM - 1) / GQ_BM), 128, 0, st>>>(W.p, W.N, W.K, W.rb, xq, xd,
                                                                                       xs, M, e);
        }
        return;
    }
    if (M <= 1) launch_gemv_q_t<WT, 1>(W, xq, xd, xs, M, e, st);
    else if (M <= 2) launch_gemv_q_t<WT, 2>(W, xq, xd, xs, M, e, st);
    else if (M <= 4) launch_gemv_q_t<WT, 4>(W, xq, xd, xs, M, e, st);
    else launch_gemv_q_t<WT, 8>(W, xq, xd, xs, M, e, st);
}
// activation rows from which the F16 GEMMs run on the tensor cores
#define TC_MIN_M 16

// cuTensorMapEncodeTiled from the driver, resolved once; the attribute for
// gemm_f16_tc_kernel's dynamic shared memory set once per device
PFN_cuTensorMapEncodeTiled_v12000 tf_encode() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void * f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000) f;
    });
    return fn;
}
bool tf_attr_ready() {
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    std::lock_guard<std::mutex> lk(mu);
    if (!done[dev]) {
        if (cudaFuncSetAttribute(gemm_f16_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TF_SMEM) != cudaSuccess)
            return false;
        done[dev] = true;
    }
    return true;
}
// 2-D f16 tensor [rows][K] (row stride K halves), boxes of 64 halves (128
// bytes) x box_rows written with the 128-byte swizzle the MMA descriptors use
bool tf_map(CUtensorMap * map, const void * base, int K, int rows, int box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 enc = tf_encode();
    if (!enc || ((uintptr_t) base & 15) || (K * 2) % 16) return false;
    const cuuint64_t dims[2] = {(cuuint64_t) K, (cuuint64_t) rows};
    const cuuint64_t strides[1] = {(cuuint64_t) K * 2};
    const cuuint32_t box[2] = {(cuuint32_t) TF_BK, (cuuint32_t) box_rows};
    const cuuint32_t es[2] = {1u, 1u};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// F16 weights x f16 activations on the tensor cores (M >= TC_MIN_M rows).
// Split-K (deterministic) when the output tiles alone leave SMs idle.
// Returns false when the shape or the environment does not allow it.
bool launch_gemm_f16_tc(const Mat & W, const __half * xh, int M, const GemvEpi & e, const GemmWs * gw, cudaStream_t st) {
    if (M < TC_MIN_M || !xh || W.K % TF_BK != 0 || !tf_attr_ready()) return false;
    CUtensorMap ta, tb;
    if (!tf_map(&ta, xh, W.K, M, TF_BM) || !tf_map(&tb, W.p, W.K, W.N, TF_BN)) return false;
    const int tx = (W.N + TF_BN - 1) / TF_BN, ty = (M + TF_BM - 1) / TF_BM, tiles = tx * ty;
    const int nkb = W.K / TF_BK;
    int splits = 1;
    if (gw && gw->ws && gw->cnt && tiles <= gw->ccap && tiles < 120) {
        // at least 4 K-steps (256 columns) per split: below that the split
        // partials' write and in-order sum cost more than the idle SMs
        splits = std::min(std::min(std::max(1, 148 / tiles), 8), std::max(1, nkb / 4));
        const size_t ldw = (size_t) tx * TF_BN;
        while (splits > 1 && (nkb % splits != 0 || (size_t) splits * M * ldw > gw->cap)) --splits;
    }
    TfArgs p{};
    p.M = M; p.N = W.N; p.K = W.K; p.kchunk = W.K / splits; p.splits = splits; p.e = e;
    p.ws = splits > 1 ? gw->ws : nullptr; p.cnt = splits > 1 ? gw->cnt : nullptr;
    gemm_f16_tc_kernel<<<dim3(tx, ty, splits), 128, TF_SMEM, st>>>(ta, tb, p);
    return true;
}

void launch_gemv(const Mat & W, const int8_t * xq, const float * xd, const int * xs, const __half * xh, int M,
                 const GemvEpi & e, cudaStream_t st, const GemmWs * gw = nullptr) {
    if (W.type == T3B_Q4_0) launch_gemv_q<T3B_Q4_0>(W, xq, xd, xs, M, e, st);
    else if (W.type == T3B_Q8_0) launch_gemv_q<T3B_Q8_0>(W, xq, xd, xs, M, e, st);
    else {
        if (launch_gemm_f16_tc(W, xh, M, e, gw, st)) return;
        if (M <= 1) launch_gemv_h_t<1>(W, xh, M, e, st);
        else if (M <= 2) launch_gemv_h_t<2>(W, xh, M, e, st);
        else launch_gemv_h_t<4>(W, xh, M, e, st);   // 4 x K=4096 halves = 32 KB smem
    }
}

// Few rows (M <= 4): activation prep and GEMV in one launch
// (gemv_prep_kernel).  Returns false when the shape does not fit it; the
// caller then runs prep_act_kernel + launch_gemv.
#define GP_MAX_M 5   // from 5 rows the per-CTA prep of every row costs more than the second launch (measured)
#define GP_SMEM_MAX (200u * 1024u)   // dynamic bytes (the static arrays and the 227 KB opt-in limit leave room)
template <int WT, int MT, int RPW>
bool launch_gemv_prep_t(const Mat & W, const float * x, int ldx, int M, const float * g, const float * b, float eps,
                        const GemvEpi & e, cudaStream_t st) {
    const size_t smem = gemv_prep_smem(WT, MT, W.K);
    static std::mutex mu;
    static bool ready[64] = {false};
    int dev = 0;
    if (smem > GP_SMEM_MAX || cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return false;
    {   // the opt-in limit (the default 48 KB counts the static arrays too)
        std::lock_guard<std::mutex> lk(mu);
        if (!ready[dev]) {
            if (cudaFuncSetAttribute(gemv_prep_kernel<WT, MT, RPW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     GP_SMEM_MAX) != cudaSuccess) {
                cudaGetLastError();   // not sticky: the caller falls back to two launches
                return false;
            }
            ready[dev] = true;
        }
    }
    // programmatic stream serialization: the kernel waits for its predecessor
    // (griddepcontrol.wait) only after issuing its weight loads
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((W.N + 8 * RPW - 1) / (8 * RPW), (M + MT - 1) / MT);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, gemv_prep_kernel<WT, MT, RPW>, W.p, W.N, W.K, W.rb, x, ldx, g, b, eps, M, e) != cudaSuccess) {
        cudaGetLastError();
        gemv_prep_kernel<WT, MT, RPW><<<cfg.gridDim, 256, smem, st>>>(W.p, W.N, W.K, W.rb, x, ldx, g, b, eps, M, e);
    }
    return true;
}
template <int WT, int MT>
bool launch_gemv_prep_r(const Mat & W, const float * x, int ldx, int M, const float * g, const float * b, float eps,
                        const GemvEpi & e, cudaStream_t st) {
    // one row per warp when two would leave SMs idle (N = 1024: 128 CTAs, not 64)
    if ((W.N + 15) / 16 < 148) return launch_gemv_prep_t<WT, MT, 1>(W, x, ldx, M, g, b, eps, e, st);
    return launch_gemv_prep_t<WT, MT, 2>(W, x, ldx, M, g, b, eps, e, st);
}
template <int WT>
bool launch_gemv_prep_w(const Mat & W, const float * x, int ldx, int M, const float * g, const float * b, float eps,
                        const GemvEpi & e, cudaStream_t st) {
    if (M <= 1) return launch_gemv_prep_r<WT, 1>(W, x, ldx, M, g, b, eps, e, st);
    if (M <= 2) return launch_gemv_prep_r<WT, 2>(W, x, ldx, M, g, b, eps, e, st);
    return launch_gemv_prep_r<WT, 4>(W, x, ldx, M, g, b, eps, e, st);
}
bool launch_gemv_prep(const Mat & W, const float * x, int ldx, int M, const float * g, const float * b, float eps,
                      const GemvEpi & e, cudaStream_t st) {
    if (M <= 0 || M >= GP_MAX_M || W.K % 256 || W.K > 8192) return false;   // K % 256: see the kernel's quantisation
    if (W.type == T3B_Q4_0) return launch_gemv_prep_w<T3B_Q4_0>(W, x, ldx, M, g, b, eps, e, st);
    if (W.type == T3B_Q8_0) return launch_gemv_prep_w<T3B_Q8_0>(W, x, ldx, M, g, b, eps, e, st);
    if (W.type == T3B_F16) return launch_gemv_prep_w<T3B_F16>(W, x, ldx, M, g, b, eps, e, st);
    return false;
}

GemvEpi epi_plain(int kind, float * y, int ldy, const float * bias, const float * res, int ldres) {
    GemvEpi e{};
    e.kind = kind; e.y = y; e.ldy = ldy; e.bias = bias; e.res = res; e.ldres = ldres;
    return e;
}

// Transformer layers + head over M activation rows already embedded in
// ctx->x.  Row m uses cache row row_of[m] at position pos[m] (device
// arrays).  head_rows: rows whose logits are produced (last `head_rows`
// rows of the M), written to logits_out rows y_row[...] (device array) or
// consecutively when y_row is null.
void run_layers(t3b_ctx * ctx, int M, const int * row_of, const int * pos, int head_first, int head_rows,
                float * logits_out, const int * y_row, cudaStream_t st, float * htrace = nullptr, bool prompt = false) {
    const int D = ctx->hp.n_embd, H = ctx->hp.n_head;
    const float eps = ctx->hp.eps;
    if (htrace) cudaMemcpyAsync(htrace, ctx->x, sizeof(float) * D, cudaMemcpyDeviceToDevice, st);
    for (int il = 0; il < ctx->hp.n_layer; ++il) {
        const Layer & Ly = ctx->L[il];
        // LN1 + QKV + K/V append (few rows: one launch)
        GemvEpi e = epi_plain(EPI_QKV, ctx->qkv, 3 * D, Ly.attn_b, nullptr, 0);
        e.kv = ctx->kv; e.row_elems = ctx->row_elems;
        e.layer_off = (size_t) il * 2 * H * ctx->max_ctx * T3B_HD;
        e.v_off = (size_t) H * ctx->max_ctx * T3B_HD;
        e.row_of = row_of; e.pos = pos; e.max_ctx = ctx->max_ctx; e.D = D; e.err = ctx->err_word;
        if (!launch_gemv_prep(Ly.attn, ctx->x, D, M, Ly.ln1g, Ly.ln1b, eps, e, st)) {
            launch_prep(ctx, ctx->x, D, M, D, Ly.ln1g, Ly.ln1b, Ly.attn.type, st);
            launch_gemv(Ly.attn, ctx->xq, ctx->xd, ctx->xs, ctx->xh, M, e, st, &ctx->gws);
        }
        // attention
        AttnArgs a{};
        a.q = ctx->qkv; a.ldq = 3 * D;
        a.kv = ctx->kv; a.row_elems = ctx->row_elems; a.layer_off = e.layer_off; a.v_off = e.v_off;
        a.row_of = row_of; a.len = pos; a.len_add = 1; a.max_ctx = ctx->max_ctx; a.n_head = H;
        a.out = ctx->attn; a.ldo = D; a.part = ctx->part; a.cnt = ctx->cnt; a.s_max = ctx->s_max; a.err = ctx->err_word;
        // many rows: the attention kernel writes the proj GEMM's Q8_0 input itself
        const bool q_attn = (M >= T3B_ATTN_ROWS_MIN || prompt) && Ly.proj.type != T3B_F16;
        if (q_attn) { a.qx = ctx->xq; a.qd = ctx->xd; a.qs = ctx->xs; }
        // a prompt chunk: consecutive positions of one cache row, causal
        if (prompt) attn_prefill_kernel<<<dim3(H, (M + T3B_PF_T - 1) / T3B_PF_T), 256, T3B_PREFILL_SMEM, st>>>(a, M);
        else if (M >= T3B_ATTN_ROWS_MIN) attn_rows_kernel<<<dim3(H, M), 128, 0, st>>>(a);
        else attn_decode_kernel<<<dim3(H, M, ctx->s_max), T3B_ATTN_CHUNK, 0, st>>>(a);
        // proj + bias + residual
        const GemvEpi ep = epi_plain(EPI_RESID, ctx->x, D, Ly.proj_b, ctx->x, D);
        if (q_attn || !launch_gemv_prep(Ly.proj, ctx->attn, D, M, nullptr, nullptr, eps, ep, st)) {
            if (!q_attn) launch_prep(ctx, ctx->attn, D, M, D, nullptr, nullptr, Ly.proj.type, st);
            launch_gemv(Ly.proj, ctx->xq, ctx->xd, ctx->xs, ctx->xh, M, ep, st, &ctx->gws);
        }
        // LN2 + fc + GELU; with the tensor-core GEMM (M >= GQ_MIN_M) its
        // epilogue writes fc2's Q8_0 input (separate buffers: fc is still
        // reading xq)
        GemvEpi ef = epi_plain(EPI_GELU, ctx->h, 4 * D, Ly.fc_b, nullptr, 0);
        const bool q_fc = M >= GQ_MIN_M && Ly.fc.type != T3B_F16 && Ly.fc2.type != T3B_F16 &&
                          Ly.fc.K % (32 * GQ_KB) == 0 && (4 * D) % GQ_BN == 0;
        if (q_fc) { ef.qx = ctx->xq2; ef.qd = ctx->xd2; ef.qs = ctx->xs2; ef.qK = 4 * D; }
        if (q_fc || !launch_gemv_prep(Ly.fc, ctx->x, D, M, Ly.ln2g, Ly.ln2b, eps, ef, st)) {
            launch_prep(ctx, ctx->x, D, M, D, Ly.ln2g, Ly.ln2b, Ly.fc.type, st);
            launch_gemv(Ly.fc, ctx->xq, ctx->xd, ctx->xs, ctx->xh, M, ef, st, &ctx->gws);
        }
        // fc2 + bias + residual
        const GemvEpi e2 = epi_plain(EPI_RESID, ctx->x, D, Ly.fc2_b, ctx->x, D);
        if (q_fc || !launch_gemv_prep(Ly.fc2, ctx->h, 4 * D, M, nullptr, nullptr, eps, e2, st)) {
            if (!q_fc) launch_prep(ctx, ctx->h, 4 * D, M, 4 * D, nullptr, nullptr, Ly.fc2.type, st);
            launch_gemv(Ly.fc2, q_fc ? ctx->xq2 : ctx->xq, q_fc ? ctx->xd2 : ctx->xd, q_fc ? ctx->xs2 : ctx->xs, ctx->xh,
                        M, e2, st, &ctx->gws);
        }
        if (htrace)
            cudaMemcpyAsync(htrace + (size_t) (il + 1) * D, ctx->x, sizeof(float) * D, cudaMemcpyDeviceToDevice, st);
    }
    if (head_rows > 0) {
        GemvEpi e = epi_plain(EPI_BIAS, logits_out, ctx->hp.n_speech_vocab, ctx->head_b, nullptr, 0);
        e.y_row = y_row;
        const float * xh0 = ctx->x + (size_t) head_first * D;
        if (!launch_gemv_prep(ctx->head, xh0, D, head_rows, ctx->lnf_g, ctx->lnf_b, eps, e, st)) {
            launch_prep(ctx, xh0, D, head_rows, D, ctx->lnf_g, ctx->lnf_b, ctx->head.type, st);
            launch_gemv(ctx->head, ctx->xq, ctx->xd, ctx->xs, ctx->xh, head_rows, e, st, &ctx->gws);
        }
    }
}

int ensure_graph(t3b_ctx * ctx, int n, bool sample, StepGraph ** out);

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

const char * t3b_last_error(const t3b_ctx * ctx) { return ctx ? ctx->err.c_str() : g_err.c_str(); }

size_t t3b_op_row_bytes(int dtype, int K) { return row_bytes(dtype, K); }

int t3b_expf_fixup_count(void) { return (int) t3_expf_fixup_n; }

t3b_ctx * t3b_create(int device, const t3b_model_desc * desc) {
    if (!desc || !desc->tensors) { set_err(nullptr, "t3b_create: null descriptor"); return nullptr; }
    const t3b_hparams & hp = desc->hp;
    if (hp.n_embd != 1024 && (hp.n_embd % 256 != 0)) { set_err(nullptr, "t3b_create: n_embd %d unsupported", hp.n_embd); return nullptr; }
    if (hp.n_head <= 0 || hp.n_embd / hp.n_head != T3B_HD) { set_err(nullptr, "t3b_create: head dim must be 64"); return nullptr; }
    if (hp.n_speech_vocab > T3B_SAMPLER_VMAX) { set_err(nullptr, "t3b_create: speech vocab %d > %d", hp.n_speech_vocab, T3B_SAMPLER_VMAX); return nullptr; }
    if (cudaSetDevice(device) != cudaSuccess) { set_err(nullptr, "t3b_create: cudaSetDevice(%d) failed", device); return nullptr; }
    t3b_ctx * ctx = new t3b_ctx();
    ctx->device = device;
    ctx->hp = hp;
    ctx->L.resize(hp.n_layer);
    auto fail = [&](const char * why) -> t3b_ctx * {
        g_err = std::string("t3b_create: ") + why + (ctx->err.empty() ? "" : (": " + ctx->err));
        for (void * p : ctx->allocs) cudaFree(p);
        if (ctx->st) cudaStreamDestroy(ctx->st);
        delete ctx;
        return nullptr;
    };
    if (cudaStreamCreateWithFlags(&ctx->st, cudaStreamNonBlocking) != cudaSuccess) return fail("stream");
    cudaEventCreate(&ctx->ev0); cudaEventCreate(&ctx->ev1);
    if (fix_table(device, &ctx->fx, &ctx->err) != T3B_OK) return fail("exp table");
    if (cudaFuncSetAttribute(sampler_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, T3B_SAMPLER_SMEM) != cudaSuccess)
        return fail("sampler shared memory attribute");
    if (cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, T3B_PREFILL_SMEM) != cudaSuccess)
        return fail("prefill attention shared memory attribute");
    if (dalloc(ctx, ctx->allocs, &ctx->err_word, 1) != T3B_OK) return fail("alloc");
    cudaMemset(ctx->err_word, 0, sizeof(unsigned));
    if (cudaHostAlloc((void **) &ctx->err_pin, sizeof(unsigned), cudaHostAllocDefault) != cudaSuccess) return fail("alloc");
    *ctx->err_pin = 0u;

    const int D = hp.n_embd;
    auto upload = [&](const t3b_tensor & t, size_t bytes, void ** dst) -> int {
        void * p = nullptr;
        if (cudaMalloc(&p, bytes) != cudaSuccess) { ctx->err = "cudaMalloc failed"; return T3B_ERR_OOM; }
        ctx->allocs.push_back(p);
        if (cudaMemcpy(p, t.data, bytes, cudaMemcpyHostToDevice) != cudaSuccess) { ctx->err = "upload failed"; return T3B_ERR_CUDA; }
        *dst = p;
        return T3B_OK;
    };
    auto nelem = [](const t3b_tensor & t) { int64_t n = 1; for (int i = 0; i < t.n_dims; ++i) n *= t.ne[i]; return n; };
    auto f32 = [&](const t3b_tensor & t, float ** dst, int64_t want) -> int {
        if (t.type != T3B_F32) { ctx->err = std::string(t.name) + ": expected F32"; return T3B_ERR_ARG; }
        if (want >= 0 && nelem(t) != want) { ctx->err = std::string(t.name) + ": wrong size"; return T3B_ERR_ARG; }
        return upload(t, (size_t) nelem(t) * 4, (void **) dst);
    };
    auto mat = [&](const t3b_tensor & t, Mat * m, int K, int N) -> int {
        if (t.type != T3B_Q4_0 && t.type != T3B_Q8_0 && t.type != T3B_F16) { ctx->err = std::string(t.name) + ": unsupported weight type"; return T3B_ERR_ARG; }
        if (t.ne[0] != K || t.ne[1] != N) { ctx->err = std::string(t.name) + ": wrong shape"; return T3B_ERR_ARG; }
        m->type = t.type; m->N = N; m->K = K; m->rb = (int) row_bytes(t.type, K);
        std::vector<uint8_t> tmp((size_t) m->rb * N);
        repack_rows(t.type, (const uint8_t *) t.data, N, K, tmp.data());
        void * p = nullptr;
        if (cudaMalloc(&p, tmp.size()) != cudaSuccess) { ctx->err = "cudaMalloc failed"; return T3B_ERR_OOM; }
        ctx->allocs.push_back(p);
        if (cudaMemcpy(p, tmp.data(), tmp.size(), cudaMemcpyHostToDevice) != cudaSuccess) { ctx->err = "upload failed"; return T3B_ERR_CUDA; }
        m->p = (uint8_t *) p;
        return T3B_OK;
    };
    int rc = T3B_OK;
    int found = 0;
    for (int i = 0; i < desc->n_tensors && rc == T3B_OK; ++i) {
        const t3b_tensor & t = desc->tensors[i];
        const std::string s(t.name ? t.name : "");
        ++found;
        if (s == "model/wpe") rc = f32(t, &ctx->wpe, (int64_t) D * hp.n_ctx);
        else if (s == "model/ln_f/g") rc = f32(t, &ctx->lnf_g, D);
        else if (s == "model/ln_f/b") rc = f32(t, &ctx->lnf_b, D);
        else if (s == "chatterbox/speech_head_bias") rc = f32(t, &ctx->head_b, hp.n_speech_vocab);
        else if (s == "chatterbox/cond_spkr/w") rc = f32(t, &ctx->spkr_w, (int64_t) D * hp.speaker_embed_size);
        else if (s == "chatterbox/cond_spkr/b") rc = f32(t, &ctx->spkr_b, D);
        else if (s == "chatterbox/builtin/speaker_emb") rc = f32(t, &ctx->builtin_spk, hp.speaker_embed_size);
        else if (s == "chatterbox/builtin/cond_prompt_speech_tokens") {
            const int64_t n = nelem(t);
            ctx->builtin_cond.assign((const int32_t *) t.data, (const int32_t *) t.data + n);
        } else if (s == "chatterbox/speech_emb" || s == "chatterbox/text_emb") {
            if (t.type != T3B_F16 || t.ne[0] != D) { ctx->err = s + ": expected F16 [n_embd, vocab]"; rc = T3B_ERR_ARG; break; }
            rc = upload(t, (size_t) nelem(t) * 2, (void **) (s == "chatterbox/speech_emb" ? &ctx->semb : &ctx->temb));
        } else if (s == "chatterbox/speech_head") rc = mat(t, &ctx->head, D, hp.n_speech_vocab);
        else {
            int il = -1; char rest[128] = {0};
            if (std::sscanf(s.c_str(), "model/h%d/%127s", &il, rest) == 2 && il >= 0 && il < hp.n_layer) {
                Layer & Ly = ctx->L[il];
                const std::string r(rest);
                if (r == "ln_1/g") rc = f32(t, &Ly.ln1g, D);
                else if (r == "ln_1/b") rc = f32(t, &Ly.ln1b, D);
                else if (r == "ln_2/g") rc = f32(t, &Ly.ln2g, D);
                else if (r == "ln_2/b") rc = f32(t, &Ly.ln2b, D);
                else if (r == "attn/c_attn/w") rc = mat(t, &Ly.attn, D, 3 * D);
                else if (r == "attn/c_attn/b") rc = f32(t, &Ly.attn_b, 3 * D);
                else if (r == "attn/c_proj/w") rc = mat(t, &Ly.proj, D, D);
                else if (r == "attn/c_proj/b") rc = f32(t, &Ly.proj_b, D);
                else if (r == "mlp/c_fc/w") rc = mat(t, &Ly.fc, D, 4 * D);
                else if (r == "mlp/c_fc/b") rc = f32(t, &Ly.fc_b, 4 * D);
                else if (r == "mlp/c_proj/w") rc = mat(t, &Ly.fc2, 4 * D, D);
                else if (r == "mlp/c_proj/b") rc = f32(t, &Ly.fc2_b, D);
                else --found;
            } else {
                --found;   // tensors outside the T3 decode path (voice encoder, ...)
            }
        }
    }
    if (rc != T3B_OK) return fail("tensor upload");
    // every tensor the path needs must be present (require_tensor, main.cpp:389-417)
    if (!ctx->wpe || !ctx->lnf_g || !ctx->lnf_b || !ctx->semb || !ctx->temb || !ctx->head.p || !ctx->head_b ||
        !ctx->spkr_w || !ctx->spkr_b)
        return fail("missing global tensor");
    for (int il = 0; il < hp.n_layer; ++il) {
        const Layer & Ly = ctx->L[il];
        if (!Ly.ln1g || !Ly.ln1b || !Ly.ln2g || !Ly.ln2b || !Ly.attn.p || !Ly.attn_b || !Ly.proj.p || !Ly.proj_b ||
            !Ly.fc.p || !Ly.fc_b || !Ly.fc2.p || !Ly.fc2_b) {
            set_err(&ctx->err, "layer %d incomplete", il);
            return fail("missing layer tensor");
        }
    }
    (void) found;
    return ctx;
}

void t3b_destroy(t3b_ctx * ctx) {
    if (!ctx) return;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->st);
    free_streams(ctx);
    if (ctx->trace) cudaFree(ctx->trace);
    if (ctx->htrace) cudaFree(ctx->htrace);
    if (ctx->hand_ev) cudaEventDestroy(ctx->hand_ev);
    for (cudaEvent_t e : ctx->q_ev) if (e) cudaEventDestroy(e);
    for (void * p : ctx->allocs) cudaFree(p);
    if (ctx->ev0) cudaEventDestroy(ctx->ev0);
    if (ctx->ev1) cudaEventDestroy(ctx->ev1);
    if (ctx->err_pin) cudaFreeHost(ctx->err_pin);
    if (ctx->io_pin) cudaFreeHost(ctx->io_pin);
    if (ctx->st) cudaStreamDestroy(ctx->st);
    delete ctx;
}

void t3b_cancel(t3b_ctx * ctx) {
    if (!ctx) return;
    ctx->cancel = 1;
    if (ctx->mega.cancel_host) *(volatile int *) ctx->mega.cancel_host = 1;
}
float t3b_last_device_ms(const t3b_ctx * ctx) { return ctx ? ctx->last_ms : 0.0f; }
void * t3b_stream_handle(const t3b_ctx * ctx) { return ctx ? (void *) ctx->st : nullptr; }

int t3b_trace_logits(t3b_ctx * ctx, int max_steps) {
    if (!ctx || max_steps < 0) return T3B_ERR_ARG;
    CK(cudaSetDevice(ctx->device));
    if (ctx->trace) { CK(cudaFree(ctx->trace)); ctx->trace = nullptr; ctx->trace_cap = 0; }
    if (max_steps > 0) {
        CK(cudaMalloc(&ctx->trace, sizeof(float) * (size_t) (max_steps + 1) * ctx->hp.n_speech_vocab));
        ctx->trace_cap = max_steps;
    }
    return T3B_OK;
}

int t3b_trace_hidden(t3b_ctx * ctx, int on) {
    if (!ctx) return T3B_ERR_ARG;
    CK(cudaSetDevice(ctx->device));
    CK(cudaStreamSynchronize(ctx->st));
    if (ctx->htrace && !on) { CK(cudaFree(ctx->htrace)); ctx->htrace = nullptr; }
    if (!ctx->htrace && on) {
        const size_t n = (size_t) (ctx->hp.n_layer + 1) * ctx->hp.n_embd;
        CK(cudaMalloc(&ctx->htrace, sizeof(float) * n));
        CK(cudaMemset(ctx->htrace, 0, sizeof(float) * n));
    }
    return T3B_OK;
}

int t3b_get_hidden_trace(t3b_ctx * ctx, float * out) {
    if (!ctx || !out || !ctx->htrace) {
        if (ctx) set_err(&ctx->err, "t3b_get_hidden_trace: tracing is off");
        return T3B_ERR_ARG;
    }
    CK(cudaSetDevice(ctx->device));
    CK(cudaStreamSynchronize(ctx->st));
    CK(cudaMemcpy(out, ctx->htrace, sizeof(float) * (size_t) (ctx->hp.n_layer + 1) * ctx->hp.n_embd,
                  cudaMemcpyDeviceToHost));
    return T3B_OK;
}

int t3b_set_wait_limit(t3b_ctx * ctx, unsigned polls) {
    if (!ctx) return T3B_ERR_ARG;
    ctx->wait_limit = polls;
    return T3B_OK;
}

unsigned long long t3b_launch_count(const t3b_ctx * ctx) { return ctx ? ctx->launches : 0ull; }

int t3b_get_logits_trace(t3b_ctx * ctx, float * out, int n) {
    if (!ctx || !out || n < 0 || n > ctx->trace_cap + 1 || !ctx->trace) {
        if (ctx) set_err(&ctx->err, "t3b_get_logits_trace: bad args or tracing off");
        return T3B_ERR_ARG;
    }
    CK(cudaSetDevice(ctx->device));
    CK(cudaMemcpy(out, ctx->trace, sizeof(float) * (size_t) n * ctx->hp.n_speech_vocab, cudaMemcpyDeviceToHost));
    return T3B_OK;
}

int t3b_stream_alloc(t3b_ctx * ctx, int n_streams, int max_ctx, int cfg) {
    if (!ctx) return T3B_ERR_ARG;
    if (n_streams <= 0 || max_ctx <= 1) { set_err(&ctx->err, "t3b_stream_alloc: bad sizes"); return T3B_ERR_ARG; }
    if (max_ctx > ctx->hp.n_ctx) max_ctx = ctx->hp.n_ctx;
    CK(cudaSetDevice(ctx->device));
    CK(cudaStreamSynchronize(ctx->st));
    free_streams(ctx);
    const int D = ctx->hp.n_embd, H = ctx->hp.n_head, V = ctx->hp.n_speech_vocab;
    ctx->S = n_streams; ctx->rps = cfg ? 2 : 1; ctx->max_ctx = max_ctx;
    ctx->params_last.clear();
    ctx->hist_cap = max_ctx;
    ctx->s_max = (max_ctx + T3B_ATTN_CHUNK - 1) / T3B_ATTN_CHUNK;
    const int rows = n_streams * ctx->rps;
    ctx->row_elems = (size_t) ctx->hp.n_layer * 2 * H * max_ctx * T3B_HD;
    const int R = std::max(rows, 512);
    ctx->R = R;
    int rc = T3B_OK;
    auto A = [&](auto ** p, size_t n) { if (rc == T3B_OK) rc = dalloc(ctx, ctx->sallocs, p, n); };
    A(&ctx->kv, ctx->row_elems * rows);
    A(&ctx->hist, (size_t) n_streams * ctx->hist_cap);
    A(&ctx->hist_len, n_streams); A(&ctx->rng_mode, n_streams); A(&ctx->done, n_streams); A(&ctx->step_tok, n_streams);
    A(&ctx->mt, (size_t) n_streams * 625); A(&ctx->ph_seed, n_streams); A(&ctx->ph_ctr, n_streams);
    A(&ctx->params, n_streams); A(&ctx->tok_out, n_streams); A(&ctx->slot_list, n_streams);
    A(&ctx->x, (size_t) R * D); A(&ctx->qkv, (size_t) R * 3 * D); A(&ctx->attn, (size_t) R * D); A(&ctx->h, (size_t) R * 4 * D);
    A(&ctx->logits, (size_t) rows * V); A(&ctx->spk, D);
    A(&ctx->xq, (size_t) R * 4 * D); A(&ctx->xd, (size_t) R * 4 * D / 32); A(&ctx->xs, (size_t) R * 4 * D / 32); A(&ctx->xh, (size_t) R * 4 * D);
    A(&ctx->xq2, (size_t) R * 4 * D); A(&ctx->xd2, (size_t) R * 4 * D / 32); A(&ctx->xs2, (size_t) R * 4 * D / 32);
    A(&ctx->part, (size_t) R * H * ctx->s_max * (T3B_HD + 2)); A(&ctx->cnt, (size_t) R * H);
    A(&ctx->row_slot, R); A(&ctx->pos, R); A(&ctx->row_of, R); A(&ctx->y_row, R);
    ctx->gws.cap = (size_t) R * 4 * D * 4;   // four splits of an R x 4096 output
    A(&ctx->gws.ws, ctx->gws.cap); A(&ctx->gws.cnt, TF_CNT);
    ctx->gws.ccap = TF_CNT;
    A(&ctx->pk_kind, R); A(&ctx->pk_id, R);
    if (rc != T3B_OK) { free_streams(ctx); return rc; }
    CK(cudaMemsetAsync(ctx->cnt, 0, sizeof(unsigned) * R * H, ctx->st));
    CK(cudaMemsetAsync(ctx->gws.cnt, 0, sizeof(unsigned) * TF_CNT, ctx->st));
    CK(cudaMemsetAsync(ctx->hist_len, 0, sizeof(int) * n_streams, ctx->st));
    CK(cudaMemsetAsync(ctx->done, 0, sizeof(int) * n_streams, ctx->st));
    CK(cudaMemsetAsync(ctx->step_tok, 0, sizeof(int) * n_streams, ctx->st));
    CK(cudaMemsetAsync(ctx->ph_ctr, 0, sizeof(unsigned long long) * n_streams, ctx->st));
    CK(cudaMemsetAsync(ctx->ph_seed, 0, sizeof(unsigned long long) * n_streams, ctx->st));
    CK(cudaMemsetAsync(ctx->kv, 0, sizeof(__half) * ctx->row_elems * rows, ctx->st));
    ctx->pos_host.assign(rows, 0);
    ctx->rng_mode_host.assign(n_streams, T3B_RNG_MT19937);
    ctx->serve = serve_create();
    // default RNG: std::mt19937 with its default seed 5489, like a
    // default-constructed engine
    for (int s = 0; s < n_streams && rc == T3B_OK; ++s) rc = t3b_set_rng(ctx, s, T3B_RNG_MT19937, 5489u, 0);
    CK(cudaStreamSynchronize(ctx->st));
    return rc;
}

int t3b_set_rng(t3b_ctx * ctx, int stream, int mode, uint64_t seed, uint64_t discard) {
    if (!ctx || stream < 0 || stream >= ctx->S) { if (ctx) set_err(&ctx->err, "t3b_set_rng: bad stream"); return T3B_ERR_ARG; }
    CK(cudaSetDevice(ctx->device));
    ctx->rng_mode_host[stream] = mode;
    CK(cudaMemcpyAsync(ctx->rng_mode + stream, &ctx->rng_mode_host[stream], sizeof(int), cudaMemcpyHostToDevice, ctx->st));
    if (mode == T3B_RNG_MT19937) {
        std::mt19937 g((uint32_t) seed);
        g.discard(discard);
        std::stringstream ss;
        ss << g;
        std::vector<uint32_t> w(625);
        for (int i = 0; i < 625; ++i) { unsigned long v; ss >> v; w[i] = (uint32_t) v; }
        return t3b_set_rng_state(ctx, stream, w.data());
    } else if (mode == T3B_RNG_PHILOX) {
        unsigned long long sd = seed, ct = discard;
        CK(cudaMemcpyAsync(ctx->ph_seed + stream, &sd, 8, cudaMemcpyHostToDevice, ctx->st));
        CK(cudaMemcpyAsync(ctx->ph_ctr + stream, &ct, 8, cudaMemcpyHostToDevice, ctx->st));
        CK(cudaStreamSynchronize(ctx->st));
        return T3B_OK;
    }
    set_err(&ctx->err, "t3b_set_rng: unknown mode %d", mode);
    return T3B_ERR_ARG;
}

int t3b_set_rng_state(t3b_ctx * ctx, int stream, const uint32_t * words625) {
    if (!ctx || stream < 0 || stream >= ctx->S || !words625) { if (ctx) set_err(&ctx->err, "t3b_set_rng_state: bad args"); return T3B_ERR_ARG; }
    if (words625[624] > 624u) { set_err(&ctx->err, "t3b_set_rng_state: index %u > 624", words625[624]); return T3B_ERR_ARG; }
    CK(cudaSetDevice(ctx->device));
    ctx->rng_mode_host[stream] = T3B_RNG_MT19937;
    CK(cudaMemcpyAsync(ctx->rng_mode + stream, &ctx->rng_mode_host[stream], sizeof(int), cudaMemcpyHostToDevice, ctx->st));
    CK(cudaMemcpyAsync(ctx->mt + (size_t) stream * 625, words625, 625 * 4, cudaMemcpyHostToDevice, ctx->st));
    CK(cudaStreamSynchronize(ctx->st));
    return T3B_OK;
}

int t3b_get_rng_state(t3b_ctx * ctx, int stream, uint32_t * words625) {
    if (!ctx || stream < 0 || stream >= ctx->S || !words625) { if (ctx) set_err(&ctx->err, "t3b_get_rng_state: bad args"); return T3B_ERR_ARG; }
    CK(cudaSetDevice(ctx->device));
    CK(cudaMemcpyAsync(words625, ctx->mt + (size_t) stream * 625, 625 * 4, cudaMemcpyDeviceToHost, ctx->st));
    CK(cudaStreamSynchronize(ctx->st));
    return T3B_OK;
}

int t3b_set_history(t3b_ctx * ctx, int stream, const int32_t * tokens, int n) {
    if (!ctx || stream < 0 || stream >= ctx->S || n < 0 || (n > 0 && !tokens)) { if (ctx) set_err(&ctx->err, "t3b_set_history: bad args"); return T3B_ERR_ARG; }
    if (n > ctx->hist_cap) { set_err(&ctx->err, "t3b_set_history: %d tokens > capacity %d", n, ctx->hist_cap); return T3B_ERR_ARG; }
    CK(cudaSetDevice(ctx->device));
    if (n) CK(cudaMemcpyAsync(ctx->hist + (size_t) stream * ctx->hist_cap, tokens, sizeof(int) * n, cudaMemcpyHostToDevice, ctx->st));
    CK(cudaMemcpyAsync(ctx->hist_len + stream, &n, sizeof(int), cudaMemcpyHostToDevice, ctx->st));
    CK(cudaStreamSynchronize(ctx->st));
    return T3B_OK;
}

int t3b_prefill(t3b_ctx * ctx, int stream, const int32_t * text, int n_text, const int32_t * cond_tokens, int n_cond,
                const float * spk_emb, float * logits_out, int32_t * prompt_len) {
    if (!ctx) return T3B_ERR_ARG;
    if (ctx->S == 0) { set_err(&ctx->err, "t3b_prefill: no streams allocated"); return T3B_ERR_STATE; }
    if (stream < 0 || stream >= ctx->S || n_text < 0 || (n_text > 0 && !text)) { set_err(&ctx->err, "t3b_prefill: bad args"); return T3B_ERR_ARG; }
    if (!cond_tokens) { cond_tokens = ctx->builtin_cond.data(); n_cond = (int) ctx->builtin_cond.size(); }
    const int P = 1 + n_cond + n_text + 1;
    if (P > ctx->max_ctx) { set_err(&ctx->err, "t3b_prefill: prompt %d exceeds context %d", P, ctx->max_ctx); return T3B_ERR_ARG; }
    for (int i = 0; i < n_text; ++i)
        if (text[i] < 0 || text[i] >= ctx->hp.n_text_vocab) { set_err(&ctx->err, "t3b_prefill: text token %d out of range", text[i]); return T3B_ERR_ARG; }
    for (int i = 0; i < n_cond; ++i)
        if (cond_tokens[i] < 0 || cond_tokens[i] >= ctx->hp.n_speech_vocab) { set_err(&ctx->err, "t3b_prefill: cond token %d out of range", cond_tokens[i]); return T3B_ERR_ARG; }
    CK(cudaSetDevice(ctx->device));
    const int D = ctx->hp.n_embd, V = ctx->hp.n_speech_vocab;
    cudaStream_t st = ctx->st;
    // speaker projection (main.cpp:603)
    const float * spk_src = ctx->builtin_spk;
    if (spk_emb) {
        CK(cudaMemcpyAsync(ctx->h, spk_emb, sizeof(float) * ctx->hp.speaker_embed_size, cudaMemcpyHostToDevice, st));
        spk_src = ctx->h;
    }
    matvec_f32_kernel<<<(D + 7) / 8, 256, 0, st>>>(ctx->spkr_w, D, ctx->hp.speaker_embed_size, spk_src, ctx->spkr_b, ctx->spk);
    std::vector<int> kind(P), id(P);
    kind[0] = 0; id[0] = 0;
    for (int i = 0; i < n_cond; ++i) { kind[1 + i] = 1; id[1 + i] = cond_tokens[i]; }
    for (int i = 0; i < n_text; ++i) { kind[1 + n_cond + i] = 2; id[1 + n_cond + i] = text[i]; }
    kind[P - 1] = 1; id[P - 1] = ctx->hp.start_speech_token;
    const int CH = ctx->R;   // rows per prefill chunk
    for (int j = 0; j < ctx->rps; ++j) {
        const int crow = stream * ctx->rps + j;
        std::vector<int> kj(kind);
        if (j == 1) for (int i = 0; i < n_text; ++i) kj[1 + n_cond + i] = 3;   // uncond: zeroed text
        for (int c0 = 0; c0 < P; c0 += CH) {
            const int n = std::min(CH, P - c0);
            std::vector<int> rowof(n, crow), pos(n);
            for (int i = 0; i < n; ++i) pos[i] = c0 + i;
            CK(cudaMemcpyAsync(ctx->pk_kind, kj.data() + c0, sizeof(int) * n, cudaMemcpyHostToDevice, st));
            CK(cudaMemcpyAsync(ctx->pk_id, id.data() + c0, sizeof(int) * n, cudaMemcpyHostToDevice, st));
            ctx->maps_slots.clear();
            CK(cudaMemcpyAsync(ctx->row_of, rowof.data(), sizeof(int) * n, cudaMemcpyHostToDevice, st));
            CK(cudaMemcpyAsync(ctx->pos, pos.data(), sizeof(int) * n, cudaMemcpyHostToDevice, st));
            embed_prompt_kernel<<<n, 256, 0, st>>>(ctx->semb, ctx->temb, ctx->wpe, ctx->spk, ctx->pk_kind, ctx->pk_id, c0, D, ctx->x);
            const bool last = c0 + n == P;
            run_layers(ctx, n, ctx->row_of, ctx->pos, n - 1, last ? 1 : 0, ctx->logits + (size_t) crow * V, nullptr, st,
                       nullptr, true);
            CK(cudaStreamSynchronize(st));   // host vectors above are reused per chunk
        }
        ctx->pos_host[crow] = P;
    }
    CK(cudaGetLastError());
    int rc = check_dev_err(ctx);
    if (rc != T3B_OK) return rc;
    // a fresh utterance: empty history, not done (run_t3: generated.clear())
    const int zero = 0;
    CK(cudaMemcpyAsync(ctx->hist_len + stream, &zero, sizeof(int), cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(ctx->done + stream, &zero, sizeof(int), cudaMemcpyHostToDevice, st));
    if (logits_out) CK(cudaMemcpyAsync(logits_out, ctx->logits + (size_t) stream * ctx->rps * V, sizeof(float) * ctx->rps * V, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (prompt_len) *prompt_len = P;
    return T3B_OK;
}

}  // extern "C"

namespace {

// Records (or reuses) a CUDA graph of one decode step over n streams:
// embed, all layers, head, and (sample) the sampler + position advance.  The
// graph reads its row maps (row_slot, row_of, slot_list), tokens and
// positions from device buffers, so one graph serves any n streams;
// upload_maps() fills the maps before a launch.
// Pinned staging area of at least `floats` floats (nullptr if it cannot be had: the caller copies directly).
float * io_pinned(t3b_ctx * ctx, size_t floats) {
    if (ctx->io_pin_cap < floats) {
        if (ctx->io_pin) cudaFreeHost(ctx->io_pin);
        ctx->io_pin = nullptr; ctx->io_pin_cap = 0;
        if (cudaHostAlloc((void **) &ctx->io_pin, floats * sizeof(float), cudaHostAllocDefault) != cudaSuccess) {
            cudaGetLastError();
            ctx->io_pin = nullptr;
            return nullptr;
        }
        ctx->io_pin_cap = floats;
    }
    return ctx->io_pin;
}

int upload_maps(t3b_ctx * ctx, const std::vector<int> & slots) {
    if (!ctx->maps_slots.empty() && ctx->maps_slots == slots) return T3B_OK;   // already on the device
    const int n = (int) slots.size(), M = n * ctx->rps;
    std::vector<int> row_slot(M), row_of(M);
    for (int i = 0; i < n; ++i)
        for (int j = 0; j < ctx->rps; ++j) {
            row_slot[i * ctx->rps + j] = slots[i];
            row_of[i * ctx->rps + j] = slots[i] * ctx->rps + j;
        }
    CK(cudaMemcpyAsync(ctx->row_slot, row_slot.data(), sizeof(int) * M, cudaMemcpyHostToDevice, ctx->st));
    CK(cudaMemcpyAsync(ctx->row_of, row_of.data(), sizeof(int) * M, cudaMemcpyHostToDevice, ctx->st));
    CK(cudaMemcpyAsync(ctx->slot_list, slots.data(), sizeof(int) * n, cudaMemcpyHostToDevice, ctx->st));
    CK(cudaStreamSynchronize(ctx->st));
    ctx->maps_slots = slots;
    return T3B_OK;
}

// Threads of a sampler CTA: a lone row finishes sooner with 512 (fewer warps
// at every barrier; measured 37 vs 41 us per configs[0] row), many rows keep
// 1024 (the element-wise passes of each row are then shorter).
inline int sampler_threads(int rows) { return rows == 1 ? 512 : T3B_SAMPLER_THREADS; }

SampArgs sampler_args(t3b_ctx * ctx, bool with_done) {
    const int V = ctx->hp.n_speech_vocab;
    SampArgs a{};
    a.cond = ctx->logits; a.cond_stride = (long long) ctx->rps * V;
    a.uncond = ctx->rps == 2 ? ctx->logits + V : nullptr; a.uncond_stride = (long long) ctx->rps * V;
    a.V = V; a.slot_of = ctx->slot_list;
    a.hist = ctx->hist; a.hist_stride = ctx->hist_cap; a.hist_len = ctx->hist_len; a.hist_append = 1;
    a.params = ctx->params; a.params_per_row = 1;
    a.rng_mode = ctx->rng_mode; a.mt = ctx->mt; a.ph_seed = ctx->ph_seed; a.ph_ctr = ctx->ph_ctr;
    a.tok_out = ctx->tok_out; a.step_tok = ctx->step_tok; a.done = with_done ? ctx->done : nullptr;
    a.stop_token = ctx->hp.stop_speech_token;
    a.fx = ctx->fx;
    return a;
}

int ensure_graph(t3b_ctx * ctx, int n, bool sample, StepGraph ** out) {
    std::vector<int> key{n, sample ? 1 : 0, ctx->htrace ? 1 : 0};
    auto it = ctx->graphs.find(key);
    if (it != ctx->graphs.end()) { *out = &it->second; return T3B_OK; }
    const int M = n * ctx->rps;
    const int V = ctx->hp.n_speech_vocab;
    StepGraph sg;
    cudaStream_t st = ctx->st;
    CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
    embed_step_kernel<<<M, 256, 0, st>>>(ctx->semb, ctx->wpe, ctx->step_tok, ctx->row_slot, ctx->pos,
                                         ctx->hp.n_embd, V, ctx->hp.n_ctx, ctx->x, ctx->err_word);
    run_layers(ctx, M, ctx->row_of, ctx->pos, 0, M, ctx->logits, ctx->row_of, st, ctx->htrace);
    if (sample) {
        SampArgs a = sampler_args(ctx, true);
        sampler_kernel<<<n, sampler_threads(n), T3B_SAMPLER_SMEM, st>>>(a);
        advance_pos_kernel<<<(M + 127) / 128, 128, 0, st>>>(ctx->pos, M);
    }
    cudaError_t ce = cudaStreamEndCapture(st, &sg.g);
    if (ce != cudaSuccess) { set_err(&ctx->err, "graph capture: %s", cudaGetErrorString(ce)); return T3B_ERR_CUDA; }
    CK(cudaGraphInstantiate(&sg.ge, sg.g, 0));
    size_t nn = 0;
    CK(cudaGraphGetNodes(sg.g, nullptr, &nn));
    std::vector<cudaGraphNode_t> nodes(nn);
    if (nn) CK(cudaGraphGetNodes(sg.g, nodes.data(), &nn));
    for (cudaGraphNode_t nd : nodes) {
        cudaGraphNodeType ty;
        CK(cudaGraphNodeGetType(nd, &ty));
        sg.n_kernels += ty == cudaGraphNodeTypeKernel;
    }
    auto res = ctx->graphs.emplace(key, sg);
    *out = &res.first->second;
    return T3B_OK;
}


// Persistent batch-1 decode (megakernel.cuh).  Eligible when one stream
// without CFG decodes a T3 with n_embd 1024 / 16 heads and every layer matrix
// in one of Q4_0 / Q8_0 / F16, at any position of the cache (contexts longer
// than MK_MAX_POS stream their K/V in tiles).  The CTA count is the SM count;
// each CTA's row slices must fit its registers.
bool mega_eligible(t3b_ctx * ctx, int n, int max_pos_after) {
    if (getenv("T3B_NO_MEGAKERNEL")) return false;
    if (n != 1 || ctx->rps != 1) return false;
    if (ctx->hp.n_embd != 1024 || ctx->hp.n_head != 16) return false;
    if (ctx->hp.n_speech_vocab > T3B_SAMPLER_VMAX) return false;
    if (max_pos_after > ctx->max_ctx) return false;   // longer than MK_MAX_POS: K/V streamed in tiles
    const int T = ctx->L[0].attn.type;
    for (const Layer & Ly : ctx->L)
        if (Ly.attn.type != T || Ly.proj.type != T || Ly.fc.type != T || Ly.fc2.type != T) return false;
    return T == T3B_Q4_0 || T == T3B_Q8_0 || T == T3B_F16;
}

const void * mega_fn(int T, bool lng) {
    if (lng)
        return T == T3B_Q4_0 ? (const void *) t3_decode_megakernel<T3B_Q4_0, true>
             : T == T3B_Q8_0 ? (const void *) t3_decode_megakernel<T3B_Q8_0, true>
                             : (const void *) t3_decode_megakernel<T3B_F16, true>;
    return T == T3B_Q4_0 ? (const void *) t3_decode_megakernel<T3B_Q4_0, false>
         : T == T3B_Q8_0 ? (const void *) t3_decode_megakernel<T3B_Q8_0, false>
                         : (const void *) t3_decode_megakernel<T3B_F16, false>;
}

int mega_prepare(t3b_ctx * ctx) {
    MegaState & m = ctx->mega;
    if (m.ready) return T3B_OK;
    int sms = 0;
    CK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device));
    const int G = sms;
    auto cdiv = [](int a, int b) { return (a + b - 1) / b; };
    // per-CTA limits of the register prefetch (MK_MAXI items of 32 elements
    // per thread) and of the row scratch.  Q4_0 layers: CTAs 1..16 run the
    // attention and the other GW = G - 16 share fc and fc2 (fc in whole
    // 32-row blocks); Q8_0: fc in blocks over all G; F16: plain row split.
    const int LT = ctx->L[0].fc.type;
    const int GW = LT == T3B_Q4_0 ? G - 16 : G;
    const int fc_items = LT == T3B_F16 ? cdiv(4 * 1024, GW) * 32 : cdiv(128, GW) * 32 * 32;
    if (G < 17 || GW < 1 || cdiv(3 * 1024, G) * 32 > MK_MAXI * MK_THREADS || fc_items > MK_MAXI * MK_THREADS ||
        cdiv(1024, GW) * 128 > MK_MAXI * MK_THREADS || cdiv(ctx->hp.n_speech_vocab, G) * 32 > MK_MAXI * MK_THREADS ||
        cdiv(ctx->hp.n_speech_vocab, G) > 128) {
        set_err(&ctx->err, "megakernel: %d SMs too few for the row split", G);
        return T3B_ERR_STATE;
    }
    std::vector<MkLayer> hl(ctx->hp.n_layer);
    for (int l = 0; l < ctx->hp.n_layer; ++l) {
        const Layer & Ly = ctx->L[l];
        hl[l].ln1g = Ly.ln1g; hl[l].ln1b = Ly.ln1b; hl[l].ln2g = Ly.ln2g; hl[l].ln2b = Ly.ln2b;
        hl[l].bqkv = Ly.attn_b; hl[l].bo = Ly.proj_b; hl[l].bfc = Ly.fc_b; hl[l].bfc2 = Ly.fc2_b;
        hl[l].qkv = {Ly.attn.p, Ly.attn.type, Ly.attn.rb};
        hl[l].o = {Ly.proj.p, Ly.proj.type, Ly.proj.rb};
        hl[l].fc = {Ly.fc.p, Ly.fc.type, Ly.fc.rb};
        hl[l].fc2 = {Ly.fc2.p, Ly.fc2.type, Ly.fc2.rb};
    }
    CK(cudaMalloc(&m.layers, sizeof(MkLayer) * hl.size()));
    CK(cudaMemcpy(m.layers, hl.data(), sizeof(MkLayer) * hl.size(), cudaMemcpyHostToDevice));
    CK(cudaMalloc(&m.buf, sizeof(float) * MK_B_TOTAL));
    CK(cudaMemset(m.buf, 0, sizeof(float) * MK_B_TOTAL));   // x-word tags start unused (epoch 0)
    // counters | abort flag | steps done, each on its own 128-byte line: one memset per launch
    CK(cudaMalloc(&m.cnt, sizeof(unsigned) * MK_CTL_WORDS));
    m.abort_flag = (int *) (m.cnt + MK_C_N * MK_C_STRIDE);
    m.steps_done = (int *) (m.cnt + (MK_C_N + 1) * MK_C_STRIDE);
    CK(cudaHostAlloc(&m.cancel_host, sizeof(int), cudaHostAllocMapped));
    *m.cancel_host = 0;
    CK(cudaHostGetDevicePointer(&m.cancel_dev, m.cancel_host, 0));
    m.smem = mk_smem_bytes();
    const int T = ctx->L[0].attn.type;
    for (int lg = 0; lg < 2; ++lg) {
        const void * fn = mega_fn(T, lg != 0);
        CK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) m.smem));
        int per_sm = 0;
        CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, MK_THREADS, m.smem));
        if (per_sm < 1) { set_err(&ctx->err, "megakernel: does not fit on an SM"); return T3B_ERR_STATE; }
    }
    m.grid = G;
    m.ready = 1;
    return T3B_OK;
}

// One cooperative launch decoding max_steps steps of stream `slot` (row
// slot).  The first token is already in step_tok (sampled from the prefill
// logits).  Returns the number of steps run in *steps.
int mega_decode(t3b_ctx * ctx, int slot, int p0, int max_steps, int ignore_stop, int * steps, float * logits_out = nullptr,
                int first_tok = -1) {
    MegaState & m = ctx->mega;
    cudaStream_t st = ctx->st;
    const int H = ctx->hp.n_head;
    MegaArgs a{};
    a.layers = m.layers; a.n_layer = ctx->hp.n_layer;
    a.semb = ctx->semb; a.wpe = ctx->wpe; a.lnfg = ctx->lnf_g; a.lnfb = ctx->lnf_b;
    a.head = {ctx->head.p, ctx->head.type, ctx->head.rb}; a.headb = ctx->head_b;
    a.V = ctx->hp.n_speech_vocab; a.eps = ctx->hp.eps;
    a.kv = ctx->kv + (size_t) slot * ctx->row_elems;
    a.layer_stride = (size_t) 2 * H * ctx->max_ctx * T3B_HD;
    a.v_off = (size_t) H * ctx->max_ctx * T3B_HD;
    a.max_ctx = ctx->max_ctx;
    a.p0 = p0; a.n_steps = max_steps; a.ignore_stop = ignore_stop; a.stop_token = ctx->hp.stop_speech_token;
    a.buf = m.buf; a.cnt = m.cnt; a.err = ctx->err_word; a.abort_flag = m.abort_flag; a.cancel = m.cancel_dev;
    a.steps_done = m.steps_done;
    a.trace = (logits_out == nullptr && ctx->trace_cap >= max_steps) ? ctx->trace : nullptr;
    a.logits_out = logits_out;
    a.sample = logits_out == nullptr;
    a.samp = sampler_args(ctx, false);
    a.samp.done = nullptr;
    a.first_tok = first_tok;
    a.spin = ctx->wait_limit ? ctx->wait_limit : MK_SPIN;
    a.htrace = ctx->htrace;
    m.epoch = m.epoch % 4095u + 1u;   // 1..4095, never the same as the previous launch's
    a.epoch = m.epoch;
    CK(cudaMemsetAsync(m.cnt, 0, sizeof(unsigned) * MK_CTL_WORDS, st));
    // debug: T3B_MK_TIMELINE=<file> stamps every phase boundary of step
    // T3B_MK_TIMELINE_STEP (default 2) per CTA and writes [G][MK_TL] u64 ns
    const char * tl_file = getenv("T3B_MK_TIMELINE");
    unsigned long long * tl = nullptr;
    if (tl_file) {
        CK(cudaMalloc(&tl, sizeof(unsigned long long) * m.grid * MK_TL));
        CK(cudaMemsetAsync(tl, 0, sizeof(unsigned long long) * m.grid * MK_TL, st));
        a.tl = tl;
        a.tl_step = getenv("T3B_MK_TIMELINE_STEP") ? atoi(getenv("T3B_MK_TIMELINE_STEP")) : 2;
    }
    void * args[] = {&a};
    // positions p0 .. p0 + max_steps - 1: past MK_MAX_POS only the LONG
    // instantiation streams K/V in tiles
    const void * fn = mega_fn(ctx->L[0].attn.type, p0 + max_steps > MK_MAX_POS);
    CK(cudaLaunchCooperativeKernel(fn, dim3(m.grid), dim3(MK_THREADS), args, m.smem, st));
    ctx->launches += 1;
    if (steps) CK(cudaMemcpyAsync(steps, m.steps_done, sizeof(int), cudaMemcpyDeviceToHost, st));
    if (tl) {
        std::vector<unsigned long long> h((size_t) m.grid * MK_TL);
        CK(cudaMemcpyAsync(h.data(), tl, sizeof(unsigned long long) * h.size(), cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
        if (FILE * f = fopen(tl_file, "wb")) { fwrite(h.data(), 8, h.size(), f); fclose(f); }
        cudaFree(tl);
    }
    return T3B_OK;
}

int check_streams(t3b_ctx * ctx, int n, const int32_t * streams, std::vector<int> & slots) {
    if (ctx->S == 0) { set_err(&ctx->err, "no streams allocated"); return T3B_ERR_STATE; }
    if (n <= 0 || n > ctx->S) { set_err(&ctx->err, "bad stream count %d", n); return T3B_ERR_ARG; }
    slots.resize(n);
    std::vector<char> seen(ctx->S, 0);
    for (int i = 0; i < n; ++i) {
        slots[i] = streams ? streams[i] : i;
        if (slots[i] < 0 || slots[i] >= ctx->S) { set_err(&ctx->err, "bad stream id %d", slots[i]); return T3B_ERR_ARG; }
        if (seen[slots[i]]) { set_err(&ctx->err, "stream %d listed twice", slots[i]); return T3B_ERR_ARG; }
        seen[slots[i]] = 1;
    }
    return T3B_OK;
}

}  // namespace

extern "C" {

int t3b_step(t3b_ctx * ctx, int n, const int32_t * streams, const int32_t * tokens, const int32_t * n_past,
             float * logits_out) {
    if (!ctx) return T3B_ERR_ARG;
    std::vector<int> slots;
    int rc = check_streams(ctx, n, streams, slots);
    if (rc != T3B_OK) return rc;
    if (!tokens) { set_err(&ctx->err, "t3b_step: tokens is NULL"); return T3B_ERR_ARG; }
    CK(cudaSetDevice(ctx->device));
    const int V = ctx->hp.n_speech_vocab;
    for (int i = 0; i < n; ++i) {
        if (tokens[i] < 0 || tokens[i] >= V) { set_err(&ctx->err, "t3b_step: token %d out of range", tokens[i]); return T3B_ERR_ARG; }
        const int p = n_past ? n_past[i] : ctx->pos_host[slots[i] * ctx->rps];
        if (p < 0 || p + 1 > ctx->max_ctx) { set_err(&ctx->err, "t3b_step: position %d outside context %d", p, ctx->max_ctx); return T3B_ERR_ARG; }
        for (int j = 0; j < ctx->rps; ++j) ctx->pos_host[slots[i] * ctx->rps + j] = p;
    }
    cudaStream_t st = ctx->st;
    const int p_first = ctx->pos_host[slots[0] * ctx->rps];
    if (mega_eligible(ctx, n, p_first + 1) && mega_prepare(ctx) == T3B_OK) {
        // eval_step of one stream: one persistent-kernel step, logits only
        rc = upload_maps(ctx, slots);
        if (rc != T3B_OK) return rc;
        float * dst = ctx->logits + (size_t) slots[0] * V;
        CK(cudaEventRecord(ctx->ev0, st));
        rc = mega_decode(ctx, slots[0], p_first, 1, 1, nullptr, dst, tokens[0]);
        if (rc != T3B_OK) return rc;
        CK(cudaEventRecord(ctx->ev1, st));
        float * pin = logits_out ? io_pinned(ctx, (size_t) V) : nullptr;
        if (logits_out) CK(cudaMemcpyAsync(pin ? pin : logits_out, dst, sizeof(float) * V, cudaMemcpyDeviceToHost, st));
        CK(cudaMemcpyAsync(ctx->err_pin, ctx->err_word, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
        if (pin) std::memcpy(logits_out, pin, sizeof(float) * V);
        cudaEventElapsedTime(&ctx->last_ms, ctx->ev0, ctx->ev1);
        ctx->pos_host[slots[0]] = p_first + 1;
        return *ctx->err_pin ? check_dev_err(ctx) : T3B_OK;
    }
    StepGraph * g = nullptr;
    rc = ensure_graph(ctx, n, false, &g);
    if (rc != T3B_OK) return rc;
    rc = upload_maps(ctx, slots);
    if (rc != T3B_OK) return rc;
    // step_tok is indexed by slot, pos by activation row
    std::vector<int> tok(ctx->S, 0);
    CK(cudaMemcpyAsync(tok.data(), ctx->step_tok, sizeof(int) * ctx->S, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    for (int i = 0; i < n; ++i) tok[slots[i]] = tokens[i];
    CK(cudaMemcpyAsync(ctx->step_tok, tok.data(), sizeof(int) * ctx->S, cudaMemcpyHostToDevice, st));
    std::vector<int> pos(n * ctx->rps);
    for (int i = 0; i < n; ++i) for (int j = 0; j < ctx->rps; ++j) pos[i * ctx->rps + j] = ctx->pos_host[slots[i] * ctx->rps + j];
    CK(cudaMemcpyAsync(ctx->pos, pos.data(), sizeof(int) * pos.size(), cudaMemcpyHostToDevice, st));
    CK(cudaEventRecord(ctx->ev0, st));
    CK(cudaGraphLaunch(g->ge, st));
    ctx->launches += (unsigned long long) g->n_kernels;
    CK(cudaEventRecord(ctx->ev1, st));
    if (logits_out)
        for (int i = 0; i < n; ++i)
            CK(cudaMemcpyAsync(logits_out + (size_t) i * ctx->rps * V, ctx->logits + (size_t) slots[i] * ctx->rps * V,
                               sizeof(float) * ctx->rps * V, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    cudaEventElapsedTime(&ctx->last_ms, ctx->ev0, ctx->ev1);
    for (int i = 0; i < n; ++i) for (int j = 0; j < ctx->rps; ++j) ctx->pos_host[slots[i] * ctx->rps + j] += 1;
    return check_dev_err(ctx);
}

int t3b_sample(t3b_ctx * ctx, int n, const int32_t * streams, const t3b_sample_params * params, const float * logits,
               int32_t * tokens_out) {
    if (!ctx) return T3B_ERR_ARG;
    std::vector<int> slots;
    int rc = check_streams(ctx, n, streams, slots);
    if (rc != T3B_OK) return rc;
    if (!params || !tokens_out) { set_err(&ctx->err, "t3b_sample: params/tokens_out NULL"); return T3B_ERR_ARG; }
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->st;
    const int V = ctx->hp.n_speech_vocab;
    // pinned staging: [host logits n * rps * V][tokens n]
    const size_t nl = logits ? (size_t) n * ctx->rps * V : 0;
    float * pin = io_pinned(ctx, nl + (size_t) n);
    if (logits) {
        if (pin) std::memcpy(pin, logits, sizeof(float) * nl);
        const float * srcl = pin ? pin : logits;
        for (int i = 0; i < n; ++i)
            CK(cudaMemcpyAsync(ctx->logits + (size_t) slots[i] * ctx->rps * V, srcl + (size_t) i * ctx->rps * V,
                               sizeof(float) * ctx->rps * V, cudaMemcpyHostToDevice, st));
    }
    // parameters and slot list: uploaded only when they differ from what the device holds
    if ((int) ctx->params_last.size() != n ||
        std::memcmp(ctx->params_last.data(), params, sizeof(t3b_sample_params) * n) != 0) {
        // (a pageable source is staged before the call returns)
        CK(cudaMemcpyAsync(ctx->params, params, sizeof(t3b_sample_params) * n, cudaMemcpyHostToDevice, st));
        ctx->params_last.assign(params, params + n);
    }
    if (ctx->maps_slots != slots) {
        ctx->maps_slots.clear();
        CK(cudaMemcpyAsync(ctx->slot_list, slots.data(), sizeof(int) * n, cudaMemcpyHostToDevice, st));
    }
    SampArgs a = sampler_args(ctx, false);
    CK(cudaEventRecord(ctx->ev0, st));
    sampler_kernel<<<n, sampler_threads(n), T3B_SAMPLER_SMEM, st>>>(a);
    CK(cudaGetLastError());
    ctx->launches += 1;
    CK(cudaEventRecord(ctx->ev1, st));
    int * tpin = pin ? (int *) (pin + nl) : nullptr;
    CK(cudaMemcpyAsync(tpin ? tpin : tokens_out, ctx->tok_out, sizeof(int) * n, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    if (tpin) std::memcpy(tokens_out, tpin, sizeof(int) * n);
    cudaEventElapsedTime(&ctx->last_ms, ctx->ev0, ctx->ev1);
    return T3B_OK;
}

int t3b_decode(t3b_ctx * ctx, int n, const int32_t * streams, const t3b_sample_params * params, int max_steps,
               int ignore_stop, int32_t * tokens_out, int32_t * n_out) {
    if (!ctx) return T3B_ERR_ARG;
    std::vector<int> slots;
    int rc = check_streams(ctx, n, streams, slots);
    if (rc != T3B_OK) return rc;
    if (!params || max_steps < 0) { set_err(&ctx->err, "t3b_decode: bad args"); return T3B_ERR_ARG; }
    CK(cudaSetDevice(ctx->device));
    cudaStream_t st = ctx->st;
    ctx->cancel = 0;
    if (ctx->mega.cancel_host) *(volatile int *) ctx->mega.cancel_host = 0;
    const int M = n * ctx->rps;
    // positions of every row must leave room for max_steps
    std::vector<int> pos(M);
    int max_pos = 0;
    for (int i = 0; i < n; ++i)
        for (int j = 0; j < ctx->rps; ++j) {
            pos[i * ctx->rps + j] = ctx->pos_host[slots[i] * ctx->rps + j];
            max_pos = std::max(max_pos, pos[i * ctx->rps + j]);
        }
    if (max_pos + max_steps > ctx->max_ctx) {
        set_err(&ctx->err, "t3b_decode: %d steps from position %d exceed context %d", max_steps, max_pos, ctx->max_ctx);
        return T3B_ERR_ARG;
    }
    StepGraph * g = nullptr;
    rc = ensure_graph(ctx, n, true, &g);
    if (rc != T3B_OK) return rc;
    rc = upload_maps(ctx, slots);
    if (rc != T3B_OK) return rc;
    CK(cudaMemcpyAsync(ctx->params, params, sizeof(t3b_sample_params) * n, cudaMemcpyHostToDevice, st));
    ctx->params_last.clear();
    CK(cudaMemcpyAsync(ctx->pos, pos.data(), sizeof(int) * M, cudaMemcpyHostToDevice, st));
    std::vector<int> zeros(ctx->S, 0);
    CK(cudaMemcpyAsync(ctx->done, zeros.data(), sizeof(int) * ctx->S, cudaMemcpyHostToDevice, st));
    // first token from the prefill logits (run_t3: sample before the loop)
    SampArgs a = sampler_args(ctx, !ignore_stop);
    const bool mega = mega_eligible(ctx, n, max_pos + max_steps) && mega_prepare(ctx) == T3B_OK;
    const bool trace = ctx->trace && ctx->trace_cap >= max_steps;
    const size_t Vb = sizeof(float) * ctx->hp.n_speech_vocab;
    if (trace) CK(cudaMemcpyAsync(ctx->trace, ctx->logits + (size_t) slots[0] * ctx->rps * ctx->hp.n_speech_vocab, Vb,
                                  cudaMemcpyDeviceToDevice, st));
    CK(cudaEventRecord(ctx->ev0, st));
    sampler_kernel<<<n, sampler_threads(n), T3B_SAMPLER_SMEM, st>>>(a);
    CK(cudaGetLastError());
    ctx->launches += 1;
    int steps_done = 0;
    if (mega) {
        // a stop token drawn from the prefill logits ends the loop at once
        int first_stop = 0;
        if (!ignore_stop) {
            int t0 = 0;
            CK(cudaMemcpyAsync(&t0, ctx->step_tok + slots[0], sizeof(int), cudaMemcpyDeviceToHost, st));
            CK(cudaStreamSynchronize(st));
            first_stop = t0 == ctx->hp.stop_speech_token;
        }
        int ran = 0;
        if (!first_stop && max_steps > 0) {
            rc = mega_decode(ctx, slots[0], pos[0], max_steps, ignore_stop, &ran);
            if (rc != T3B_OK) return rc;
        }
        CK(cudaEventRecord(ctx->ev1, st));
        CK(cudaStreamSynchronize(st));
        cudaEventElapsedTime(&ctx->last_ms, ctx->ev0, ctx->ev1);
        rc = check_dev_err(ctx);
        if (rc != T3B_OK) return rc;
        if (ctx->mega.cancel_host && *ctx->mega.cancel_host) {
            *ctx->mega.cancel_host = 0;
            set_err(&ctx->err, "t3b_decode: cancelled");
            return T3B_ERR_CANCELLED;
        }
        ctx->pos_host[slots[0]] = pos[0] + ran;
        std::vector<int> hl(ctx->S);
        CK(cudaMemcpy(hl.data(), ctx->hist_len, sizeof(int) * ctx->S, cudaMemcpyDeviceToHost));
        const int cnt = std::min(hl[slots[0]], max_steps + 1);
        if (tokens_out) CK(cudaMemcpy(tokens_out, ctx->hist + (size_t) slots[0] * ctx->hist_cap, sizeof(int) * cnt,
                                      cudaMemcpyDeviceToHost));
        if (n_out) n_out[0] = cnt;
        return T3B_OK;
    }
    for (int s = 0; s < max_steps; ++s) {
        // at most 16 steps queued ahead of the GPU, so that a cancel (or
        // the done flags) is seen within that many steps
        if (s > 0 && (s % 8) == 0) {
            cudaEvent_t & q = ctx->q_ev[(s / 8) & 1];
            if (!q) CK(cudaEventCreateWithFlags(&q, cudaEventDisableTiming));
            else if (s >= 16) CK(cudaEventSynchronize(q));
            CK(cudaEventRecord(q, st));
        }
        if (ctx->cancel) { set_err(&ctx->err, "t3b_decode: cancelled"); CK(cudaStreamSynchronize(st)); return T3B_ERR_CANCELLED; }
        if (!ignore_stop && s > 0 && (s % 16) == 0) {
            std::vector<int> d(ctx->S);
            CK(cudaMemcpyAsync(d.data(), ctx->done, sizeof(int) * ctx->S, cudaMemcpyDeviceToHost, st));
            CK(cudaStreamSynchronize(st));
            bool all = true;
            for (int i = 0; i < n; ++i) all = all && d[slots[i]];
            if (all) break;
        }
        CK(cudaGraphLaunch(g->ge, st));
        ctx->launches += (unsigned long long) g->n_kernels;
        if (trace)
            CK(cudaMemcpyAsync(ctx->trace + (size_t) (s + 1) * ctx->hp.n_speech_vocab,
                               ctx->logits + (size_t) slots[0] * ctx->rps * ctx->hp.n_speech_vocab, Vb,
                               cudaMemcpyDeviceToDevice, st));
        ++steps_done;
    }
    CK(cudaEventRecord(ctx->ev1, st));
    CK(cudaStreamSynchronize(st));
    cudaEventElapsedTime(&ctx->last_ms, ctx->ev0, ctx->ev1);
    rc = check_dev_err(ctx);
    if (rc != T3B_OK) return rc;
    // tokens = each stream's history; positions advanced on the device
    std::vector<int> hl(ctx->S);
    CK(cudaMemcpy(hl.data(), ctx->hist_len, sizeof(int) * ctx->S, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(pos.data(), ctx->pos, sizeof(int) * M, cudaMemcpyDeviceToHost));
    for (int i = 0; i < n; ++i) {
        const int cnt = std::min(hl[slots[i]], max_steps + 1);
        if (tokens_out)
            CK(cudaMemcpy(tokens_out + (size_t) i * (max_steps + 1), ctx->hist + (size_t) slots[i] * ctx->hist_cap,
                          sizeof(int) * cnt, cudaMemcpyDeviceToHost));
        if (n_out) n_out[i] = cnt;
        for (int j = 0; j < ctx->rps; ++j) ctx->pos_host[slots[i] * ctx->rps + j] = pos[i * ctx->rps + j];
    }
    (void) steps_done;
    return T3B_OK;
}

// S3Gen hand-off: the stream's speech tokens go from its device history
// straight into the caller's device buffer (the S3Gen input), ordered on the
// caller's stream by an event; no host round trip.
int t3b_s3gen_tokens(t3b_ctx * ctx, int stream, int32_t * tokens_dev, int cap, int32_t * n_dev, int append_silence,
                     void * consumer_stream) {
    if (!ctx) return T3B_ERR_ARG;
    if (ctx->S == 0) { set_err(&ctx->err, "t3b_s3gen_tokens: no streams allocated"); return T3B_ERR_STATE; }
    if (stream < 0 || stream >= ctx->S || !tokens_dev || !n_dev || cap < 0) {
        set_err(&ctx->err, "t3b_s3gen_tokens: bad args");
        return T3B_ERR_ARG;
    }
    CK(cudaSetDevice(ctx->device));
    if (!ctx->hand_ev) CK(cudaEventCreateWithFlags(&ctx->hand_ev, cudaEventDisableTiming));
    s3gen_tokens_kernel<<<1, 1024, 0, ctx->st>>>(ctx->hist + (size_t) stream * ctx->hist_cap, ctx->hist_len + stream,
                                                T3B_S3_VOCAB, T3B_S3_SILENCE, append_silence ? T3B_S3_LOOKAHEAD : 0,
                                                tokens_dev, cap, n_dev);
    CK(cudaGetLastError());
    CK(cudaEventRecord(ctx->hand_ev, ctx->st));
    if (consumer_stream) CK(cudaStreamWaitEvent((cudaStream_t) consumer_stream, ctx->hand_ev, 0));
    return T3B_OK;
}

}  // extern "C"

#include "serve.cuh"

extern "C" {

// ----------------------------- op-level ----------------------------------

int t3b_op_repack(int dtype, const void * gguf_rows_host, int N, int K, void * out_dev) {
    if (!gguf_rows_host || !out_dev || N <= 0 || K <= 0 || K % 32) { set_err(nullptr, "t3b_op_repack: bad args"); return T3B_ERR_ARG; }
    std::vector<uint8_t> tmp(row_bytes(dtype, K) * N);
    repack_rows(dtype, (const uint8_t *) gguf_rows_host, N, K, tmp.data());
    if (cudaMemcpy(out_dev, tmp.data(), tmp.size(), cudaMemcpyHostToDevice) != cudaSuccess) { set_err(nullptr, "t3b_op_repack: copy failed"); return T3B_ERR_CUDA; }
    return T3B_OK;
}

}  // extern "C"

namespace {
// scratch for op-level calls (per device, grown on demand)
struct OpScratch { int8_t * xq = nullptr; float * xd = nullptr; int * xs = nullptr; __half * xh = nullptr; size_t cap = 0;
                   float * part = nullptr; unsigned * cnt = nullptr; size_t pcap = 0, ccap = 0;
                   unsigned * errw = nullptr;   // device error word of the op-level attention on this device
                   GemmWs gws;                  // split-K workspace of the tensor-core F16 GEMM
                   bool pf_attr = false;        // attn_prefill_kernel's shared-memory attribute set on this device
                 };
std::mutex g_op_mu;
std::map<int, OpScratch> g_op;
}

extern "C" {

int t3b_op_gemv(int dtype, const void * w_dev, int N, int K, const float * x_dev, int M, const float * ln_g,
                const float * ln_b, float eps, const float * bias_dev, const float * residual_dev, int epilogue,
                float * y_dev, void * cuda_stream) {
    if (!w_dev || !x_dev || !y_dev || N <= 0 || K <= 0 || K % 256 || M <= 0 || epilogue < 0 || epilogue > 2 ||
        (epilogue == 2 && !residual_dev) || (dtype != T3B_Q4_0 && dtype != T3B_Q8_0 && dtype != T3B_F16)) {
        set_err(nullptr, "t3b_op_gemv: bad args");
        return T3B_ERR_ARG;
    }
    cudaStream_t st = (cudaStream_t) cuda_stream;
    int dev = 0; cudaGetDevice(&dev);
    OpScratch * sc;
    {
        std::lock_guard<std::mutex> lk(g_op_mu);
        sc = &g_op[dev];
        const size_t need = (size_t) M * K;
        if (sc->cap < need) {
            cudaFree(sc->xq); cudaFree(sc->xd); cudaFree(sc->xs); cudaFree(sc->xh);
            if (cudaMalloc(&sc->xq, need) != cudaSuccess || cudaMalloc(&sc->xd, need / 32 * 4) != cudaSuccess ||
                cudaMalloc(&sc->xs, need / 32 * 4) != cudaSuccess || cudaMalloc(&sc->xh, need * 2) != cudaSuccess) {
                sc->cap = 0; set_err(nullptr, "t3b_op_gemv: scratch allocation failed"); return T3B_ERR_OOM;
            }
            sc->cap = need;
        }
        const size_t wsn = (size_t) 8 * M * ((N + TF_BN - 1) / TF_BN * TF_BN);
        if (dtype == T3B_F16 && M >= TC_MIN_M && sc->gws.cap < wsn) {
            cudaFree(sc->gws.ws);
            if (!sc->gws.cnt) {
                if (cudaMalloc(&sc->gws.cnt, sizeof(unsigned) * TF_CNT) != cudaSuccess ||
                    cudaMemsetAsync(sc->gws.cnt, 0, sizeof(unsigned) * TF_CNT, st) != cudaSuccess) {
                    set_err(nullptr, "t3b_op_gemv: scratch allocation failed"); return T3B_ERR_OOM;
                }
                sc->gws.ccap = TF_CNT;
            }
            if (cudaMalloc(&sc->gws.ws, sizeof(float) * wsn) != cudaSuccess) {
                sc->gws.ws = nullptr; sc->gws.cap = 0; set_err(nullptr, "t3b_op_gemv: scratch allocation failed"); return T3B_ERR_OOM;
            }
            sc->gws.cap = wsn;
        }
    }
    Mat W; W.type = dtype; W.N = N; W.K = K; W.rb = (int) row_bytes(dtype, K); W.p = (uint8_t *) w_dev;
    const int kind = epilogue == 0 ? EPI_BIAS : (epilogue == 1 ? EPI_GELU : EPI_RESID);
    const GemvEpi ge = epi_plain(kind, y_dev, N, bias_dev, residual_dev, N);
    if (!launch_gemv_prep(W, x_dev, K, M, ln_g, ln_b, eps, ge, st)) {   // M <= 4: one launch
        const int qmode = dtype == T3B_F16 ? 2 : 1;
        prep_act_kernel<<<M, 256, K * sizeof(float), st>>>(x_dev, K, K, ln_g, ln_b, eps, qmode, sc->xq, sc->xd, sc->xs, sc->xh);
        launch_gemv(W, sc->xq, sc->xd, sc->xs, sc->xh, M, ge, st, &sc->gws);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_err(nullptr, "t3b_op_gemv: %s", cudaGetErrorString(e)); return T3B_ERR_CUDA; }
    return T3B_OK;
}

int t3b_op_attention(const float * q_dev, const void * k_dev, const void * v_dev, int M, int n_head, int max_ctx,
                     const int32_t * len_dev, float * out_dev, void * cuda_stream) {
    if (!q_dev || !k_dev || !v_dev || !len_dev || !out_dev || M <= 0 || n_head <= 0 || max_ctx <= 0) {
        set_err(nullptr, "t3b_op_attention: bad args");
        return T3B_ERR_ARG;
    }
    if ((((uintptr_t) k_dev) | ((uintptr_t) v_dev)) & 15) {
        set_err(nullptr, "t3b_op_attention: K and V caches must be 16-byte aligned");
        return T3B_ERR_ARG;
    }
    cudaStream_t st = (cudaStream_t) cuda_stream;
    int dev = 0; cudaGetDevice(&dev);
    const int s_max = (max_ctx + T3B_ATTN_CHUNK - 1) / T3B_ATTN_CHUNK;
    OpScratch * sc;
    {
        std::lock_guard<std::mutex> lk(g_op_mu);
        sc = &g_op[dev];
        const size_t pneed = (size_t) M * n_head * s_max * (T3B_HD + 2), cneed = (size_t) M * n_head;
        if (sc->pcap < pneed) {
            cudaFree(sc->part);
            if (cudaMalloc(&sc->part, pneed * 4) != cudaSuccess) { sc->pcap = 0; set_err(nullptr, "t3b_op_attention: scratch allocation failed"); return T3B_ERR_OOM; }
            sc->pcap = pneed;
        }
        if (sc->ccap < cneed) {
            cudaFree(sc->cnt);
            if (cudaMalloc(&sc->cnt, cneed * 4) != cudaSuccess) { sc->ccap = 0; set_err(nullptr, "t3b_op_attention: scratch allocation failed"); return T3B_ERR_OOM; }
            // on the caller's stream: the kernel below must see zeros
            if (cudaMemsetAsync(sc->cnt, 0, cneed * 4, st) != cudaSuccess) { set_err(nullptr, "t3b_op_attention: memset failed"); return T3B_ERR_CUDA; }
            sc->ccap = cneed;
        }
        if (!sc->errw) {
            if (cudaMalloc(&sc->errw, 4) != cudaSuccess) { set_err(nullptr, "t3b_op_attention: scratch allocation failed"); return T3B_ERR_OOM; }
            if (cudaMemsetAsync(sc->errw, 0, 4, st) != cudaSuccess) { set_err(nullptr, "t3b_op_attention: memset failed"); return T3B_ERR_CUDA; }
        }
    }
    unsigned * errw = sc->errw;
    // caches: [M][n_head][max_ctx][64]; K and V given separately
    AttnArgs a{};
    a.q = q_dev; a.ldq = n_head * T3B_HD;
    a.kv = (const __half *) k_dev; a.row_elems = (size_t) n_head * max_ctx * T3B_HD; a.layer_off = 0;
    a.v_off = (size_t) ((const __half *) v_dev - (const __half *) k_dev);
    a.row_of = nullptr; a.len = len_dev; a.len_add = 0; a.max_ctx = max_ctx; a.n_head = n_head;
    a.out = out_dev; a.ldo = n_head * T3B_HD; a.part = sc->part; a.cnt = sc->cnt; a.s_max = s_max; a.err = errw;
    if (M >= T3B_ATTN_ROWS_MIN) attn_rows_kernel<<<dim3(n_head, M), 128, 0, st>>>(a);
    else attn_decode_kernel<<<dim3(n_head, M, s_max), T3B_ATTN_CHUNK, 0, st>>>(a);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_err(nullptr, "t3b_op_attention: %s", cudaGetErrorString(e)); return T3B_ERR_CUDA; }
    return T3B_OK;
}

int t3b_op_attention_prompt(const float * q_dev, const void * k_dev, const void * v_dev, int M, int n_head, int max_ctx,
                            const int32_t * pos_dev, float * out_dev, void * cuda_stream) {
    if (!q_dev || !k_dev || !v_dev || !pos_dev || !out_dev || M <= 0 || n_head <= 0 || max_ctx <= 0) {
        set_err(nullptr, "t3b_op_attention_prompt: bad args");
        return T3B_ERR_ARG;
    }
    if ((((uintptr_t) k_dev) | ((uintptr_t) v_dev)) & 15) {
        set_err(nullptr, "t3b_op_attention_prompt: K and V caches must be 16-byte aligned");
        return T3B_ERR_ARG;
    }
    cudaStream_t st = (cudaStream_t) cuda_stream;
    int dev = 0; cudaGetDevice(&dev);
    OpScratch * sc;
    {
        std::lock_guard<std::mutex> lk(g_op_mu);
        sc = &g_op[dev];
        if (!sc->errw) {
            if (cudaMalloc(&sc->errw, 4) != cudaSuccess) { set_err(nullptr, "t3b_op_attention_prompt: scratch allocation failed"); return T3B_ERR_OOM; }
            if (cudaMemsetAsync(sc->errw, 0, 4, st) != cudaSuccess) { set_err(nullptr, "t3b_op_attention_prompt: memset failed"); return T3B_ERR_CUDA; }
        }
        if (!sc->pf_attr) {
            if (cudaFuncSetAttribute(attn_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, T3B_PREFILL_SMEM) != cudaSuccess) {
                set_err(nullptr, "t3b_op_attention_prompt: shared memory attribute");
                return T3B_ERR_CUDA;
            }
            sc->pf_attr = true;
        }
    }
    AttnArgs a{};
    a.q = q_dev; a.ldq = n_head * T3B_HD;
    a.kv = (const __half *) k_dev; a.row_elems = 0; a.layer_off = 0;
    a.v_off = (size_t) ((const __half *) v_dev - (const __half *) k_dev);
    a.row_of = nullptr; a.len = pos_dev; a.len_add = 1; a.max_ctx = max_ctx; a.n_head = n_head;
    a.out = out_dev; a.ldo = n_head * T3B_HD; a.err = sc->errw;
    attn_prefill_kernel<<<dim3(n_head, (M + T3B_PF_T - 1) / T3B_PF_T), 256, T3B_PREFILL_SMEM, st>>>(a, M);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_err(nullptr, "t3b_op_attention_prompt: %s", cudaGetErrorString(e)); return T3B_ERR_CUDA; }
    return T3B_OK;
}

int t3b_op_sample_philox(const float * cond_dev, const float * uncond_dev, int rows, int V, const int32_t * hist_dev,
                         const int32_t * hist_len_dev, int hist_stride, const t3b_sample_params * params_dev,
                         const uint64_t * seed_dev, const uint64_t * counter_dev, int32_t * tokens_out_dev,
                         void * cuda_stream) {
    if (!cond_dev || rows <= 0 || V <= 1 || V > T3B_SAMPLER_VMAX || !params_dev || !seed_dev || !counter_dev || !tokens_out_dev) {
        set_err(nullptr, "t3b_op_sample_philox: bad args");
        return T3B_ERR_ARG;
    }
    int dev = 0; cudaGetDevice(&dev);
    ExpFix fx;
    if (fix_table(dev, &fx, nullptr) != T3B_OK) return T3B_ERR_CUDA;
    static bool attr_set[64] = {false};
    if (dev < 64 && !attr_set[dev]) {
        cudaFuncSetAttribute(sampler_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, T3B_SAMPLER_SMEM);
        attr_set[dev] = true;
    }
    SampArgs a{};
    a.cond = cond_dev; a.cond_stride = V; a.uncond = uncond_dev; a.uncond_stride = V; a.V = V; a.slot_of = nullptr;
    a.hist = (int *) hist_dev; a.hist_stride = hist_stride; a.hist_len = (int *) hist_len_dev; a.hist_append = 0;
    a.params = params_dev; a.params_per_row = 1; a.rng_mode = nullptr; a.mt = nullptr;
    a.ph_seed = (const unsigned long long *) seed_dev; a.ph_ctr = (unsigned long long *) counter_dev;
    a.tok_out = tokens_out_dev; a.step_tok = nullptr; a.done = nullptr; a.stop_token = -1; a.fx = fx;
    // debug: T3B_SAMPLER_TIMELINE=<file> writes stage stamps of row 0 (T3B_SAMPLER_TL u64 ns)
    const char * tl_file = getenv("T3B_SAMPLER_TIMELINE");
    if (tl_file) { cudaMalloc(&a.tl, T3B_SAMPLER_TL * 8); cudaMemsetAsync(a.tl, 0, T3B_SAMPLER_TL * 8, (cudaStream_t) cuda_stream); }
    sampler_kernel<<<rows, T3B_SAMPLER_THREADS, T3B_SAMPLER_SMEM, (cudaStream_t) cuda_stream>>>(a);
    if (tl_file) {
        unsigned long long h[T3B_SAMPLER_TL];
        cudaMemcpyAsync(h, a.tl, sizeof h, cudaMemcpyDeviceToHost, (cudaStream_t) cuda_stream);
        cudaStreamSynchronize((cudaStream_t) cuda_stream);
        if (FILE * f = fopen(tl_file, "wb")) { fwrite(h, 8, T3B_SAMPLER_TL, f); fclose(f); }
        cudaFree(a.tl);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_err(nullptr, "t3b_op_sample_philox: %s", cudaGetErrorString(e)); return T3B_ERR_CUDA; }
    return T3B_OK;
}

int t3b_op_expf(const float * in_dev, float * out_dev, int n, void * cuda_stream) {
    if (!in_dev || !out_dev || n < 0) { set_err(nullptr, "t3b_op_expf: bad args"); return T3B_ERR_ARG; }
    int dev = 0; cudaGetDevice(&dev);
    ExpFix fx;
    if (fix_table(dev, &fx, nullptr) != T3B_OK) return T3B_ERR_CUDA;
    if (n) expf_test_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t) cuda_stream>>>(in_dev, out_dev, n, fx);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) { set_err(nullptr, "t3b_op_expf: %s", cudaGetErrorString(e)); return T3B_ERR_CUDA; }
    return T3B_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free decode attention (t3b_op_attention_noalloc)
//
// For callers that may not allocate device memory on their decode path: the
// split partials and completion counters of attn_decode_kernel live in fixed
// static device arrays instead of cudaMalloc'd scratch.  In host code these
// symbols are host-side stand-ins, never device addresses: their device
// addresses are resolved once per device with cudaGetSymbolAddress (with that
// device current) and cached.  Nothing here calls cudaMalloc or cudaFree.
// ---------------------------------------------------------------------------
#define T3B_NOALLOC_PART_FLOATS (1u << 20)   // 4 MiB of (m, l, o[64]) split records
#define T3B_NOALLOC_CNT 4096u                // (row, head) completion counters
static __device__ __align__(256) float g_noalloc_part[T3B_NOALLOC_PART_FLOATS];
static __device__ __align__(256) unsigned g_noalloc_cnt[T3B_NOALLOC_CNT + 64];   // + error word

namespace {
struct NoAllocScratch { float * part = nullptr; unsigned * cnt = nullptr; };
std::mutex g_noalloc_mu;
std::map<int, NoAllocScratch> g_noalloc;
}

extern "C" int t3b_op_attention_noalloc(const float * q_dev, const void * k_dev, const void * v_dev, int M,
                                        int n_head, int max_ctx, const int32_t * len_dev, float * out_dev,
                                        void * cuda_stream) {
    if (!q_dev || !k_dev || !v_dev || !len_dev || !out_dev || M <= 0 || n_head <= 0 || max_ctx <= 0) {
        set_err(nullptr, "t3b_op_attention_noalloc: bad args");
        return T3B_ERR_ARG;
    }
    if ((((uintptr_t) k_dev) | ((uintptr_t) v_dev)) & 15) {
        set_err(nullptr, "t3b_op_attention_noalloc: K and V caches must be 16-byte aligned");
        return T3B_ERR_ARG;
    }
    const long long s_max = (max_ctx + T3B_ATTN_CHUNK - 1) / T3B_ATTN_CHUNK;
    const long long records = M >= T3B_ATTN_ROWS_MIN ? 0 : (long long) M * n_head * s_max;   // many rows: no split
    if (records * (T3B_HD + 2) > (long long) T3B_NOALLOC_PART_FLOATS || (long long) M * n_head > T3B_NOALLOC_CNT) {
        set_err(nullptr, "t3b_op_attention_noalloc: %d rows x %d heads x %lld splits exceeds the static scratch "
                "(%u partial records, %u counters)", M, n_head, s_max,
                T3B_NOALLOC_PART_FLOATS / (T3B_HD + 2), T3B_NOALLOC_CNT);
        return T3B_ERR_ARG;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { set_err(nullptr, "t3b_op_attention_noalloc: no device"); return T3B_ERR_CUDA; }
    NoAllocScratch sc;
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        auto it = g_noalloc.find(dev);
        if (it == g_noalloc.end()) {
            NoAllocScratch n;
            cudaError_t e1 = cudaGetSymbolAddress((void **) &n.part, g_noalloc_part);
            cudaError_t e2 = cudaGetSymbolAddress((void **) &n.cnt, g_noalloc_cnt);
            if (e1 != cudaSuccess || e2 != cudaSuccess) {
                set_err(nullptr, "t3b_op_attention_noalloc: cudaGetSymbolAddress failed: %s",
                        cudaGetErrorString(e1 != cudaSuccess ? e1 : e2));
                return T3B_ERR_CUDA;
            }
            it = g_noalloc.emplace(dev, n).first;
        }
        sc = it->second;
    }
    cudaStream_t st = (cudaStream_t) cuda_stream;
    const bool rows = M >= T3B_ATTN_ROWS_MIN;   // same kernel choice as t3b_op_attention
    cudaError_t e = cudaSuccess;
    // the split-K counters must start at zero; the array keeps the previous
    // call's contents, so clear the ones this call uses.  The error word is
    // left alone: t3b_op_check reads and clears it.
    if (!rows) e = cudaMemsetAsync(sc.cnt, 0, sizeof(unsigned) * (size_t) M * n_head, st);
    if (e != cudaSuccess) { set_err(nullptr, "t3b_op_attention_noalloc: %s", cudaGetErrorString(e)); return T3B_ERR_CUDA; }
    AttnArgs a{};
    a.q = q_dev; a.ldq = n_head * T3B_HD;
    a.kv = (const __half *) k_dev; a.row_elems = (size_t) n_head * max_ctx * T3B_HD; a.layer_off = 0;
    a.v_off = (size_t) ((const __half *) v_dev - (const __half *) k_dev);
    a.row_of = nullptr; a.len = len_dev; a.len_add = 0; a.max_ctx = max_ctx; a.n_head = n_head;
    a.out = out_dev; a.ldo = n_head * T3B_HD; a.part = sc.part; a.cnt = sc.cnt; a.s_max = (int) s_max;
    a.err = sc.cnt + T3B_NOALLOC_CNT;
    if (rows) attn_rows_kernel<<<dim3(n_head, M), 128, 0, st>>>(a);
    else attn_decode_kernel<<<dim3(n_head, M, (unsigned) s_max), T3B_ATTN_CHUNK, 0, st>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) { set_err(nullptr, "t3b_op_attention_noalloc: %s", cudaGetErrorString(e)); return T3B_ERR_CUDA; }
    return T3B_OK;
}

// Reads and clears the device error words of the op-level attention entry
// points on the current device, after the stream's work so far.
extern "C" int t3b_op_check(void * cuda_stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { set_err(nullptr, "t3b_op_check: no device"); return T3B_ERR_CUDA; }
    cudaStream_t st = (cudaStream_t) cuda_stream;
    unsigned * words[2] = {nullptr, nullptr};
    {
        std::lock_guard<std::mutex> lk(g_op_mu);
        auto it = g_op.find(dev);
        if (it != g_op.end()) words[0] = it->second.errw;
    }
    {
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        auto it = g_noalloc.find(dev);
        if (it != g_noalloc.end()) words[1] = it->second.cnt + T3B_NOALLOC_CNT;
    }
    if (cudaStreamSynchronize(st) != cudaSuccess) { set_err(nullptr, "t3b_op_check: stream failed"); return T3B_ERR_CUDA; }
    unsigned w = 0;
    for (unsigned * p : words) {
        if (!p) continue;
        unsigned v = 0;
        if (cudaMemcpy(&v, p, sizeof v, cudaMemcpyDeviceToHost) != cudaSuccess ||
            cudaMemset(p, 0, sizeof v) != cudaSuccess) {
            set_err(nullptr, "t3b_op_check: error word read failed");
            return T3B_ERR_CUDA;
        }
        w |= v;
    }
    if (w) {
        set_err(nullptr, "op-level device check failed (error word 0x%x:%s%s)", w,
                (w & T3B_DEVERR_POS) ? " length-out-of-range" : "", (w & T3B_DEVERR_TOKEN) ? " token-out-of-range" : "");
        return T3B_ERR_DEVICE;
    }
    return T3B_OK;
}
