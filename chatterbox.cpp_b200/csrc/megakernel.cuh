// megakernel.cuh — persistent batch-1 T3 decode: one cooperative launch runs
// n_steps full decode steps (embedding, 24 layers, head, sampler).
//
// Why: at batch 1 a T3 step moves ~190 MB (25-30 us of HBM time on a B200)
// but is a chain of ~120 dependent matrix-vector products, each needing the
// whole previous vector.  As separate kernels every link costs a launch;
// here every CTA (one per SM) stays resident and the links become waits on
// per-phase arrival counters: a producer CTA stores its slice of the output
// vector, then one thread releases it with a fenced atomic increment; a
// consumer CTA has ONE thread poll the counter (with a short back-off) and
// then reads the whole vector once.  (Polling the data itself with every
// thread put ~150K loads per round on the same few L2 lines and delayed the
// producers' stores; one poller per CTA keeps the hot line cool.)  Each CTA
// issues the loads of its weight slice for a phase BEFORE waiting for that
// phase's input, so weight streaming overlaps the dependency latency.
//
// Phases per layer, Q8_0 / F16 weights (rows split evenly over the G CTAs):
//   P1 LN1 + QKV GEMV (+ K/V append to the f16 cache)        -> q,k,v slots
//   P2 attention, CTA h < n_head owns head h; for Q8_0 weights the same CTA
//      also quantises its 64 outputs (Q8_0 blocks 2h, 2h+1) and forms the
//      out-projection over them for all 1024 rows       -> per-head partials
//   P3 (F16 weights only) proj GEMV + bias + residual        -> x_mid slots
//   P4 x_mid = sum of the 16 head partials + bias + residual (every CTA),
//      LN2 + fc GEMV + bias + GELU                            -> h slots
//   P5 fc2 GEMV + bias + residual                             -> x slots
// Q4_0 weights ("OWN" layout): CTAs 1..16 are attention CTAs that compute
// their own head's q/k/v rows from weights bulk-copied into shared memory
// during the previous layer (no q/k/v hand-off), then P2 as above; the other
// 132 CTAs are workers that run P4 and P5 alone; x and h move as tagged
// 64-bit words (value + launch/layer tag) instead of counter hand-offs.
// Then LN_f + head GEMV -> logit slots, CTA 0 runs the sampler, publishes the
// token slot, and every CTA builds the next step's embedding itself.
//
// Every wait is bounded (MK_SPIN polls); on timeout the CTA raises the abort
// flag and the error word, and all CTAs leave at their next wait.
#pragma once

#include "kernels.cuh"

#define MK_THREADS 512
#define MK_MAX_POS 640            // positions whose K/V fit the attention stage at once
#define MK_TP 320                 // longer contexts: positions per streamed K/V tile (K rows then V rows)
#define MK_SPIN (1u << 21)        // default polls per wait before giving up (~1 s); MegaArgs.spin
#define MK_MAXI 3                 // weight items (32-element blocks) per thread per phase

// activation buffers (floats) and arrival counters (one 128-byte line each)
#define MK_B_QKV 0
#define MK_B_ATT (MK_B_QKV + 3072)
#define MK_B_XM (MK_B_ATT + 1024)
#define MK_B_H (MK_B_XM + 1024)
#define MK_B_X (MK_B_H + 4096)
#define MK_B_LOG (MK_B_X + 1024)
#define MK_B_TOK (MK_B_LOG + T3B_SAMPLER_VMAX)
#define MK_B_PART (MK_B_TOK + 32)          // [16 heads][1024] out-projection partials
#define MK_B_HQ (MK_B_PART + 16 * 1024)     // fc output h in Q8_0: quants [4096] i8
#define MK_B_HD (MK_B_HQ + 1024)            //   block scales [128]
#define MK_B_HS (MK_B_HD + 128)             //   block sums [128]
#define MK_B_XT (MK_B_HS + 128)             // Q4_0 layout: x as tagged words [1024] u64 (2048 floats)
#define MK_B_HT (MK_B_XT + 2048)            // Q4_0 layout: h in Q8_0 as tagged words [1280] u64
#define MK_HPH 7                            // long contexts: helper workers per head (worker CTAs 1..112)
#define MK_HR_WORDS 66                      //   one helper's result: max, sum, o[64]
#define MK_HMAX 2048                        //   helped up to this many positions (slices of <= 256)
#define MK_B_HR (MK_B_HT + 2560)            // the helpers' results as tagged words [16][MK_HPH][66] u64
#define MK_B_TOTAL (MK_B_HR + 2 * 16 * MK_HPH * MK_HR_WORDS)
enum { MK_C_QKV, MK_C_ATT, MK_C_XM, MK_C_H, MK_C_X, MK_C_LOG, MK_C_TOK, MK_C_N };
#define MK_C_STRIDE 32   // counters 128 bytes apart
#define MK_CTL_WORDS ((MK_C_N + 2) * MK_C_STRIDE)   // counters, abort flag, steps done

struct MkMat { const uint8_t * w; int type; int rb; };
struct MkLayer {
    const float * ln1g, * ln1b, * ln2g, * ln2b, * bqkv, * bo, * bfc, * bfc2;
    MkMat qkv, o, fc, fc2;
};

struct MegaArgs {
    const MkLayer * layers; int n_layer;
    const __half * semb; const float * wpe; const float * lnfg; const float * lnfb;
    MkMat head; const float * headb;
    int V; float eps;
    __half * kv; size_t layer_stride; size_t v_off; int max_ctx;
    int p0, n_steps, ignore_stop, stop_token;
    float * buf;              // MK_B_TOTAL floats
    unsigned * cnt;           // MK_C_N * MK_C_STRIDE counters, zero at launch
    unsigned * err; int * abort_flag; const int * cancel;
    int * steps_done;
    float * trace;                 // nullable: [n_steps + 1][V] logits, row 0 = prefill
    float * logits_out;            // nullable: logits of the last step (eval_step)
    int sample;                    // 0: stop after the head (eval_step without sampling)
    unsigned long long * tl;       // nullable: [G][MK_TL] globaltimer stamps of step tl_step
    int tl_step;
    int first_tok;                 // token of the first step (< 0: the stream's step_tok)
    unsigned epoch;                // launch number (1..4095): high bits of the x-word tags
    unsigned spin;                 // polls before a wait for another CTA or a staging copy gives up
    float * htrace;                // nullable: [n_layer + 1][1024] residual stream of step 0 (embedding, each layer's output)
    SampArgs samp;
};
#define MK_TL 1024        // timeline stamps per CTA: layer l at l * MK_TLL + i, head and sampler from MK_TLH
#define MK_TLL 32
#define MK_TLH 800

struct MegaState {
    int ready = 0;
    MkLayer * layers = nullptr;
    float * buf = nullptr;
    unsigned * cnt = nullptr;
    int * abort_flag = nullptr;
    int * steps_done = nullptr;
    int * cancel_host = nullptr;   // mapped pinned flag written by t3b_cancel
    int * cancel_dev = nullptr;
    int grid = 0;
    size_t smem = 0;
    unsigned epoch = 0;   // launches so far (mod 4095): tag space of the x words
};
inline void mega_free(MegaState & m) {
    if (m.layers) cudaFree(m.layers);
    if (m.buf) cudaFree(m.buf);
    if (m.cnt) cudaFree(m.cnt);   // abort_flag and steps_done live in the same block
    if (m.cancel_host) cudaFreeHost(m.cancel_host);
    m = MegaState();
}

// ---------------------------------------------------------------------------
// phase hand-off: release = stores, CTA barrier, fence, counter increment;
// acquire = one thread polls the counter, CTA barrier, L2-coherent reads
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned * p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void mk_release(unsigned * c) {
    __syncthreads();
    if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(c) : "memory");
}

// Wait until *c >= target.  Returns false (every thread) when the wait gave
// up or another CTA aborted.
__device__ __forceinline__ bool mk_acquire(const unsigned * c, unsigned target, const MegaArgs & a) {
    __shared__ int ok_s;
    if (threadIdx.x == 0) {
        int ok = 1;
        unsigned spins = 0;
        while (ld_acquire_u32(c) < target) {
            __nanosleep(20);
            if (++spins > a.spin || ((spins & 255u) == 0 && *(volatile int *) a.abort_flag)) {
                if (spins > a.spin) { atomicOr(a.err, T3B_DEVERR_TIMEOUT); atomicExch(a.abort_flag, 1); }
                ok = 0;
                break;
            }
        }
        ok_s = ok;
    }
    __syncthreads();
    return ok_s != 0;
}

// wait, then copy n (<= 4096, multiple of 4) floats of src into dst (smem);
// every load is issued before the first store so the copy is one round trip
__device__ __forceinline__ bool mk_wait_vec(const unsigned * c, unsigned target, const float * src, int n, float * dst,
                                            const MegaArgs & a) {
    if (!mk_acquire(c, target, a)) return false;
    float4 v[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int i = (threadIdx.x + u * MK_THREADS) * 4;
        if (i < n) v[u] = __ldcg((const float4 *) (src + i));
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int i = (threadIdx.x + u * MK_THREADS) * 4;
        if (i < n) *(float4 *) (dst + i) = v[u];
    }
    __syncthreads();
    return true;
}

// x hand-off without a release fence (Q4_0 layout): each element is one
// 64-bit word {tag, value} stored with a single relaxed store, tag = launch
// epoch << 20 | layer occurrence k, so a word whose tag matches is the value
// of that occurrence.  Warp 0 of the consumer polls all 1024 words (32 per
// lane) until every tag matches, then writes the values to dst (smem).
__device__ __forceinline__ unsigned mk_xtag(unsigned epoch, unsigned k) { return (epoch << 20) | (k & 0xfffffu); }
__device__ __forceinline__ void mk_st_x(unsigned long long * p, unsigned tag, float v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(((unsigned long long) tag << 32) | __float_as_uint(v))
                 : "memory");
}
__device__ __forceinline__ bool mk_wait_x(const unsigned long long * src, unsigned tag, float * dst, const MegaArgs & a) {
    __shared__ int okx;
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        unsigned long long w[32];
        int ok = 1;
        for (unsigned spins = 0;; ++spins) {
#pragma unroll
            for (int q = 0; q < 32; ++q)
                asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w[q]) : "l"(src + q * 32 + lane) : "memory");
            bool all = true;
#pragma unroll
            for (int q = 0; q < 32; ++q) all = all && (unsigned) (w[q] >> 32) == tag;
            if (__all_sync(0xffffffffu, all)) break;
            int stop = 0;
            if (lane == 0 && (spins > a.spin || ((spins & 255u) == 0 && *(volatile int *) a.abort_flag))) {
                if (spins > a.spin) { atomicOr(a.err, T3B_DEVERR_TIMEOUT); atomicExch(a.abort_flag, 1); }
                stop = 1;
            }
            if (__shfl_sync(0xffffffffu, stop, 0)) { ok = 0; break; }
            __nanosleep(20);
        }
        if (ok) {
#pragma unroll
            for (int q = 0; q < 32; ++q) dst[q * 32 + lane] = __uint_as_float((unsigned) w[q]);
        }
        if (lane == 0) okx = ok;
    }
    __syncthreads();
    return okx != 0;
}

// LayerNorm parameters of this thread's two elements (2*tid, 2*tid+1),
// loaded before a wait
struct MkLn { float2 g, b; };
__device__ __forceinline__ MkLn mk_ln_prefetch(const float * g, const float * b) {
    MkLn p;
    p.g = __ldg((const float2 *) g + threadIdx.x);
    p.b = __ldg((const float2 *) b + threadIdx.x);
    return p;
}

// ---------------------------------------------------------------------------
// activation prep in shared memory (same arithmetic as prep_act_kernel)
// ---------------------------------------------------------------------------
struct MkAct {
    float * v;      // input vector [K]
    int8_t * q;     // Q8_0 quants [K]
    float * d;      // block scales [K/32]
    int * s;        // block sums [K/32]
    __half * h;     // f16 copy [K] (F16 weights)
};

// h hand-off without a release fence (Q4_0 layout), in the tagged-word form
// of the x hand-off: words [0, 1024) carry four quants each (block b in words
// 8b .. 8b+7), words 1024 + b and 1152 + b the block's scale and sum.  Warps
// 0 and 1 each poll their 640 words (20 per lane) until every tag matches.
#define MK_HT_WORDS 1280
__device__ __forceinline__ bool mk_wait_h(const unsigned long long * src, unsigned tag, const MkAct & x, const MegaArgs & a) {
    __shared__ int okh[2];
    if (threadIdx.x < 64) {
        const int t = threadIdx.x, lane = t & 31;
        unsigned long long w[MK_HT_WORDS / 64];
        int ok = 1;
        for (unsigned spins = 0;; ++spins) {
#pragma unroll
            for (int q = 0; q < MK_HT_WORDS / 64; ++q)
                asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w[q]) : "l"(src + q * 64 + t) : "memory");
            bool all = true;
#pragma unroll
            for (int q = 0; q < MK_HT_WORDS / 64; ++q) all = all && (unsigned) (w[q] >> 32) == tag;
            if (__all_sync(0xffffffffu, all)) break;
            int stop = 0;
            if (lane == 0 && (spins > a.spin || ((spins & 255u) == 0 && *(volatile int *) a.abort_flag))) {
                if (spins > a.spin) { atomicOr(a.err, T3B_DEVERR_TIMEOUT); atomicExch(a.abort_flag, 1); }
                stop = 1;
            }
            if (__shfl_sync(0xffffffffu, stop, 0)) { ok = 0; break; }
            __nanosleep(20);
        }
        if (ok) {
#pragma unroll
            for (int q = 0; q < MK_HT_WORDS / 64; ++q) {
                const int j = q * 64 + t;
                const unsigned v = (unsigned) w[q];
                if (j < 1024) *(unsigned *) (x.q + 4 * j) = v;
                else if (j < 1152) x.d[j - 1024] = __uint_as_float(v);
                else x.s[j - 1152] = (int) v;
            }
        }
        if (lane == 0) okh[t >> 5] = ok;
    }
    __syncthreads();
    return okh[0] != 0 && okh[1] != 0;
}


// Sum over the CTA in double with a single barrier: warp trees, then every
// warp reduces the 16 warp partials itself (same order in every warp).
__device__ __forceinline__ double mk_block_sum_d(double v, double * red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[w] = v;
    __syncthreads();
    double r = red[lane & (MK_THREADS / 32 - 1)];
#pragma unroll
    for (int o = MK_THREADS / 64; o; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    __syncthreads();   // red is reused by the next reduction
    return r;
}

// Sum of two doubles over the CTA with a single barrier (see mk_block_sum_d).
__device__ __forceinline__ double2 mk_block_sum_d2(double a, double b, double * red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) { a += __shfl_xor_sync(0xffffffffu, a, o); b += __shfl_xor_sync(0xffffffffu, b, o); }
    if (lane == 0) { red[w] = a; red[16 + w] = b; }
    __syncthreads();
    double ra = red[lane & 15], rb = red[16 + (lane & 15)];
#pragma unroll
    for (int o = 8; o; o >>= 1) { ra += __shfl_xor_sync(0xffffffffu, ra, o); rb += __shfl_xor_sync(0xffffffffu, rb, o); }
    __syncthreads();
    return make_double2(ra, rb);
}

// LayerNorm of a 1024-vector followed by its Q8_0 re-quantisation (or f16
// rounding for F16 weights), x0/x1 = elements 2*tid and 2*tid+1 held in
// registers.  Mean and variance come from one reduction of sum(x) and
// sum(x^2) in double (var = E[x^2] - mean^2), which differs from ggml's
// two-pass float form only in the last bits of the statistics.  Each thread
// quantises the two elements it normalised: 16 lanes share a 32-element
// block, so the normalised vector never goes through shared memory.
__device__ void mk_ln_quant(float x0, float x1, const MkLn & p, float eps, double * redd, const MkAct & x, bool f16) {
    const int tid = threadIdx.x, K = 2 * MK_THREADS;
    const double d0 = x0, d1 = x1;
    const double2 m = mk_block_sum_d2(d0 + d1, d0 * d0 + d1 * d1, redd);
    const double meand = m.x / K;
    const float mean = (float) meand;
    const float var = (float) fmax(m.y / K - meand * meand, 0.0);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    const float y0 = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x0, mean), scale), p.g.x), p.b.x);
    const float y1 = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x1, mean), scale), p.g.y), p.b.y);
    if (f16) {
        *(__half2 *) (x.h + 2 * tid) = __halves2half2(__float2half_rn(y0), __float2half_rn(y1));
    } else {
        float mx = fmaxf(fabsf(y0), fabsf(y1));
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float d = __fdiv_rn(mx, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        const int q0 = (int) roundf(__fmul_rn(y0, id)), q1 = (int) roundf(__fmul_rn(y1, id));
        *(short *) (x.q + 2 * tid) = (short) ((q0 & 0xff) | ((q1 & 0xff) << 8));
        int s = q0 + q1;
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if ((tid & 15) == 0) { x.d[tid >> 4] = __half2float(__float2half_rn(d)); x.s[tid >> 4] = s; }
    }
    __syncthreads();
}

// Q8_0 re-quantisation of the K-vector (K = 1024 or 4096): eight lanes own
// one 32-element block (four elements each), so every block of the vector is
// processed at once instead of warps walking blocks one after another.
__device__ __forceinline__ void mk_quant_block(const MkAct & x, int g, int sub) {
    const float4 v = *(const float4 *) (x.v + g * 32 + sub * 4);
    float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 4));
    const float d = __fdiv_rn(m, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    const int q0 = (int) roundf(__fmul_rn(v.x, id)), q1 = (int) roundf(__fmul_rn(v.y, id));
    const int q2 = (int) roundf(__fmul_rn(v.z, id)), q3 = (int) roundf(__fmul_rn(v.w, id));
    *(int *) (x.q + g * 32 + sub * 4) = (q0 & 0xff) | ((q1 & 0xff) << 8) | ((q2 & 0xff) << 16) | ((q3 & 0xff) << 24);
    int s = q0 + q1 + q2 + q3;
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    if (sub == 0) { x.d[g] = __half2float(__float2half_rn(d)); x.s[g] = s; }
}

__device__ void mk_quantize(const MkAct & x, int K, bool f16) {
    const int tid = threadIdx.x;
    if (f16) {
        for (int i = tid; i < K; i += MK_THREADS) x.h[i] = __float2half_rn(x.v[i]);
    } else {
        const int g = tid >> 3, sub = tid & 7;              // 64 groups of 8 lanes
        if (g < K / 32) mk_quant_block(x, g, sub);          // K = 1024: warps 8..15 idle
        if (K == 4096) mk_quant_block(x, g + 64, sub);      // K = 4096: blocks 64..127
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// weight slices: items are (row, 32-element block) pairs of rows [r0, r1)
// ---------------------------------------------------------------------------
template <int T> struct MkW { static constexpr int QW = T == T3B_Q4_0 ? 1 : (T == T3B_Q8_0 ? 2 : 4); };

template <int T>
struct MkPref {
    uint4 q[MK_MAXI][MkW<T>::QW];
    float d[MK_MAXI];
};

// Weights are streamed once per step: their lines are marked first to leave
// L2, so the K/V cache, the hand-off buffers and the kernel's own code (the
// sampler and head run once per step) stay resident across steps instead of
// being pushed out by 175 MB of weights (28% faster sampler, 8% per step).
__device__ __forceinline__ unsigned long long mk_pol_stream() {
    unsigned long long pol;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ uint4 ldg_v4(const void * p) {
    uint4 v;
    asm volatile("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p), "l"(mk_pol_stream()));
    return v;
}
__device__ __forceinline__ float ldg_h(const void * p) {
    unsigned short h;
    asm volatile("ld.global.nc.L2::cache_hint.u16 %0, [%1], %2;" : "=h"(h) : "l"(p), "l"(mk_pol_stream()));
    return __half2float(__ushort_as_half(h));
}
__device__ __forceinline__ uint32_t mk_ld_w32(const void * p) {
    uint32_t v;
    asm volatile("ld.global.nc.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(v) : "l"(p), "l"(mk_pol_stream()));
    return v;
}

// volatile loads: issued here, before the caller's wait, and not sunk past it
template <int T>
__device__ __forceinline__ void mk_prefetch(const MkMat & W, int K, int r0, int r1, MkPref<T> & pf) {
    const int NB = K / 32;
    const int nit = (r1 - r0) * NB;
#pragma unroll
    for (int j = 0; j < MK_MAXI; ++j) {
        const int i = threadIdx.x + j * MK_THREADS;
        if (i < nit) {
            const int row = r0 + i / NB, b = i % NB;
            const uint8_t * wr = W.w + (size_t) row * W.rb;
            if (T == T3B_Q4_0) {
                pf.q[j][0] = ldg_v4(wr + b * 16);
                pf.d[j] = ldg_h(wr + K / 2 + b * 2);
            } else if (T == T3B_Q8_0) {
                pf.q[j][0] = ldg_v4(wr + b * 32);
                pf.q[j][1 % MkW<T>::QW] = ldg_v4(wr + b * 32 + 16);
                pf.d[j] = ldg_h(wr + K + b * 2);
            } else {
#pragma unroll
                for (int c = 0; c < MkW<T>::QW; ++c) pf.q[j][c] = ldg_v4(wr + b * 64 + c * 16);
                pf.d[j] = 1.0f;
            }
        }
    }
}

// Dot products of the prefetched items with the prepared activation; row
// sums (bias not added) land in rowsum[0 .. r1-r0).  All item partials are
// formed first and their warp reductions run side by side.
template <int T>
__device__ __forceinline__ float mk_item_dot(const MkPref<T> & pf, int j, int b, const MkAct & x) {
    float v = 0.0f;
    if (T == T3B_Q4_0) {
        const int4 x0 = *(const int4 *) (x.q + b * 32), x1 = *(const int4 *) (x.q + b * 32 + 16);
        const uint4 qv = pf.q[j][0];
        int si = 0;
        si = __dp4a((int) (qv.x & 0x0F0F0F0Fu), x0.x, si);
        si = __dp4a((int) ((qv.x >> 4) & 0x0F0F0F0Fu), x1.x, si);
        si = __dp4a((int) (qv.y & 0x0F0F0F0Fu), x0.y, si);
        si = __dp4a((int) ((qv.y >> 4) & 0x0F0F0F0Fu), x1.y, si);
        si = __dp4a((int) (qv.z & 0x0F0F0F0Fu), x0.z, si);
        si = __dp4a((int) ((qv.z >> 4) & 0x0F0F0F0Fu), x1.z, si);
        si = __dp4a((int) (qv.w & 0x0F0F0F0Fu), x0.w, si);
        si = __dp4a((int) ((qv.w >> 4) & 0x0F0F0F0Fu), x1.w, si);
        si -= 8 * x.s[b];
        v = __fmul_rn(__fmul_rn((float) si, pf.d[j]), x.d[b]);
    } else if (T == T3B_Q8_0) {
        const int4 x0 = *(const int4 *) (x.q + b * 32), x1 = *(const int4 *) (x.q + b * 32 + 16);
        const uint4 q0 = pf.q[j][0], q1 = pf.q[j][1 % MkW<T>::QW];
        int si = 0;
        si = __dp4a((int) q0.x, x0.x, si); si = __dp4a((int) q0.y, x0.y, si);
        si = __dp4a((int) q0.z, x0.z, si); si = __dp4a((int) q0.w, x0.w, si);
        si = __dp4a((int) q1.x, x1.x, si); si = __dp4a((int) q1.y, x1.y, si);
        si = __dp4a((int) q1.z, x1.z, si); si = __dp4a((int) q1.w, x1.w, si);
        v = __fmul_rn(__fmul_rn((float) si, pf.d[j]), x.d[b]);
    } else {
#pragma unroll
        for (int c = 0; c < MkW<T>::QW; ++c) {
            const uint4 wv = pf.q[j][c];
            const __half2 * wp = (const __half2 *) &wv;
            const uint4 xv = *(const uint4 *) (x.h + b * 32 + c * 8);
            const __half2 * xp = (const __half2 *) &xv;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float2 wf = __half22float2(wp[t]), xf = __half22float2(xp[t]);
                v = fmaf(wf.x, xf.x, v);
                v = fmaf(wf.y, xf.y, v);
            }
        }
    }
    return v;
}

template <int T>
__device__ void mk_dot(const MkPref<T> & pf, int K, int r0, int r1, const MkAct & x, float * part, float * rowsum) {
    const int NB = K / 32, NP = NB / 32;   // warp portions per row
    const int nit = (r1 - r0) * NB;
    const int tid = threadIdx.x, lane = tid & 31;
    float v[MK_MAXI];
#pragma unroll
    for (int j = 0; j < MK_MAXI; ++j) {
        const int i = j * MK_THREADS + tid;
        v[j] = i < nit ? mk_item_dot<T>(pf, j, i % NB, x) : 0.0f;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
#pragma unroll
        for (int j = 0; j < MK_MAXI; ++j) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
#pragma unroll
    for (int j = 0; j < MK_MAXI; ++j) {
        const int i0 = j * MK_THREADS + (tid & ~31);
        if (lane == 0 && i0 < nit) part[i0 / 32] = v[j];
    }
    __syncthreads();
    for (int r = tid; r < r1 - r0; r += MK_THREADS) {
        float acc = 0.0f;
        for (int p = 0; p < NP; ++p) acc = __fadd_rn(acc, part[r * NP + p]);
        rowsum[r] = acc;
    }
    __syncthreads();
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
__device__ __forceinline__ int mk_r0(int N, int c, int G) { return (int) (((long long) N * c) / G); }

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
// phase timeline (debug): stamp point `i` of the traced step
#define MK_STAMP(i) do { if (a.tl && step == a.tl_step && tid == 0 && (i) < MK_TL) a.tl[(size_t) cta * MK_TL + (i)] = globaltimer_ns(); } while (0)


// Dynamic shared memory.  Q4_0 layers (the attention CTAs compute their
// head's q/k/v rows from weights staged in shared memory):
//   attention scratch | GEMV scratch | K rows | q/k/v weights, then V rows.
// Q8_0 / F16 layers: K rows | V rows | attention scratch, the GEMV scratch
// overlapping the K rows.
#define MK_ATT_BYTES ((256 + MK_MAX_POS + 1024 + 128) * 4)   // q/k/v[192] | p[MK_MAX_POS] | o[16][64] | head out[64] + Q8_0
#define MK_SCR_BYTES 8192                                     // Q8_0 of a 4096-vector, f16 copy of a 1024-vector, dot partials
#define MK_KV_BYTES (MK_MAX_POS * T3B_HD * 2)
#define MK_QKVW_ROW 576                                       // Q4_0 row of K = 1024: 512 quant bytes + 32 f16 scales
#define MK_QKVW_BYTES (3 * T3B_HD * MK_QKVW_ROW)
constexpr size_t mk_smem_bytes() {
    return (size_t) MK_ATT_BYTES + MK_SCR_BYTES + MK_KV_BYTES + (MK_QKVW_BYTES > MK_KV_BYTES ? MK_QKVW_BYTES : MK_KV_BYTES);
}
static_assert(mk_smem_bytes() >= 2 * MK_KV_BYTES + MK_ATT_BYTES, "K/V stage layout must fit");
// Q4_0 workers: their fc rows (one 32-row block, K = 1024) and fc2 rows (up
// to 8 rows of K = 4096) of two layer uses, bulk-copied into the top of
// shared memory one layer ahead; above the sampler's arrays (CTA 0) and the
// staged head rows
#define MK_FW_BYTES 18432                                     // 32 x 576 = 8 x 2304 bytes
#define MK_SMEM_TOTAL (MK_ATT_BYTES + MK_SCR_BYTES + MK_KV_BYTES + (MK_QKVW_BYTES > MK_KV_BYTES ? MK_QKVW_BYTES : MK_KV_BYTES))
#define MK_FW_OFF (MK_SMEM_TOTAL - 4 * MK_FW_BYTES)
static_assert(MK_SMEM_TOTAL == mk_smem_bytes(), "layout total");
static_assert(mk_smem_bytes() - 4 * MK_FW_BYTES >= T3B_SAMPLER_SMEM, "worker weight buffers must clear the sampler");
static_assert(mk_smem_bytes() - 4 * MK_FW_BYTES >= MK_ATT_BYTES + MK_SCR_BYTES + MK_KV_BYTES, "and the head rows");
static_assert(4096 + 1024 + 2048 + MK_MAXI * MK_THREADS / 32 * 4 <= MK_SCR_BYTES, "GEMV scratch must fit");

// cp.async of n K or V rows (64 f16 each) into shared memory
__device__ __forceinline__ void mk_stage_kv(__half * dst, const __half * src, int n) {
    const int nchunk = n * (T3B_HD * 2 / 16);
    const unsigned d0 = (unsigned) __cvta_generic_to_shared(dst);
    for (int i = threadIdx.x; i < nchunk; i += MK_THREADS)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d0 + i * 16), "l"(src + i * 8) : "memory");
}
__device__ __forceinline__ void mk_cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

// --- bulk copies (TMA engine, no multicast) completing on an mbarrier -------
__device__ __forceinline__ unsigned mk_saddr(const void * p) { return (unsigned) __cvta_generic_to_shared(p); }
__device__ __forceinline__ void mk_mbar_init(unsigned long long * mb) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(mk_saddr(mb)) : "memory");
}
// the phase's single arrival, announcing `bytes` of copies that complete on mb
__device__ __forceinline__ void mk_mbar_expect(unsigned long long * mb, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(mk_saddr(mb)), "r"(bytes) : "memory");
}
// bytes: multiple of 16; both addresses 16-byte aligned
__device__ __forceinline__ void mk_bulk_g2s(void * dst, const void * src, unsigned bytes, unsigned long long * mb) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(mk_saddr(dst)), "l"(src), "r"(bytes), "r"(mk_saddr(mb)) : "memory");
}
// wait for phase `parity` of mb; false after `limit` polls
__device__ __forceinline__ bool mk_mbar_wait(unsigned long long * mb, unsigned parity, unsigned limit = MK_SPIN) {
    const unsigned ad = mk_saddr(mb);
    for (unsigned spins = 0;; ++spins) {
        unsigned done;
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                     : "=r"(done) : "r"(ad), "r"(parity) : "memory");
        if (done) return true;
        if (spins >= limit) return false;
        __nanosleep(20);
    }
}
// bulk copy of weights: L2 evict-first, like every other weight stream
__device__ __forceinline__ void mk_bulk_g2s_w(void * dst, const void * src, unsigned bytes, unsigned long long * mb) {
    unsigned long long pol;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
                 ::"r"(mk_saddr(dst)), "l"(src), "r"(bytes), "r"(mk_saddr(mb)), "l"(pol) : "memory");
}
__device__ __forceinline__ void mk_fence_proxy_async() { asm volatile("fence.proxy.async;" ::: "memory"); }
// head h's q, k and v rows (64 each) of a Q4_0 q/k/v matrix (K = 1024):
// three contiguous sections, one bulk copy each
#define MK_QKVW_SEC (T3B_HD * MK_QKVW_ROW)
__device__ __forceinline__ void mk_bulk_qkvw(unsigned char * dst, const MkMat & W, int h, unsigned long long * mb) {
    unsigned long long pol;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    for (int sec = 0; sec < 3; ++sec)
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
                     ::"r"(mk_saddr(dst + sec * MK_QKVW_SEC)),
                     "l"(W.w + (size_t) (sec * 1024 + h * T3B_HD) * MK_QKVW_ROW), "r"((unsigned) MK_QKVW_SEC),
                     "r"(mk_saddr(mb)), "l"(pol) : "memory");
}

// q/k/v of one head from the staged Q4_0 rows.  Lane = 8 * g + c: row group
// g of the warp's four rows, blocks c, c+8, c+16, c+24 summed in that order,
// then a butterfly over the eight lanes.  Warp w takes rows 12w .. 12w+11.
// Raw row sums (no bias) go to out[192].
__device__ __forceinline__ void mk_qkv_own(const unsigned char * wst, const MkAct & x, float * out) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, g = lane >> 3, c = lane & 7;
    int4 xa[4], xb[4];
    float dx[4];
    int sx8[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int b = c + 8 * j;
        xa[j] = *(const int4 *) (x.q + b * 32);
        xb[j] = *(const int4 *) (x.q + b * 32 + 16);
        dx[j] = x.d[b];
        sx8[j] = 8 * x.s[b];
    }
    float acc[3];
#pragma unroll
    for (int it = 0; it < 3; ++it) {
        const unsigned char * rp = wst + (size_t) (w * 12 + it * 4 + g) * MK_QKVW_ROW;
        float t = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int b = c + 8 * j;
            const uint4 qv = *(const uint4 *) (rp + b * 16);
            const float dw = __half2float(*(const __half *) (rp + 512 + b * 2));
            int si = 0;
            si = __dp4a((int) (qv.x & 0x0F0F0F0Fu), xa[j].x, si);
            si = __dp4a((int) ((qv.x >> 4) & 0x0F0F0F0Fu), xb[j].x, si);
            si = __dp4a((int) (qv.y & 0x0F0F0F0Fu), xa[j].y, si);
            si = __dp4a((int) ((qv.y >> 4) & 0x0F0F0F0Fu), xb[j].y, si);
            si = __dp4a((int) (qv.z & 0x0F0F0F0Fu), xa[j].z, si);
            si = __dp4a((int) ((qv.z >> 4) & 0x0F0F0F0Fu), xb[j].z, si);
            si = __dp4a((int) (qv.w & 0x0F0F0F0Fu), xa[j].w, si);
            si = __dp4a((int) ((qv.w >> 4) & 0x0F0F0F0Fu), xb[j].w, si);
            si -= sx8[j];
            t = __fadd_rn(t, __fmul_rn(__fmul_rn((float) si, dw), dx[j]));
        }
        acc[it] = t;
    }
#pragma unroll
    for (int o = 4; o; o >>= 1)
#pragma unroll
        for (int it = 0; it < 3; ++it) acc[it] = __fadd_rn(acc[it], __shfl_xor_sync(0xffffffffu, acc[it], o));
    if (c == 0) {
#pragma unroll
        for (int it = 0; it < 3; ++it) out[w * 12 + it * 4 + g] = acc[it];
    }
}

// Row sums of `rows` (<= 64) staged Q4_0 rows of K = 1024 with the lane
// layout of mk_qkv_own (8 lanes per row, blocks c, c+8, c+16, c+24).
__device__ __forceinline__ void mk_rows_q4_smem(const unsigned char * wst, int rows, const MkAct & x, float * out) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, g = lane >> 3, c = lane & 7;
    const int row = w * 4 + g;   // 16 warps x 4 row groups
    float t = 0.0f;
    if (row < rows) {
        const unsigned char * rp = wst + (size_t) row * MK_QKVW_ROW;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int b = c + 8 * j;
            const int4 xa = *(const int4 *) (x.q + b * 32), xb = *(const int4 *) (x.q + b * 32 + 16);
            const uint4 qv = *(const uint4 *) (rp + b * 16);
            const float dw = __half2float(*(const __half *) (rp + 512 + b * 2));
            int si = 0;
            si = __dp4a((int) (qv.x & 0x0F0F0F0Fu), xa.x, si);
            si = __dp4a((int) ((qv.x >> 4) & 0x0F0F0F0Fu), xb.x, si);
            si = __dp4a((int) (qv.y & 0x0F0F0F0Fu), xa.y, si);
            si = __dp4a((int) ((qv.y >> 4) & 0x0F0F0F0Fu), xb.y, si);
            si = __dp4a((int) (qv.z & 0x0F0F0F0Fu), xa.z, si);
            si = __dp4a((int) ((qv.z >> 4) & 0x0F0F0F0Fu), xb.z, si);
            si = __dp4a((int) (qv.w & 0x0F0F0F0Fu), xa.w, si);
            si = __dp4a((int) ((qv.w >> 4) & 0x0F0F0F0Fu), xb.w, si);
            si -= 8 * x.s[b];
            t = __fadd_rn(t, __fmul_rn(__fmul_rn((float) si, dw), x.d[b]));
        }
    }
#pragma unroll
    for (int o = 4; o; o >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (c == 0 && row < rows) out[row] = t;
}

// Row sums of Q4_0 rows staged in shared memory (row stride rb bytes, K/32
// blocks per row) in mk_dot's order: one warp takes a 32-block portion of a
// row (lane = block), a butterfly adds the lanes, and each row adds its
// portions in order.  At most 32 (row, portion) pairs: two per warp.
__device__ __forceinline__ void mk_dot_q4_smem(const unsigned char * wst, int rb, int K, int rows, const MkAct & x,
                                               float * part, float * rowsum) {
    const int NB = K / 32, NP = NB / 32;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int npairs = rows * NP;
    float v[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int pp = w + u * (MK_THREADS / 32);
        v[u] = 0.0f;
        if (pp < npairs) {
            const int r = pp / NP, b = (pp % NP) * 32 + lane;
            const unsigned char * rp = wst + (size_t) r * rb;
            const int4 x0 = *(const int4 *) (x.q + b * 32), x1 = *(const int4 *) (x.q + b * 32 + 16);
            const uint4 qv = *(const uint4 *) (rp + b * 16);
            const float dw = __half2float(*(const __half *) (rp + K / 2 + b * 2));
            int si = 0;
            si = __dp4a((int) (qv.x & 0x0F0F0F0Fu), x0.x, si);
            si = __dp4a((int) ((qv.x >> 4) & 0x0F0F0F0Fu), x1.x, si);
            si = __dp4a((int) (qv.y & 0x0F0F0F0Fu), x0.y, si);
            si = __dp4a((int) ((qv.y >> 4) & 0x0F0F0F0Fu), x1.y, si);
            si = __dp4a((int) (qv.z & 0x0F0F0F0Fu), x0.z, si);
            si = __dp4a((int) ((qv.z >> 4) & 0x0F0F0F0Fu), x1.z, si);
            si = __dp4a((int) (qv.w & 0x0F0F0F0Fu), x0.w, si);
            si = __dp4a((int) ((qv.w >> 4) & 0x0F0F0F0Fu), x1.w, si);
            si -= 8 * x.s[b];
            v[u] = __fmul_rn(__fmul_rn((float) si, dw), x.d[b]);
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1)
#pragma unroll
        for (int u = 0; u < 2; ++u) v[u] += __shfl_xor_sync(0xffffffffu, v[u], o);
#pragma unroll
    for (int u = 0; u < 2; ++u) {
        const int pp = w + u * (MK_THREADS / 32);
        if (lane == 0 && pp < npairs) part[pp] = v[u];
    }
    __syncthreads();
    for (int r = tid; r < rows; r += MK_THREADS) {
        float acc = 0.0f;
        for (int p = 0; p < NP; ++p) acc = __fadd_rn(acc, part[r * NP + p]);
        rowsum[r] = acc;
    }
    __syncthreads();
}

// LN_f + speech_head rows of this CTA; the head keeps its own weight type.
// hw (Q4_0 head, Q4_0 layers): this CTA's head rows, bulk-copied into
// shared memory during the last layer (completion: phase `hpar` of hmb);
// the dot then reads them there instead of a register prefetch, whose issue
// alone took ~3 us.
template <int HT>
__device__ __noinline__ bool mk_head(const MegaArgs & a, int step, int GW, const MkAct & act, float * part,
                                     float * rowsum, double * redd, float * xbuf, bool tagged,
                                     const unsigned char * hw, unsigned long long * hmb, unsigned hpar) {
    const int D = 1024, tid = threadIdx.x, G = gridDim.x;
    const int r0 = mk_r0(a.V, blockIdx.x, G), r1 = mk_r0(a.V, blockIdx.x + 1, G);
    MkPref<HT> pf;
    if (!hw) mk_prefetch<HT>(a.head, D, r0, r1, pf);
    const MkLn lp = mk_ln_prefetch(a.lnfg, a.lnfb);
    const float hb = tid < r1 - r0 ? __ldg(a.headb + r0 + tid) : 0.0f;
    const unsigned kx = (unsigned) ((step + 1) * a.n_layer);           // x hand-offs so far
    const int cta = blockIdx.x;
    MK_STAMP(MK_TLH + 9);
    float2 xv;
    if (tagged) {
        if (!mk_wait_x((const unsigned long long *) (a.buf + MK_B_XT), mk_xtag(a.epoch, kx), xbuf, a)) return false;
        xv = *(const float2 *) (xbuf + 2 * tid);
    } else {
        if (!mk_acquire(a.cnt + MK_C_X * MK_C_STRIDE, kx * GW, a)) return false;   // GW fc2 workers per layer
        xv = __ldcg((const float2 *) (a.buf + MK_B_X) + tid);
    }
    MK_STAMP(MK_TLH + 7);
    mk_ln_quant(xv.x, xv.y, lp, a.eps, redd, act, HT == T3B_F16);
    if (hw) {
        __shared__ int okhd;
        if (tid == 0) {
            const bool ok = mk_mbar_wait(hmb, hpar, a.spin);
            if (!ok) { atomicOr(a.err, T3B_DEVERR_TIMEOUT); atomicExch(a.abort_flag, 1); }
            okhd = ok;
        }
        __syncthreads();
        if (!okhd) return false;
        mk_rows_q4_smem(hw, r1 - r0, act, rowsum);
        __syncthreads();
    } else {
        mk_dot<HT>(pf, D, r0, r1, act, part, rowsum);
    }
    MK_STAMP(MK_TLH + 8);
    float * tr = a.trace ? a.trace + (size_t) (step + 1) * a.V : nullptr;
    float * lg = a.buf + MK_B_LOG;
    if (tid < r1 - r0) {
        const int n = r0 + tid;
        const float v = __fadd_rn(rowsum[tid], hb);
        if (tr) tr[n] = v;
        if (a.logits_out) a.logits_out[n] = v;
        lg[n] = v;
    }
    mk_release(a.cnt + MK_C_LOG * MK_C_STRIDE);
    return true;
}


// Bulk prefetch of a CTA's weight slice into L2 (one instruction, no
// completion to track): issued one phase ahead so the register prefetch of
// that phase hits L2 instead of HBM.
__device__ __forceinline__ void mk_l2_prefetch_rows(const MkMat & W, int r0, int r1) {
    if (threadIdx.x == 0) {
        const unsigned bytes = (unsigned) ((r1 - r0) * W.rb);
        if (bytes >= 16u)
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(W.w + (size_t) r0 * W.rb), "r"(bytes & ~15u)
                         : "memory");
    }
}
__device__ __forceinline__ void mk_l2_prefetch(const MkMat & W, int N) {
    mk_l2_prefetch_rows(W, mk_r0(N, blockIdx.x, gridDim.x), mk_r0(N, blockIdx.x + 1, gridDim.x));
}
// fc rows of a CTA: whole 32-row blocks when the CTA publishes h in Q8_0
__device__ __forceinline__ int mk_fc_r0(int c, int G, bool blocks) {
    return blocks ? mk_r0(128, c, G) * 32 : mk_r0(4096, c, G);
}

// rows of one GEMV phase: prefetch (before the caller's wait)
#define MK_GEMV_BEGIN(W, K, N)                                                                      \
    const int r0_ = mk_r0((N), blockIdx.x, gridDim.x), r1_ = mk_r0((N), blockIdx.x + 1, gridDim.x); \
    MkPref<T> pf_;                                                                                 \
    mk_prefetch<T>((W), (K), r0_, r1_, pf_);


// Bulk-copy bookkeeping of a CTA, one register (every thread holds the same
// value): per mbarrier i (0: K rows + q/k/v weights, 1: V rows / tile
// buffer B, 2: head rows, 3: tile buffer A, 4 and 5: a worker's fc + fc2
// rows of even and odd layer uses, 6: a helper's q rows and K/V slice) bit
// 2i = a phase was issued and not yet waited for, bit 2i+1 = that phase's
// parity; bits 16, 17 and 18 = the parity of the next phase of mbarriers 1,
// 3 and 6.
#define CP_OUT(i) ((cp >> (2 * (i))) & 1u)
#define CP_PAR(i) ((cp >> (2 * (i) + 1)) & 1u)
#define CP_ISSUE(i, par) (cp = (cp & ~(3u << (2 * (i)))) | ((1u | (((unsigned) (par) & 1u) << 1)) << (2 * (i))))
#define CP_DONE(i) (cp &= ~(1u << (2 * (i))))
// issue on mbarrier 1 or 3, whose phases alternate parity
#define CP_ISSUE_NEXT(i, nb) do { CP_ISSUE(i, (cp >> (nb)) & 1u); cp ^= 1u << (nb); } while (0)

// waits (bounded, MK_SPIN polls each) for every copy phase still in flight
#define MK_NMBAR 7
#define CP_PENDING 0x3fffu   // bits 0..13: phases issued per mbarrier
__device__ __noinline__ void mk_drain(unsigned long long * mbar, unsigned cp) {
#pragma unroll 1
    for (int i = 0; i < MK_NMBAR; ++i)
        if (CP_OUT(i)) mk_mbar_wait(&mbar[i], CP_PAR(i));
}

// every exit first waits (bounded) for this CTA's copies still in flight
#define MK_BAIL do {                                                                  \
        asm volatile("cp.async.wait_all;" ::: "memory");                              \
        if (tid == 0 && (cp & CP_PENDING)) mk_drain(mbar, cp);                       \
        return;                                                                       \
    } while (0)

// ---------------------------------------------------------------------------
// contexts longer than MK_MAX_POS: K/V streamed in tiles of MK_TP positions
// (out of line: the loop is rarely taken, and inlined into the layer loop its
// code slowed every phase of the common case by ~9%)
// ---------------------------------------------------------------------------
// Tile i of positions [0, npos) of one head (K rows, then V rows at row
// MK_TP) into buffer A (kst, mbarrier 3) or B (vst, mbarrier 1), issued by
// the CTA's copy thread; every thread updates the bookkeeping.  The current
// position is never copied: its K/V come from the q/k/v outputs.
__device__ __noinline__ unsigned mk_issue_tile(unsigned cp, int i, int npos, const __half * kb, size_t v_off, bool inB,
                                               __half * kst, __half * vst, unsigned long long * mbar) {
    if (threadIdx.x == MK_THREADS - 32) {
        const int t0 = i * MK_TP;
        const int n = max(0, min(MK_TP, npos - t0));
        const unsigned rb = (unsigned) n * T3B_HD * 2;
        __half * dst = inB ? vst : kst;
        unsigned long long * mb = inB ? &mbar[1] : &mbar[3];
        mk_fence_proxy_async();   // K/V rows this CTA stored (generic proxy) are read by the bulk copy
        mk_mbar_expect(mb, 2u * rb);
        if (n > 0) {
            mk_bulk_g2s(dst, kb + (size_t) t0 * T3B_HD, rb, mb);
            mk_bulk_g2s(dst + (size_t) MK_TP * T3B_HD, kb + v_off + (size_t) t0 * T3B_HD, rb, mb);
        }
    }
    if (inB) CP_ISSUE_NEXT(1, 16);
    else CP_ISSUE_NEXT(3, 17);
    return cp;
}

// One head's attention over L = pos + 1 > MK_MAX_POS positions: tiles
// through buffers A and B with an online softmax (running max, per-thread
// sums and per-warp outputs rescaled when the max grows).  Tile 0 is
// expected in A (tile0_ready: it came with the q/k/v weights), tile 1 in B
// (issued by the caller); this issues tiles 2.. as buffers free up.  Writes
// the per-warp outputs og[16][64] and returns the softmax denominator, or a
// negative value (every thread) when a copy wait gave up; *cpp is updated.
__device__ __noinline__ float mk_attend_tiled(unsigned * cpp, bool tile0_ready, int pos, const __half * kb, size_t v_off,
                                              const float * qkvh, __half * kst, __half * vst, float * pw, float * rf,
                                              float * og, unsigned long long * mbar, int * okf, unsigned spin,
                                              unsigned * err, int * abort_flag) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int L = pos + 1, nt = (L + MK_TP - 1) / MK_TP;
    unsigned cp = *cpp;
    float m_run = -INFINITY, l_t = 0.0f;
    float2 o0 = make_float2(0.0f, 0.0f), o1 = make_float2(0.0f, 0.0f);
    for (int i = 0; i < nt; ++i) {
        const bool inB = (i & 1) != 0;
        const int bi = inB ? 1 : 3;
        __half * tb = inB ? vst : kst;
        if (!(tile0_ready && i == 0)) {
            if (tid == 0) {
                const bool ok = mk_mbar_wait(&mbar[bi], CP_PAR(bi), spin);
                if (!ok) { atomicOr(err, T3B_DEVERR_TIMEOUT); atomicExch(abort_flag, 1); }
                *okf = ok;
            }
            __syncthreads();
            if (!*okf) { *cpp = cp; return -1.0f; }
            CP_DONE(bi);
        }
        const int t0 = i * MK_TP, n = min(MK_TP, L - t0);
        if (i == nt - 1 && tid < 2 * T3B_HD) {   // the current position, f16 as in the cache
            const int c = tid & 63, vv = tid >> 6;
            tb[(size_t) (vv * MK_TP + pos - t0) * T3B_HD + c] = __float2half_rn(qkvh[64 + tid]);
        }
        __syncthreads();
        float sc = -INFINITY;
        if (tid < n) {
            const uint4 * kp = (const uint4 *) (tb + (size_t) tid * T3B_HD);
            float dot = 0.0f;
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
                const int c = (cc + tid) & 7;
                const uint4 uu = kp[c];
                const float4 qa = *(const float4 *) (qkvh + c * 8), qb = *(const float4 *) (qkvh + c * 8 + 4);
                const __half2 * hp = (const __half2 *) &uu;
                const float2 f0 = __half22float2(hp[0]), f1 = __half22float2(hp[1]);
                const float2 f2 = __half22float2(hp[2]), f3 = __half22float2(hp[3]);
                dot = fmaf(qa.x, f0.x, dot); dot = fmaf(qa.y, f0.y, dot);
                dot = fmaf(qa.z, f1.x, dot); dot = fmaf(qa.w, f1.y, dot);
                dot = fmaf(qb.x, f2.x, dot); dot = fmaf(qb.y, f2.y, dot);
                dot = fmaf(qb.z, f3.x, dot); dot = fmaf(qb.w, f3.y, dot);
            }
            sc = dot * 0.125f;
        }
        const float lm = warp_max(sc);
        if (lane == 0) rf[w] = lm;
        __syncthreads();
        const float m_new = fmaxf(m_run, warp_max(rf[lane & 15]));
        const float resc = expf(m_run - m_new);   // 0 for the first tile
        m_run = m_new;
        const float p = tid < n ? expf(sc - m_new) : 0.0f;
        if (tid < n) pw[tid] = p;
        l_t = __fmaf_rn(l_t, resc, p);
        __syncthreads();
        const __half * vt = tb + (size_t) MK_TP * T3B_HD;
        o0.x *= resc; o0.y *= resc; o1.x *= resc; o1.y *= resc;
        int j = w;
        for (; j + 16 < n; j += 32) {
            const float2 v0 = __half22float2(*(const __half2 *) (vt + (size_t) j * T3B_HD + 2 * lane));
            const float2 v1 = __half22float2(*(const __half2 *) (vt + (size_t) (j + 16) * T3B_HD + 2 * lane));
            const float p0 = pw[j], p1 = pw[j + 16];
            o0.x = fmaf(p0, v0.x, o0.x); o0.y = fmaf(p0, v0.y, o0.y);
            o1.x = fmaf(p1, v1.x, o1.x); o1.y = fmaf(p1, v1.y, o1.y);
        }
        if (j < n) {
            const float2 v0 = __half22float2(*(const __half2 *) (vt + (size_t) j * T3B_HD + 2 * lane));
            const float p0 = pw[j];
            o0.x = fmaf(p0, v0.x, o0.x); o0.y = fmaf(p0, v0.y, o0.y);
        }
        __syncthreads();   // tile buffer, pw and rf free again
        if (i + 2 < nt) cp = mk_issue_tile(cp, i + 2, pos, kb, v_off, inB, kst, vst, mbar);
    }
    const float ls = warp_sum(l_t);
    if (lane == 0) rf[32 + w] = ls;
    og[w * 64 + 2 * lane] = o0.x + o1.x;
    og[w * 64 + 2 * lane + 1] = o0.y + o1.y;
    __syncthreads();
    *cpp = cp;
    return warp_sum(lane < 16 ? rf[32 + lane] : 0.0f);
}

// ---------------------------------------------------------------------------
// Contexts of MK_MAX_POS < L <= MK_HMAX positions (Q4_0 layout): each head's
// positions split over its attention CTA and MK_HPH idle worker CTAs.  A
// slice is C = ceil(L / (MK_HPH + 1)) positions; helper j takes positions
// [j C, (j + 1) C), the attention CTA the rest (with the current position).
// A helper computes the head's q itself (LN1 of x, its 64 q rows bulk-copied
// with its K/V slice), attends its slice and publishes (max, sum, o[64]) as
// tagged words; the attention CTA merges them with its own slice in helper
// order.  One K/V stream of a long head is then 8 SMs' work instead of one's.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int mk_hslice(int L) { return (L + MK_HPH) / (MK_HPH + 1); }

// Attention of one slice by the CTA: keys j < n (<= MK_THREADS), K row j at
// ks + 64 j, V row j at vs + 64 j (shared memory), query q[64] (shared).
// Writes the per-warp outputs og[16][64]; returns {max score, sum of p}.
__device__ float2 mk_attend_slice(int n, const float * q, const __half * ks, const __half * vs, float * pw, float * rf,
                                  float * og) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    float sc = -INFINITY;
    if (tid < n) {
        const uint4 * kp = (const uint4 *) (ks + (size_t) tid * T3B_HD);
        float dot = 0.0f;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
            const int c = (cc + tid) & 7;
            const uint4 uu = kp[c];
            const float4 qa = *(const float4 *) (q + c * 8), qb = *(const float4 *) (q + c * 8 + 4);
            const __half2 * hp = (const __half2 *) &uu;
            const float2 f0 = __half22float2(hp[0]), f1 = __half22float2(hp[1]);
            const float2 f2 = __half22float2(hp[2]), f3 = __half22float2(hp[3]);
            dot = fmaf(qa.x, f0.x, dot); dot = fmaf(qa.y, f0.y, dot);
            dot = fmaf(qa.z, f1.x, dot); dot = fmaf(qa.w, f1.y, dot);
            dot = fmaf(qb.x, f2.x, dot); dot = fmaf(qb.y, f2.y, dot);
            dot = fmaf(qb.z, f3.x, dot); dot = fmaf(qb.w, f3.y, dot);
        }
        sc = dot * 0.125f;
    }
    const float lm = warp_max(sc);
    if (lane == 0) rf[w] = lm;
    __syncthreads();
    const float mx = warp_max(rf[lane & 15]);
    const float p = tid < n ? expf(sc - mx) : 0.0f;
    if (tid < n) pw[tid] = p;
    const float ls = warp_sum(p);
    if (lane == 0) rf[32 + w] = ls;
    __syncthreads();
    const float l = warp_sum(lane < 16 ? rf[32 + lane] : 0.0f);
    float2 o0 = make_float2(0.0f, 0.0f), o1 = make_float2(0.0f, 0.0f);
    int j = w;
    for (; j + 16 < n; j += 32) {
        const float2 v0 = __half22float2(*(const __half2 *) (vs + (size_t) j * T3B_HD + 2 * lane));
        const float2 v1 = __half22float2(*(const __half2 *) (vs + (size_t) (j + 16) * T3B_HD + 2 * lane));
        const float p0 = pw[j], p1 = pw[j + 16];
        o0.x = fmaf(p0, v0.x, o0.x); o0.y = fmaf(p0, v0.y, o0.y);
        o1.x = fmaf(p1, v1.x, o1.x); o1.y = fmaf(p1, v1.y, o1.y);
    }
    if (j < n) {
        const float2 v0 = __half22float2(*(const __half2 *) (vs + (size_t) j * T3B_HD + 2 * lane));
        const float p0 = pw[j];
        o0.x = fmaf(p0, v0.x, o0.x); o0.y = fmaf(p0, v0.y, o0.y);
    }
    og[w * 64 + 2 * lane] = o0.x + o1.x;
    og[w * 64 + 2 * lane + 1] = o0.y + o1.y;
    __syncthreads();
    return make_float2(mx, l);
}

// A helper's slice: q = its head's 64 q rows (staged Q4_0, the attention
// CTA's lane layout and bias order, so q is the same bits) on the prepared
// LN1 activation, the slice's attention, then {max, sum, o[64]} as tagged
// words at dst.
__device__ __noinline__ void mk_help(const unsigned char * qw, const MkAct & act, const float * bq, int n,
                                     const __half * ks, const __half * vs, float * att_s, float * rf,
                                     unsigned long long * dst, unsigned tag) {
    const int tid = threadIdx.x;
    float * q = att_s;              // [64]
    float * pw = att_s + 256;       // [n]
    float * og = att_s + 256 + MK_MAX_POS;   // [16][64]
    mk_rows_q4_smem(qw, T3B_HD, act, att_s + 64);
    __syncthreads();
    if (tid < T3B_HD) q[tid] = __fadd_rn(__fadd_rn(0.0f, att_s[64 + tid]), __ldg(bq + tid));
    __syncthreads();
    const float2 ml = mk_attend_slice(n, q, ks, vs, pw, rf, og);
    if (tid < T3B_HD) {
        float o = 0.0f;
#pragma unroll
        for (int gg = 0; gg < 16; ++gg) o += og[gg * 64 + tid];
        mk_st_x(dst + 2 + tid, tag, o);
    }
    if (tid == 0) { mk_st_x(dst, tag, ml.x); mk_st_x(dst + 1, tag, ml.y); }
    __syncthreads();
}

// The attention CTA's side: its own slice (L_own keys, K rows at kst, V rows
// at kst + 64 L_own), then the merge with the MK_HPH helpers' results for
// this head (src: [MK_HPH][66] tagged words, polled by warp 0): the combined
// output goes to og[0][*] (og[1..15][*] zeroed) and the combined sum is
// returned, so the caller's sum over og / denominator gives the attention.
// Negative (every thread) when the wait gave up.
__device__ __noinline__ float mk_attend_helped(int L_own, const float * qkvh, const __half * kst, float * pw, float * rf,
                                               float * og, float * hr, const unsigned long long * src, unsigned tag,
                                               unsigned spin, unsigned * err, int * abort_flag, int * okf) {
    const int tid = threadIdx.x;
    const float2 ml = mk_attend_slice(L_own, qkvh, kst, kst + (size_t) L_own * T3B_HD, pw, rf, og);
    constexpr int NW = MK_HPH * MK_HR_WORDS, NQ = (NW + 31) / 32;
    if (tid < 32) {
        const int lane = tid;
        unsigned long long wv[NQ];
        int ok = 1;
        for (unsigned spins = 0;; ++spins) {
#pragma unroll
            for (int q = 0; q < NQ; ++q) {
                const int i = q * 32 + lane;
                if (i < NW) asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(wv[q]) : "l"(src + i) : "memory");
                else wv[q] = (unsigned long long) tag << 32;
            }
            bool all = true;
#pragma unroll
            for (int q = 0; q < NQ; ++q) all = all && (unsigned) (wv[q] >> 32) == tag;
            if (__all_sync(0xffffffffu, all)) break;
            int stop = 0;
            if (lane == 0 && (spins > spin || ((spins & 255u) == 0 && *(volatile int *) abort_flag))) {
                if (spins > spin) { atomicOr(err, T3B_DEVERR_TIMEOUT); atomicExch(abort_flag, 1); }
                stop = 1;
            }
            if (__shfl_sync(0xffffffffu, stop, 0)) { ok = 0; break; }
            __nanosleep(20);
        }
        if (ok) {
#pragma unroll
            for (int q = 0; q < NQ; ++q) {
                const int i = q * 32 + lane;
                if (i < NW) hr[i] = __uint_as_float((unsigned) wv[q]);
            }
        }
        if (lane == 0) *okf = ok;
    }
    __syncthreads();
    if (!*okf) return -1.0f;
    // merge in order: own slice, helpers 0 .. MK_HPH - 1
    float M = ml.x;
#pragma unroll
    for (int jh = 0; jh < MK_HPH; ++jh) M = fmaxf(M, hr[jh * MK_HR_WORDS]);
    const float so = expf(ml.x - M);
    float lt = ml.y * so;
#pragma unroll
    for (int jh = 0; jh < MK_HPH; ++jh) lt = fmaf(hr[jh * MK_HR_WORDS + 1], expf(hr[jh * MK_HR_WORDS] - M), lt);
    float o = 0.0f;
    if (tid < T3B_HD) {
#pragma unroll
        for (int gg = 0; gg < 16; ++gg) o += og[gg * 64 + tid];
        o *= so;
#pragma unroll
        for (int jh = 0; jh < MK_HPH; ++jh) o = fmaf(hr[jh * MK_HR_WORDS + 2 + tid], expf(hr[jh * MK_HR_WORDS] - M), o);
    }
    __syncthreads();   // every read of og is done
    for (int i = tid; i < 16 * T3B_HD; i += MK_THREADS) og[i] = i < T3B_HD ? o : 0.0f;
    __syncthreads();
    return lt;
}

// LONG: the instantiation that can stream K/V in tiles past MK_MAX_POS
// positions.  The host launches it only when a decode will pass that many
// positions; the common instantiation carries none of that code, which
// (measured) keeps every phase of the short-context step ~12% faster.
template <int T, bool LONG>
__global__ __launch_bounds__(MK_THREADS, 1) void t3_decode_megakernel(MegaArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int D = 1024;
    __shared__ __align__(16) float xres[1024];   // layer input x (residual for P3)
    __shared__ __align__(16) float xmid[1024];   // x after attention (residual for P5)
    __shared__ double redd[32];
    __shared__ float rowsum[128];
    __shared__ int tokv;
    // scratch (reused by every phase): vec[4096] f32 | q[4096] i8 | d,s [128] | h[4096] f16 | part
    constexpr bool FUSE = T != T3B_F16;   // out-projection folded into the attention CTAs
    constexpr bool OWN = T == T3B_Q4_0;   // attention CTAs compute their head's q/k/v themselves
    constexpr bool LLX = OWN;             // x and h handed off as tagged words (no release fence)
    unsigned long long * bXT = (unsigned long long *) (a.buf + MK_B_XT);
    float * vec = (float *) smem;         // (Q8_0 / F16 layout only)
    MkAct act;
    float * part;
    __half * kst, * vst;
    float * att_s;
    if (OWN) {
        unsigned char * scr = smem + MK_ATT_BYTES;
        act.v = nullptr;
        act.q = (int8_t *) scr;
        act.d = (float *) (scr + 4096);
        act.s = (int *) (scr + 4096 + 512);
        act.h = (__half *) (scr + 4096 + 1024);
        part = (float *) (scr + 4096 + 1024 + 2048);
        att_s = (float *) smem;
        kst = (__half *) (smem + MK_ATT_BYTES + MK_SCR_BYTES);
        vst = (__half *) (smem + MK_ATT_BYTES + MK_SCR_BYTES + MK_KV_BYTES);   // after the q/k/v weights are used
    } else {
        act.v = vec;
        act.q = (int8_t *) (smem + 16384);
        act.d = (float *) (smem + 16384 + 4096);
        act.s = (int *) (smem + 16384 + 4096 + 512);
        act.h = (__half *) (smem + 16384 + 4096 + 1024);
        part = (float *) (smem + 16384 + 4096 + 1024 + 8192);
        kst = (__half *) smem;   // the attention stage (and, in CTA 0, the sampler) reuse the scratch bytes
        vst = kst + MK_MAX_POS * T3B_HD;
        att_s = (float *) (smem + 2 * MK_KV_BYTES);
    }
    unsigned char * const qkvw = (unsigned char *) vst;   // OWN: staged q/k/v weights of this CTA's head

    const int tid = threadIdx.x, cta = blockIdx.x, G = gridDim.x;
    const int NL = a.n_layer;
    const int Hn = 16;
    // attention CTAs: 1..16 when they stage weights (CTA 0 runs the sampler,
    // whose arrays would overwrite the staged rows), else 0..15
    const bool att = OWN ? (cta >= 1 && cta <= Hn) : cta < Hn;
    const int hh_ = OWN ? cta - 1 : cta;
    // fc / fc2 workers: with OWN the attention CTAs sit out P4 and P5 (their
    // bulk copies for the next layer are in flight then, and a release fence
    // in those CTAs would wait for them); worker wi of GW takes the rows
    const bool worker = !OWN || !att;
    const int GW = OWN ? G - Hn : G;
    const int wi = OWN ? (cta == 0 ? 0 : cta - Hn) : cta;
    // long contexts (LONG, Q4_0): workers 1 .. 16 MK_HPH help head (wi - 1) / MK_HPH with slice (wi - 1) % MK_HPH
    const bool helper = LONG && OWN && worker && wi >= 1 && wi <= 16 * MK_HPH;
    const int hh_h = helper ? (wi - 1) / MK_HPH : 0, hj_h = helper ? (wi - 1) % MK_HPH : 0;
    // OWN staging: mbar[0] = a use's K rows + q/k/v weights (use u = step *
    // n_layer + layer completes phase u), plus its V rows when K and V of
    // positions [0, pos] fit the K stage together ("packed": V at row pos+1);
    // otherwise mbar[1] = the V rows, loaded into the weight stage after the
    // q/k/v rows are computed.
    // mbar[2] (every CTA, Q4_0 head): this CTA's head rows, one phase per step.
    // Contexts longer than MK_MAX_POS (any layout): K/V tiles stream through
    // buffer A (kst; mbar[3]) and buffer B (vst; mbar[1]).
    // cp: which phases are in flight and their parities (CP_* above).
    // mbar[4], mbar[5] (Q4_0 workers): fc + fc2 rows of layer uses u with
    // u & 1 = 0 and 1; use u completes phase u >> 1.
    __shared__ __align__(8) unsigned long long mbar[MK_NMBAR];
    __shared__ int okf;
    unsigned cp = 0u;
    if (tid == 0) {
#pragma unroll
        for (int i = 0; i < MK_NMBAR; ++i) mk_mbar_init(&mbar[i]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // Q4_0 head with at most 64 rows per CTA: its rows are bulk-copied into the
    // K stage (free by then in every CTA) during the last layer, when no fenced
    // release can be waiting: the attention CTAs have all released and the x/h
    // hand-offs are tagged
    const int hr0 = mk_r0(a.V, cta, G), hr1 = mk_r0(a.V, cta + 1, G);
    const bool hstage = OWN && a.head.type == T3B_Q4_0 && hr1 - hr0 <= 64 && a.head.rb == MK_QKVW_ROW;
    auto issue_head = [&](int step_) {
        if (tid == MK_THREADS - 32) {
            const unsigned bytes = (unsigned) (hr1 - hr0) * MK_QKVW_ROW;
            mk_mbar_expect(&mbar[2], bytes);
            if (bytes) mk_bulk_g2s_w(kst, a.head.w + (size_t) hr0 * MK_QKVW_ROW, bytes, &mbar[2]);
        }
        CP_ISSUE(2, step_);
    };
    // OWN attention CTAs: bulk copies of use u's K rows [0, npos) of layer nl
    // and of that layer's q/k/v weights for this head, issued by the last
    // warp's first thread (not the hand-off poller)
    auto packed = [](int p) { return 2 * (p + 1) <= MK_MAX_POS; };
    auto tiled = [](int p) { return LONG && p + 1 > MK_MAX_POS; };
    auto helped = [](int p) { return LONG && OWN && p + 1 > MK_MAX_POS && p + 1 <= MK_HMAX; };
    auto issue_kw = [&](int u, int nl, int npos) {
        if (tid == MK_THREADS - 32) {
            const bool hp = helped(npos);
            const bool tl = tiled(npos) && !hp;
            const bool pk = packed(npos);
            // helped: the own slice, positions [c0, npos), K at row 0, V at row npos + 1 - c0
            const int c0 = hp ? MK_HPH * mk_hslice(npos + 1) : 0;
            const int nk = hp ? npos - c0 : (tl ? MK_TP : npos);
            const unsigned rb = (unsigned) nk * T3B_HD * 2;
            const __half * kb = a.kv + (size_t) nl * a.layer_stride + (size_t) hh_ * a.max_ctx * T3B_HD + (size_t) c0 * T3B_HD;
            mk_fence_proxy_async();   // K/V rows this CTA stored (generic proxy) are read by the bulk copy
            mk_mbar_expect(&mbar[0], (pk || tl || hp ? 2u : 1u) * rb + MK_QKVW_BYTES);
            if (nk > 0) {
                mk_bulk_g2s(kst, kb, rb, &mbar[0]);
                if (hp) mk_bulk_g2s(kst + (size_t) (nk + 1) * T3B_HD, kb + a.v_off, rb, &mbar[0]);
                else if (tl) mk_bulk_g2s(kst + (size_t) MK_TP * T3B_HD, kb + a.v_off, rb, &mbar[0]);
                else if (pk) mk_bulk_g2s(kst + (size_t) (npos + 1) * T3B_HD, kb + a.v_off, rb, &mbar[0]);
            }
            mk_bulk_qkvw(qkvw, a.layers[nl].qkv, hh_, &mbar[0]);
        }
        CP_ISSUE(0, u);
    };
    // Q4_0 workers: fc rows (block mode) and fc2 rows of each layer use go
    // into shared memory by bulk copies issued two uses ahead, when use u - 2's
    // dots are done, so the weights are resident when a phase starts and no
    // weight load sits in the load queue ahead of a hand-off poll
    const int n_uses = a.n_steps * NL;
    const int fr0 = mk_fc_r0(wi, GW, true), fr1 = mk_fc_r0(wi + 1, GW, true);
    const int f2r0 = mk_r0(D, wi, GW), f2r1 = mk_r0(D, wi + 1, GW);
    const bool wstage = OWN && worker && (fr1 - fr0) * MK_QKVW_ROW <= MK_FW_BYTES &&
                        (f2r1 - f2r0) * 4 * MK_QKVW_ROW <= MK_FW_BYTES && a.layers[0].fc.rb == MK_QKVW_ROW &&
                        a.layers[0].fc2.rb == 4 * MK_QKVW_ROW;
    unsigned char * const wbuf = smem + MK_FW_OFF;   // [fc | fc2] of uses u & 1 = 0, then 1
    auto issue_w = [&](int u) {
        const int j = u & 1;
        if (tid == MK_THREADS - 32) {
            const MkLayer & Lu = a.layers[u % NL];
            const unsigned b1 = (unsigned) (fr1 - fr0) * MK_QKVW_ROW, b2 = (unsigned) (f2r1 - f2r0) * 4 * MK_QKVW_ROW;
            mk_fence_proxy_async();   // the buffers were last read by generic loads
            mk_mbar_expect(&mbar[4 + j], b1 + b2);
            if (b1) mk_bulk_g2s_w(wbuf + 2 * j * MK_FW_BYTES, Lu.fc.w + (size_t) fr0 * MK_QKVW_ROW, b1, &mbar[4 + j]);
            if (b2) mk_bulk_g2s_w(wbuf + (2 * j + 1) * MK_FW_BYTES, Lu.fc2.w + (size_t) f2r0 * 4 * MK_QKVW_ROW, b2,
                                  &mbar[4 + j]);
        }
        CP_ISSUE(4 + j, (u >> 1) & 1);
    };
    if (wstage) {
        issue_w(0);
        if (n_uses > 1) issue_w(1);
    }
    unsigned * cQKV = a.cnt + MK_C_QKV * MK_C_STRIDE, * cATT = a.cnt + MK_C_ATT * MK_C_STRIDE;
    unsigned * cXM = a.cnt + MK_C_XM * MK_C_STRIDE, * cH = a.cnt + MK_C_H * MK_C_STRIDE;
    unsigned * cX = a.cnt + MK_C_X * MK_C_STRIDE, * cLOG = a.cnt + MK_C_LOG * MK_C_STRIDE;
    unsigned * cTOK = a.cnt + MK_C_TOK * MK_C_STRIDE;
    float * bQKV = a.buf + MK_B_QKV, * bATT = a.buf + MK_B_ATT, * bXM = a.buf + MK_B_XM;
    float * bH = a.buf + MK_B_H, * bX = a.buf + MK_B_X, * bLOG = a.buf + MK_B_LOG;
    float * bPART = a.buf + MK_B_PART;
    int8_t * bHQ = (int8_t *) (a.buf + MK_B_HQ);
    float * bHD = a.buf + MK_B_HD;
    int * bHS = (int *) (a.buf + MK_B_HS);
    int * bTOK = (int *) (a.buf + MK_B_TOK);

    int tok;
    {
        const int slot0 = a.samp.slot_of ? a.samp.slot_of[0] : 0;
        if (a.first_tok >= 0) {
            tok = a.first_tok;
            if (cta == 0 && tid == 0) a.samp.step_tok[slot0] = tok;   // the stream's last input token
        } else {
            tok = a.samp.step_tok[slot0];
        }
    }
    if (OWN && att) issue_kw(0, 0, a.p0);   // use 0: layer 0 of the first step
    for (int step = 0; step < a.n_steps; ++step) {
        // host cancel flag (mapped memory, a PCIe round trip): one thread of
        // CTA 0 reads it at the start of the step; the value is needed only
        // after the sampler, so the read overlaps the whole step
        int cancelled = 0;
        if (cta == 0 && tid == 0 && a.cancel) cancelled = *(volatile const int *) a.cancel;
        const int pos = a.p0 + step;
        // embedding: x = speech_emb[tok] + wpe[pos]
        for (int i = tid; i < D; i += MK_THREADS) {
            xres[i] = __fadd_rn(__half2float(a.semb[(size_t) tok * D + i]), a.wpe[(size_t) pos * D + i]);
            if (a.htrace && step == 0 && cta == 0) a.htrace[i] = xres[i];
        }
        __syncthreads();
        for (int l = 0; l < NL; ++l) {
            const MkLayer & Ly = a.layers[l];
            const unsigned k = (unsigned) (step * NL + l) + 1u;   // occurrence of this layer's phases
            // out-projection weights of this CTA's head (FUSE): blocks 2h, 2h+1
            // of rows tid and tid + 512 (quants and the two block scales).
            // OWN loads them before the layer-input wait, the others before
            // the q/k/v wait, so they arrive while the CTA waits.
            uint4 ow[2][MkW<T>::QW * 2];
            unsigned ows[2] = {0u, 0u};
            auto load_ow = [&]() {
                if (FUSE) {
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const uint8_t * wr = Ly.o.w + (size_t) (tid + u * MK_THREADS) * Ly.o.rb;
                        constexpr int QB = T == T3B_Q4_0 ? 16 : 32;
#pragma unroll
                        for (int c = 0; c < MkW<T>::QW * 2; ++c) ow[u][c] = ldg_v4(wr + 2 * hh_ * QB + c * 16);
                        ows[u] = mk_ld_w32(wr + (size_t) (D / 32) * QB + 4 * hh_);
                    }
                }
            };
            // ---------------- P1: LN1 + QKV (+ K/V append) ----------------
            if (OWN) {
                if (att) load_ow();
                // every CTA takes the layer input (P4's residual); the
                // attention CTAs normalise it and compute their head's q/k/v
                // rows from the staged weights, then append K/V at pos
                const MkLn lp = mk_ln_prefetch(Ly.ln1g, Ly.ln1b);
                const float bq = att && tid < 3 * T3B_HD ? __ldg(Ly.bqkv + (tid >> 6) * D + hh_ * T3B_HD + (tid & 63)) : 0.0f;
                const bool hwork = helper && helped(pos);
                const int hC = hwork ? mk_hslice(pos + 1) : 0;
                const int hn = hC;   // a helper's slice is full: MK_HPH C < pos
                if (hwork) {
                    // this layer's q rows of the head and the slice's K/V rows
                    // (positions [j C, (j + 1) C), all cached) into the free
                    // stages: K rows at kst, V rows after them, q rows at vst
                    if (tid == MK_THREADS - 32) {
                        const __half * kb = a.kv + (size_t) l * a.layer_stride + (size_t) hh_h * a.max_ctx * T3B_HD +
                                            (size_t) hj_h * hC * T3B_HD;
                        const unsigned rb = (unsigned) hn * T3B_HD * 2;
                        mk_fence_proxy_async();   // the stages were last read by generic loads
                        mk_mbar_expect(&mbar[6], 2u * rb + (unsigned) MK_QKVW_SEC);
                        mk_bulk_g2s(kst, kb, rb, &mbar[6]);
                        mk_bulk_g2s(kst + (size_t) hn * T3B_HD, kb + a.v_off, rb, &mbar[6]);
                        mk_bulk_g2s_w(qkvw, Ly.qkv.w + (size_t) hh_h * T3B_HD * MK_QKVW_ROW, (unsigned) MK_QKVW_SEC, &mbar[6]);
                    }
                    CP_ISSUE_NEXT(6, 18);
                }
                MK_STAMP(l * MK_TLL + 0);
                float2 xv;
                if (l > 0 && LLX) {
                    if (!mk_wait_x(bXT, mk_xtag(a.epoch, k - 1u), xres, a)) MK_BAIL;
                    xv = *(const float2 *) (xres + 2 * tid);
                } else if (l > 0) {
                    if (!mk_acquire(cX, (k - 1u) * GW, a)) MK_BAIL;
                    xv = __ldcg((const float2 *) bX + tid);
                    *(float2 *) (xres + 2 * tid) = xv;
                } else {
                    xv = *(const float2 *) (xres + 2 * tid);
                }
                MK_STAMP(l * MK_TLL + 1);
                if (hwork) {
                    mk_ln_quant(xv.x, xv.y, lp, a.eps, redd, act, false);
                    if (tid == 0) {
                        const bool ok = mk_mbar_wait(&mbar[6], CP_PAR(6), a.spin);
                        if (!ok) { atomicOr(a.err, T3B_DEVERR_TIMEOUT); atomicExch(a.abort_flag, 1); }
                        okf = ok;
                    }
                    __syncthreads();
                    if (!okf) MK_BAIL;
                    CP_DONE(6);
                    mk_help(qkvw, act, Ly.bqkv + hh_h * T3B_HD, hn, kst, kst + (size_t) hn * T3B_HD, att_s, (float *) redd,
                            (unsigned long long *) (a.buf + MK_B_HR) + (size_t) (hh_h * MK_HPH + hj_h) * MK_HR_WORDS,
                            mk_xtag(a.epoch, k));
                }
                if (att) {
                    float * qkvh = att_s;   // [192]
                    const __half * kb = a.kv + (size_t) l * a.layer_stride + (size_t) hh_ * a.max_ctx * T3B_HD;
                    mk_ln_quant(xv.x, xv.y, lp, a.eps, redd, act, false);
                    MK_STAMP(l * MK_TLL + 12);
                    if (tid == 0) {   // K rows and q/k/v weights of this use
                        const bool ok = mk_mbar_wait(&mbar[0], (unsigned) (k - 1u) & 1u, a.spin);
                        if (!ok) { atomicOr(a.err, T3B_DEVERR_TIMEOUT); atomicExch(a.abort_flag, 1); }
                        okf = ok;
                    }
                    __syncthreads();
                    if (!okf) MK_BAIL;
                    CP_DONE(0);
                    MK_STAMP(l * MK_TLL + 14);
                    mk_qkv_own(qkvw, act, qkvh);
                    __syncthreads();
                    MK_STAMP(l * MK_TLL + 15);
                    const bool pk = packed(pos);
                    __half * vrow = pk ? kst + (size_t) (pos + 1) * T3B_HD : vst;
                    if (helped(pos)) {
                        // the own slice (and its V rows) came with the weights
                    } else if (tiled(pos)) {
                        // tile 0 came with the weights; tile 1 replaces them
                        cp = mk_issue_tile(cp, 1, pos, kb, a.v_off, true, kst, vst, mbar);
                    } else if (!pk) {
                        // V rows [0, pos) replace the weights (every read of
                        // them finished before the barrier above).  Issued by
                        // the last warp, which has no part in the K/V append.
                        if (tid == MK_THREADS - 32) {
                            mk_mbar_expect(&mbar[1], (unsigned) pos * T3B_HD * 2);
                            if (pos > 0) mk_bulk_g2s(vst, kb + a.v_off, (unsigned) pos * T3B_HD * 2, &mbar[1]);
                        }
                        CP_ISSUE_NEXT(1, 16);
                    }
                    MK_STAMP(l * MK_TLL + 16);
                    if (tid < 3 * T3B_HD) {
                        const float v = __fadd_rn(__fadd_rn(0.0f, qkvh[tid]), bq);   // mk_dot's row sum + bias
                        qkvh[tid] = v;
                        if (tid >= T3B_HD) {
                            const int vv = tid >= 2 * T3B_HD, c = tid & 63;
                            const __half hv = __float2half_rn(v);
                            (vv ? (__half *) (kb + a.v_off) : (__half *) kb)[(size_t) pos * T3B_HD + c] = hv;
                            if (!tiled(pos)) (vv ? vrow : kst)[(size_t) pos * T3B_HD + c] = hv;
                            else if (helped(pos)) {
                                const int c0 = MK_HPH * mk_hslice(pos + 1), lo = pos + 1 - c0;
                                kst[(size_t) ((vv ? lo : 0) + pos - c0) * T3B_HD + c] = hv;
                            }
                        }
                    }
                    __syncthreads();
                    MK_STAMP(l * MK_TLL + 13);
                }
            } else {
                MK_GEMV_BEGIN(Ly.qkv, D, 3 * D)
                if (FUSE) mk_l2_prefetch_rows(Ly.fc, mk_fc_r0(cta, G, true), mk_fc_r0(cta + 1, G, true));   // P4's rows
                else mk_l2_prefetch(Ly.o, D);
                const MkLn lp = mk_ln_prefetch(Ly.ln1g, Ly.ln1b);
                const float bias = tid < r1_ - r0_ ? __ldg(Ly.bqkv + r0_ + tid) : 0.0f;
                MK_STAMP(l * MK_TLL + 0);
                // layer input: this thread's elements 2*tid, 2*tid+1 (the
                // embedding of layer 0 is already in xres)
                float2 xv;
                if (l > 0) {
                    if (!mk_acquire(cX, (k - 1u) * G, a)) MK_BAIL;
                    xv = __ldcg((const float2 *) bX + tid);
                    *(float2 *) (xres + 2 * tid) = xv;
                } else {
                    xv = *(const float2 *) (xres + 2 * tid);
                }
                MK_STAMP(l * MK_TLL + 1);
                mk_ln_quant(xv.x, xv.y, lp, a.eps, redd, act, T == T3B_F16);
                MK_STAMP(l * MK_TLL + 14);
                mk_dot<T>(pf_, D, r0_, r1_, act, part, rowsum);
                MK_STAMP(l * MK_TLL + 15);
                __half * kb = a.kv + (size_t) l * a.layer_stride;
                if (tid < r1_ - r0_) {
                    const int n = r0_ + tid;
                    const float v = __fadd_rn(rowsum[tid], bias);
                    if (n >= D) {
                        const int which = n >= 2 * D, rem = n - D - which * D;
                        __half * base = kb + (which ? a.v_off : 0);
                        base[((size_t) (rem >> 6) * a.max_ctx + pos) * T3B_HD + (rem & 63)] = __float2half_rn(v);
                    }
                    bQKV[n] = v;
                }
                MK_STAMP(l * MK_TLL + 16);
                mk_release(cQKV);
                MK_STAMP(l * MK_TLL + 2);
            }
            // ---------------- P2: attention (one CTA per head) ----------------
            if (att) {
                const int h = hh_;
                const __half * kb = a.kv + (size_t) l * a.layer_stride + (size_t) h * a.max_ctx * T3B_HD;
                const __half * vb = kb + a.v_off;
                if (!OWN && tiled(pos)) {
                    cp = mk_issue_tile(cp, 0, pos, kb, a.v_off, false, kst, vst, mbar);
                    cp = mk_issue_tile(cp, 1, pos, kb, a.v_off, true, kst, vst, mbar);
                } else if (!OWN) {
                    // stage K/V of positions [0, pos) while q/k/v are computed
                    mk_stage_kv(kst, kb, pos);
                    mk_stage_kv(vst, vb, pos);
                    mk_cp_commit();
                }
                if (!OWN) load_ow();
                float * qkvh = att_s;   // [192]
                if (!OWN) {
                    const bool ok = mk_acquire(cQKV, k * G, a);
                    MK_STAMP(l * MK_TLL + 12);
                    if (tid < 192) qkvh[tid] = __ldcg(bQKV + (tid / 64) * D + h * 64 + (tid & 63));
                    asm volatile("cp.async.wait_all;" ::: "memory");
                    __syncthreads();
                    if (!ok) MK_BAIL;
                    MK_STAMP(l * MK_TLL + 3);
                    if (tid < T3B_HD && !tiled(pos)) {
                        kst[(size_t) pos * T3B_HD + tid] = __float2half_rn(qkvh[64 + tid]);
                        vst[(size_t) pos * T3B_HD + tid] = __float2half_rn(qkvh[128 + tid]);
                    }
                    __syncthreads();
                    MK_STAMP(l * MK_TLL + 13);
                }
                const int L = pos + 1;
                const int lane = tid & 31, w = tid >> 5;
                float * rf = (float *) redd;   // 64 floats: [0,16) max, [32,48) sum
                float * pw = att_s + 256;      // [L] (or one tile's) softmax weights
                float lsum;
                float2 o0 = make_float2(0.0f, 0.0f), o1 = make_float2(0.0f, 0.0f);
                if (!tiled(pos)) {
                    // scores: thread t owns keys t and t + 512; each thread walks the
                    // 8 16-byte chunks of its K row in a rotated order so the warp's
                    // shared-memory reads spread over all banks
                    float sc[2];
                    float lm = -INFINITY;
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const int j = tid + u * MK_THREADS;
                        sc[u] = -INFINITY;
                        if (j < L) {
                            const uint4 * kp = (const uint4 *) (kst + (size_t) j * T3B_HD);
                            float dot = 0.0f;
#pragma unroll
                            for (int cc = 0; cc < 8; ++cc) {
                                const int c = (cc + tid) & 7;
                                const uint4 uu = kp[c];
                                const float4 qa = *(const float4 *) (qkvh + c * 8), qb = *(const float4 *) (qkvh + c * 8 + 4);
                                const __half2 * hp = (const __half2 *) &uu;
                                const float2 f0 = __half22float2(hp[0]), f1 = __half22float2(hp[1]);
                                const float2 f2 = __half22float2(hp[2]), f3 = __half22float2(hp[3]);
                                dot = fmaf(qa.x, f0.x, dot); dot = fmaf(qa.y, f0.y, dot);
                                dot = fmaf(qa.z, f1.x, dot); dot = fmaf(qa.w, f1.y, dot);
                                dot = fmaf(qb.x, f2.x, dot); dot = fmaf(qb.y, f2.y, dot);
                                dot = fmaf(qb.z, f3.x, dot); dot = fmaf(qb.w, f3.y, dot);
                            }
                            sc[u] = dot * 0.125f;
                            lm = fmaxf(lm, sc[u]);
                        }
                    }
                    lm = warp_max(lm);
                    if (lane == 0) rf[w] = lm;
                    __syncthreads();
                    const float mx = warp_max(rf[lane & 15]);
                    float ls = 0.0f;
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const int j = tid + u * MK_THREADS;
                        if (j < L) { const float p = expf(sc[u] - mx); pw[j] = p; ls += p; }
                    }
                    ls = warp_sum(ls);
                    if (lane == 0) rf[32 + w] = ls;
                    const bool vwait = OWN && CP_OUT(1);   // V rows loaded separately (not packed)
                    if (vwait && tid == 0) {   // this layer's V rows
                        const bool ok = mk_mbar_wait(&mbar[1], CP_PAR(1), a.spin);
                        if (!ok) { atomicOr(a.err, T3B_DEVERR_TIMEOUT); atomicExch(a.abort_flag, 1); }
                        okf = ok;
                        MK_STAMP(l * MK_TLL + 3);
                    }
                    __syncthreads();
                    if (vwait) {
                        if (!okf) MK_BAIL;
                        CP_DONE(1);
                    }
                    const __half * vsrc = (OWN && packed(pos)) ? kst + (size_t) (pos + 1) * T3B_HD : vst;
                    lsum = warp_sum(lane < 16 ? rf[32 + lane] : 0.0f);
                    MK_STAMP(l * MK_TLL + 9);
                    // o[d] = sum_j p_j v_j[d]: warp w takes keys j = w (mod 16), lane l
                    // dims 2l, 2l+1; two accumulators hide the load latency
                    {
                        int j = w;
                        for (; j + 16 < L; j += 32) {
                            const float2 v0 = __half22float2(*(const __half2 *) (vsrc + (size_t) j * T3B_HD + 2 * lane));
                            const float2 v1 = __half22float2(*(const __half2 *) (vsrc + (size_t) (j + 16) * T3B_HD + 2 * lane));
                            const float p0 = pw[j], p1 = pw[j + 16];
                            o0.x = fmaf(p0, v0.x, o0.x); o0.y = fmaf(p0, v0.y, o0.y);
                            o1.x = fmaf(p1, v1.x, o1.x); o1.y = fmaf(p1, v1.y, o1.y);
                        }
                        if (j < L) {
                            const float2 v0 = __half22float2(*(const __half2 *) (vsrc + (size_t) j * T3B_HD + 2 * lane));
                            const float p0 = pw[j];
                            o0.x = fmaf(p0, v0.x, o0.x); o0.y = fmaf(p0, v0.y, o0.y);
                        }
                    }
                } else if (helped(pos)) {
                    // own slice + the helpers' results (out of line)
                    const int c0 = MK_HPH * mk_hslice(pos + 1);
                    lsum = mk_attend_helped(pos + 1 - c0, qkvh, kst, pw, rf, att_s + 256 + MK_MAX_POS,
                                            (float *) (smem + MK_ATT_BYTES),
                                            (const unsigned long long *) (a.buf + MK_B_HR) + (size_t) h * MK_HPH * MK_HR_WORDS,
                                            mk_xtag(a.epoch, k), a.spin, a.err, a.abort_flag, &okf);
                    if (lsum < 0.0f) MK_BAIL;
                    MK_STAMP(l * MK_TLL + 9);
                } else {
                    // L > MK_MAX_POS: K/V streamed in tiles (out of line)
                    lsum = mk_attend_tiled(&cp, OWN, pos, kb, a.v_off, qkvh, kst, vst, pw, rf, att_s + 256 + MK_MAX_POS,
                                           mbar, &okf, a.spin, a.err, a.abort_flag);
                    if (lsum < 0.0f) MK_BAIL;
                    MK_STAMP(l * MK_TLL + 9);
                }
                {
                    float * og = att_s + 256 + MK_MAX_POS;   // [16][64]
                    if (!tiled(pos)) {
                        og[w * 64 + 2 * lane] = o0.x + o1.x;
                        og[w * 64 + 2 * lane + 1] = o0.y + o1.y;
                    }
                    __syncthreads();
                    MK_STAMP(l * MK_TLL + 17);

                    float * ho = og + 16 * 64;   // this head's 64 outputs
                    if (tid < 64) {
                        float t = 0.0f;
#pragma unroll
                        for (int gg = 0; gg < 16; ++gg) t += og[gg * 64 + tid];
                        t = t / lsum;
                        if (FUSE) ho[tid] = t;
                        else bATT[h * 64 + tid] = t;
                    }
                    if (FUSE) {
                        // Q8_0 of the two blocks (what the proj GEMV's activation
                        // prep does to blocks 2h, 2h+1 of the attention vector),
                        // by warp 0 with every lane in every shuffle
                        int8_t * hq = (int8_t *) (ho + 64);
                        float * hd = ho + 64 + 16;
                        int * hs = (int *) (ho + 64 + 18);
                        __syncthreads();
                        if (tid < 32) {
                            const float v0 = ho[lane], v1 = ho[32 + lane];
                            const float m0 = warp_max(fabsf(v0)), m1 = warp_max(fabsf(v1));
                            const float d0 = __fdiv_rn(m0, 127.0f), d1 = __fdiv_rn(m1, 127.0f);
                            const float i0 = d0 != 0.0f ? __fdiv_rn(1.0f, d0) : 0.0f;
                            const float i1 = d1 != 0.0f ? __fdiv_rn(1.0f, d1) : 0.0f;
                            const int q0 = (int) roundf(__fmul_rn(v0, i0)), q1 = (int) roundf(__fmul_rn(v1, i1));
                            hq[lane] = (int8_t) q0;
                            hq[32 + lane] = (int8_t) q1;
                            const int s0 = warp_sum_i(q0), s1 = warp_sum_i(q1);
                            if (lane == 0) {
                                hd[0] = __half2float(__float2half_rn(d0)); hd[1] = __half2float(__float2half_rn(d1));
                                hs[0] = s0; hs[1] = s1;
                            }
                        }
                        __syncthreads();
                        MK_STAMP(l * MK_TLL + 18);
                        const int4 xa = *(const int4 *) hq, xb = *(const int4 *) (hq + 16);
                        const int4 xc = *(const int4 *) (hq + 32), xe = *(const int4 *) (hq + 48);
                        const float dx0 = hd[0], dx1 = hd[1];
#pragma unroll
                        for (int u = 0; u < 2; ++u) {
                            int s0 = 0, s1 = 0;
                            if (T == T3B_Q4_0) {
                                const uint4 w0 = ow[u][0], w1 = ow[u][1];
                                s0 = __dp4a((int) (w0.x & 0x0F0F0F0Fu), xa.x, s0); s0 = __dp4a((int) ((w0.x >> 4) & 0x0F0F0F0Fu), xb.x, s0);
                                s0 = __dp4a((int) (w0.y & 0x0F0F0F0Fu), xa.y, s0); s0 = __dp4a((int) ((w0.y >> 4) & 0x0F0F0F0Fu), xb.y, s0);
                                s0 = __dp4a((int) (w0.z & 0x0F0F0F0Fu), xa.z, s0); s0 = __dp4a((int) ((w0.z >> 4) & 0x0F0F0F0Fu), xb.z, s0);
                                s0 = __dp4a((int) (w0.w & 0x0F0F0F0Fu), xa.w, s0); s0 = __dp4a((int) ((w0.w >> 4) & 0x0F0F0F0Fu), xb.w, s0);
                                s1 = __dp4a((int) (w1.x & 0x0F0F0F0Fu), xc.x, s1); s1 = __dp4a((int) ((w1.x >> 4) & 0x0F0F0F0Fu), xe.x, s1);
                                s1 = __dp4a((int) (w1.y & 0x0F0F0F0Fu), xc.y, s1); s1 = __dp4a((int) ((w1.y >> 4) & 0x0F0F0F0Fu), xe.y, s1);
                                s1 = __dp4a((int) (w1.z & 0x0F0F0F0Fu), xc.z, s1); s1 = __dp4a((int) ((w1.z >> 4) & 0x0F0F0F0Fu), xe.z, s1);
                                s1 = __dp4a((int) (w1.w & 0x0F0F0F0Fu), xc.w, s1); s1 = __dp4a((int) ((w1.w >> 4) & 0x0F0F0F0Fu), xe.w, s1);
                                s0 -= 8 * hs[0];
                                s1 -= 8 * hs[1];
                            } else {
                                const uint4 w0 = ow[u][0], w1 = ow[u][1 % (MkW<T>::QW * 2)];
                                const uint4 w2 = ow[u][2 % (MkW<T>::QW * 2)], w3 = ow[u][3 % (MkW<T>::QW * 2)];
                                s0 = __dp4a((int) w0.x, xa.x, s0); s0 = __dp4a((int) w0.y, xa.y, s0);
                                s0 = __dp4a((int) w0.z, xa.z, s0); s0 = __dp4a((int) w0.w, xa.w, s0);
                                s0 = __dp4a((int) w1.x, xb.x, s0); s0 = __dp4a((int) w1.y, xb.y, s0);
                                s0 = __dp4a((int) w1.z, xb.z, s0); s0 = __dp4a((int) w1.w, xb.w, s0);
                                s1 = __dp4a((int) w2.x, xc.x, s1); s1 = __dp4a((int) w2.y, xc.y, s1);
                                s1 = __dp4a((int) w2.z, xc.z, s1); s1 = __dp4a((int) w2.w, xc.w, s1);
                                s1 = __dp4a((int) w3.x, xe.x, s1); s1 = __dp4a((int) w3.y, xe.y, s1);
                                s1 = __dp4a((int) w3.z, xe.z, s1); s1 = __dp4a((int) w3.w, xe.w, s1);
                            }
                            const float dw0 = __half2float(__ushort_as_half((unsigned short) (ows[u] & 0xffffu)));
                            const float dw1 = __half2float(__ushort_as_half((unsigned short) (ows[u] >> 16)));
                            const float t0 = __fmul_rn(__fmul_rn((float) s0, dw0), dx0);
                            const float t1 = __fmul_rn(__fmul_rn((float) s1, dw1), dx1);
                            bPART[h * D + tid + u * MK_THREADS] = __fadd_rn(t0, t1);
                        }
                    }
                }
                MK_STAMP(l * MK_TLL + 19);
                __syncthreads();
                MK_STAMP(l * MK_TLL + 2);
                mk_release(cATT);
                MK_STAMP(l * MK_TLL + 5);
                // K and V rows are consumed (the release's barrier): stage the
                // next layer's (use k); layer 0 of the next step is staged
                // after the head, whose release would otherwise wait for it
                if (OWN && (l + 1 < NL || hstage)) {
                    // only once every head has released: bulk traffic in
                    // flight slows the release of the CTAs still storing
                    if (!mk_acquire(cATT, k * Hn, a)) MK_BAIL;
                    if (l + 1 < NL) issue_kw((int) k, l + 1, pos);
                    else issue_head(step);
                }
                MK_STAMP(l * MK_TLL + 4);
            }
            // ---------------- P3: proj + bias + residual (F16 weights) --------
            if (!FUSE) {
                MK_GEMV_BEGIN(Ly.o, D, D)
                mk_l2_prefetch(Ly.fc, 4 * D);
                const float bias = tid < r1_ - r0_ ? __ldg(Ly.bo + r0_ + tid) : 0.0f;
                if (!mk_wait_vec(cATT, k * Hn, bATT, D, vec, a)) MK_BAIL;
                MK_STAMP(l * MK_TLL + 5);
                mk_quantize(act, D, T == T3B_F16);
                mk_dot<T>(pf_, D, r0_, r1_, act, part, rowsum);
                if (tid < r1_ - r0_) {
                    const int n = r0_ + tid;
                    bXM[n] = __fadd_rn(__fadd_rn(rowsum[tid], bias), xres[n]);
                }
                mk_release(cXM);
            }
            // (OWN: no bulk L2 prefetches; their traffic slowed other CTAs' releases more than it saved)
            if (!OWN && l + 1 == NL) mk_l2_prefetch(a.head, a.V);   // every CTA has head rows
            // ---------------- P4: LN2 + fc + GELU ------------------------------
            if (worker) {
                // with the fused out-projection each worker owns whole 32-row
                // blocks of fc (128 blocks: one block or none per worker) and
                // publishes its slice of h already in Q8_0, which is fc2's
                // input; the F16 path publishes h as floats
                const int r0_ = mk_fc_r0(wi, GW, FUSE), r1_ = mk_fc_r0(wi + 1, GW, FUSE);
                const int uj = (int) (k - 1u) & 1;   // buffer pair of this use (wstage)
                MkPref<T> pf_;
                if (!wstage) mk_prefetch<T>(Ly.fc, D, r0_, r1_, pf_);
                if (!OWN) mk_l2_prefetch_rows(Ly.fc2, mk_r0(D, wi, GW), mk_r0(D, wi + 1, GW));
                const MkLn lp = mk_ln_prefetch(Ly.ln2g, Ly.ln2b);
                const float bias = tid < r1_ - r0_ ? __ldg(Ly.bfc + r0_ + tid) : 0.0f;
                float x0, x1;   // x_mid elements 2*tid, 2*tid+1
                if (FUSE) {
                    // x_mid = (sum over heads of the partials) + proj bias + x,
                    // heads added in order 0..15
                    const float2 bo = __ldg((const float2 *) Ly.bo + tid);
                    if (!mk_acquire(cATT, k * Hn, a)) MK_BAIL;
                    float2 p[16];
#pragma unroll
                    for (int hh = 0; hh < 16; ++hh) p[hh] = __ldcg((const float2 *) (bPART + hh * D) + tid);
                    x0 = p[0].x; x1 = p[0].y;
#pragma unroll
                    for (int hh = 1; hh < 16; ++hh) { x0 = __fadd_rn(x0, p[hh].x); x1 = __fadd_rn(x1, p[hh].y); }
                    const float2 xr = *(const float2 *) (xres + 2 * tid);
                    x0 = __fadd_rn(__fadd_rn(x0, bo.x), xr.x);
                    x1 = __fadd_rn(__fadd_rn(x1, bo.y), xr.y);
                } else {
                    if (!mk_acquire(cXM, k * G, a)) MK_BAIL;
                    const float2 xm = __ldcg((const float2 *) bXM + tid);
                    x0 = xm.x; x1 = xm.y;
                }
                *(float2 *) (xmid + 2 * tid) = make_float2(x0, x1);   // P5's residual (read after barriers)
                MK_STAMP(l * MK_TLL + 6);
                if (wstage && tid == 0) {   // this use's fc + fc2 rows (issued a layer ago)
                    const bool ok = mk_mbar_wait(&mbar[4 + uj], ((k - 1u) >> 1) & 1u, a.spin);
                    if (!ok) { atomicOr(a.err, T3B_DEVERR_TIMEOUT); atomicExch(a.abort_flag, 1); }
                    okf = ok;
                }
                if (r1_ > r0_) {   // CTA-uniform
                    mk_ln_quant(x0, x1, lp, a.eps, redd, act, T == T3B_F16);
                    if (OWN && wstage) {
                        if (!okf) MK_BAIL;
                        mk_dot_q4_smem(wbuf + 2 * uj * MK_FW_BYTES, MK_QKVW_ROW, D, r1_ - r0_, act, part, rowsum);
                    } else {
                        mk_dot<T>(pf_, D, r0_, r1_, act, part, rowsum);
                    }
                    if (OWN) MK_STAMP(l * MK_TLL + 10);   // fc dot done
                    if (FUSE) {
                        // warp w: GELU of block w of this CTA's rows, then
                        // Q8_0 with the arithmetic of mk_quant_block
                        const int w = tid >> 5, lane = tid & 31;
                        if (w < (r1_ - r0_) / 32) {
                            const float v = gelu_ggml(__fadd_rn(rowsum[tid], bias));
                            float mx = fabsf(v);
#pragma unroll
                            for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                            const float d = __fdiv_rn(mx, 127.0f);
                            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
                            const int q = (int) roundf(__fmul_rn(v, id));
                            int sq = q;
#pragma unroll
                            for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
                            if (LLX) {
                                // four lanes' quants per tagged word
                                const unsigned qb = (unsigned) q & 0xffu;
                                const unsigned q1 = __shfl_down_sync(0xffffffffu, qb, 1);
                                const unsigned q2 = __shfl_down_sync(0xffffffffu, qb, 2);
                                const unsigned q3 = __shfl_down_sync(0xffffffffu, qb, 3);
                                const int b = (r0_ >> 5) + w;
                                const unsigned tg = mk_xtag(a.epoch, k);
                                unsigned long long * ht = (unsigned long long *) (a.buf + MK_B_HT);
                                if ((lane & 3) == 0)
                                    mk_st_x(ht + b * 8 + (lane >> 2), tg, __uint_as_float(qb | (q1 << 8) | (q2 << 16) | (q3 << 24)));
                                if (lane == 0) {
                                    mk_st_x(ht + 1024 + b, tg, __half2float(__float2half_rn(d)));
                                    mk_st_x(ht + 1152 + b, tg, __int_as_float(sq));
                                }
                            } else {
                                bHQ[r0_ + tid] = (int8_t) q;
                                if (lane == 0) {
                                    bHD[(r0_ >> 5) + w] = __half2float(__float2half_rn(d));
                                    bHS[(r0_ >> 5) + w] = sq;
                                }
                            }
                        }
                    } else if (tid < r1_ - r0_) {
                        bH[r0_ + tid] = gelu_ggml(__fadd_rn(rowsum[tid], bias));
                    }
                    MK_STAMP(l * MK_TLL + 20);   // h slice stored
                }
                if (LLX) __syncthreads();
                else mk_release(cH);
                MK_STAMP(l * MK_TLL + 21);
                if (wstage) {
                    if (!okf) MK_BAIL;
                    CP_DONE(4 + uj);
                }
            }
            // ---------------- P5: fc2 + bias + residual ------------------------
            if (worker) {
                const int r0_ = mk_r0(D, wi, GW), r1_ = mk_r0(D, wi + 1, GW);
                MkPref<T> pf_;
                if (!wstage) mk_prefetch<T>(Ly.fc2, 4 * D, r0_, r1_, pf_);
                if (l + 1 < NL && !OWN) mk_l2_prefetch(a.layers[l + 1].qkv, 3 * D);
                const float bias = tid < r1_ - r0_ ? __ldg(Ly.bfc2 + r0_ + tid) : 0.0f;
                if (OWN) MK_STAMP(l * MK_TLL + 3);   // fc2 weights issued
                if (FUSE) {
                    // h arrives in Q8_0: 4096 quants, 128 scales, 128 sums
                    if (LLX) {
                        if (!mk_wait_h((const unsigned long long *) (a.buf + MK_B_HT), mk_xtag(a.epoch, k), act, a)) MK_BAIL;
                        if (l + 1 == NL && hstage) issue_head(step);
                    } else {
                        if (!mk_acquire(cH, k * GW, a)) MK_BAIL;
                        if (tid < 256) *(int4 *) (act.q + 16 * tid) = __ldcg((const int4 *) bHQ + tid);
                        else if (tid < 384) act.d[tid - 256] = __ldcg(bHD + tid - 256);
                        else act.s[tid - 384] = __ldcg(bHS + tid - 384);
                        __syncthreads();
                    }
                    MK_STAMP(l * MK_TLL + 7);
                } else {
                    if (!mk_wait_vec(cH, k * GW, bH, 4 * D, vec, a)) MK_BAIL;
                    MK_STAMP(l * MK_TLL + 7);
                    mk_quantize(act, 4 * D, true);
                }
                if (!OWN) MK_STAMP(l * MK_TLL + 10);
                if (OWN && wstage) {
                    mk_dot_q4_smem(wbuf + (2 * ((k - 1u) & 1u) + 1) * MK_FW_BYTES, 4 * MK_QKVW_ROW, 4 * D, r1_ - r0_, act,
                                   part, rowsum);
                    MK_STAMP(l * MK_TLL + 22);
                    if ((int) k + 1 < n_uses) issue_w((int) k + 1);   // use k - 1 + 2 into the buffers just read
                } else {
                    mk_dot<T>(pf_, 4 * D, r0_, r1_, act, part, rowsum);
                }
                MK_STAMP(l * MK_TLL + 11);
                if (tid < r1_ - r0_) {
                    const int n = r0_ + tid;
                    const float xo = __fadd_rn(__fadd_rn(rowsum[tid], bias), xmid[n]);
                    if (LLX) mk_st_x(bXT + n, mk_xtag(a.epoch, k), xo);
                    else bX[n] = xo;
                    if (a.htrace && step == 0) a.htrace[(size_t) (l + 1) * D + n] = xo;
                }
                if (LLX) __syncthreads();
                else mk_release(cX);
                MK_STAMP(l * MK_TLL + 8);
            }
        }
        // ---------------- head: LN_f + speech_head ------------------------------
        MK_STAMP(MK_TLH + 0);
        {
            bool ok;
            if (a.head.type == T3B_F16)
                ok = mk_head<T3B_F16>(a, step, GW, act, part, rowsum, redd, xres, LLX, nullptr, nullptr, 0u);
            else if (a.head.type == T3B_Q8_0)
                ok = mk_head<T3B_Q8_0>(a, step, GW, act, part, rowsum, redd, xres, LLX, nullptr, nullptr, 0u);
            else
                ok = mk_head<T3B_Q4_0>(a, step, GW, act, part, rowsum, redd, xres, LLX, hstage ? (const unsigned char *) kst : nullptr,
                                       &mbar[2], (unsigned) step & 1u);
            if (ok) CP_DONE(2);
            if (!ok) MK_BAIL;
        }
        // OWN: layer 0 of the next step (K rows up to this step's position)
        if (OWN && att && step + 1 < a.n_steps) issue_kw((step + 1) * NL, 0, pos + 1);
        MK_STAMP(MK_TLH + 1);
        if (!a.sample) MK_BAIL;   // eval_step: logits only
        // ---------------- sampler (CTA 0) and token broadcast -------------------
        if (cta == 0) {
            if (!mk_acquire(cLOG, (unsigned) (step + 1) * G, a)) MK_BAIL;
            SampArgs sa = a.samp;
            sa.cond = bLOG; sa.cond_stride = 0; sa.uncond = nullptr;   // read through L2 by the sampler
            sa.tl = (a.tl && step == a.tl_step) ? a.tl + MK_TLH + 10 : nullptr;
            sa.mt_resident = step > 0;   // this CTA's shared copy of the mt19937 words is current
            MK_STAMP(MK_TLH + 2);
            const int t = sample_row_block(sa, 0, smem);
            MK_STAMP(MK_TLH + 3);
            if (tid == 0) {
                const int stop = (t == a.stop_token && !a.ignore_stop) || cancelled || t < 0;
                *bTOK = (t & 0xffff) | (stop ? 0x10000 : 0);
                *a.steps_done = step + 1;
            }
            mk_release(cTOK);
        }
        {
            if (!mk_acquire(cTOK, (unsigned) (step + 1), a)) MK_BAIL;
            MK_STAMP(MK_TLH + 4);
            if (tid == 0) tokv = __ldcg(bTOK);
            __syncthreads();
            const int tv = tokv;
            if (tv & 0x10000) MK_BAIL;
            tok = tv & 0xffff;
        }
    }
    MK_BAIL;
}
