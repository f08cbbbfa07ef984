// kernels.cuh — multi-kernel T3 step: activation prep, dequant GEMV with
// fused epilogues, decode attention, embeddings, fused sampler.
//
// Weight row layouts in HBM (written by t3b_op_repack / t3b_create from the
// GGUF blocks, which are 18 B (Q4_0) / 34 B (Q8_0) and so never 16-byte
// aligned):
//   Q4_0: [K/2 bytes: block b's 16 nibble bytes at 16*b][K/32 f16 scales]
//   Q8_0: [K bytes: block b's 32 int8 at 32*b]           [K/32 f16 scales]
//   F16 : [K halves]
// Every row is a multiple of 16 bytes, so a warp streams a row with 128-bit
// loads and each lane owns whole 32-element blocks.
#pragma once

#include "common.cuh"
#include "t3_expf.h"
#include "../../include/t3b200.h"
#include <cuda.h>   // CUtensorMap (TMA descriptors)

// ---------------------------------------------------------------------------
// GEMV epilogue
// ---------------------------------------------------------------------------
enum { EPI_BIAS = 0, EPI_GELU = 1, EPI_RESID = 2, EPI_QKV = 3 };

struct GemvEpi {
    int kind;
    float * y; int ldy;
    const float * bias;
    const float * res; int ldres;
    // EPI_QKV: append K/V (columns D..3D) to the f16 caches.  Cache row
    // layout: [layer][K,V][head][max_ctx][64].
    __half * kv; size_t row_elems; size_t layer_off; size_t v_off;
    const int * row_of;  // activation row -> cache row
    const int * pos;     // activation row -> position
    const int * y_row;   // nullable: activation row -> output row of y
    int max_ctx; int D;
    unsigned * err;
    // gemm_q_mma_kernel with EPI_GELU only (nullable): write the output rows
    // re-quantised to Q8_0 (the next GEMM's activation prep) instead of y
    int8_t * qx; float * qd; int * qs; int qK;
};

__device__ __forceinline__ void epi_store(const GemvEpi & e, int m, int n, float acc) {
    float v = e.bias ? __fadd_rn(acc, e.bias[n]) : acc;
    if (e.kind == EPI_GELU) v = gelu_ggml(v);
    else if (e.kind == EPI_RESID) v = __fadd_rn(v, e.res[(size_t) m * e.ldres + n]);
    e.y[(size_t) (e.y_row ? e.y_row[m] : m) * e.ldy + n] = v;
    if (e.kind == EPI_QKV && n >= e.D) {
        const int which = n >= 2 * e.D ? 1 : 0;
        const int rem = n - e.D - which * e.D;
        const int h = rem >> 6, d = rem & 63;
        const int p = e.pos[m];
        if (p < 0 || p >= e.max_ctx) { atomicOr(e.err, T3B_DEVERR_POS); return; }
        __half * base = e.kv + (size_t) e.row_of[m] * e.row_elems + e.layer_off + (which ? e.v_off : 0);
        base[((size_t) h * e.max_ctx + p) * T3B_HD + d] = __float2half_rn(v);
    }
}

// ---------------------------------------------------------------------------
// Activation prep: optional LayerNorm, then Q8_0 re-quantisation (for
// Q4_0/Q8_0 weights) or f16 rounding (for F16 weights) — what ggml's CPU
// backend does to src1 before a quantised / f16 mul_mat.
// One CTA of 256 threads per row; dynamic smem = K floats.
// ---------------------------------------------------------------------------
// rows x n floats from global memory (row stride ld) into shared memory
// (row stride n), by the whole block, with four loads per thread in flight
// (16-byte ones when every row start is 16-byte aligned): one memory round
// trip for up to 4 * blockDim.x loads, where a plain strided loop waits on
// each of its K / blockDim.x iterations in turn.
__device__ __forceinline__ void rows_to_smem(float * dst, const float * __restrict__ src, int ld, int rows, int n) {
    const int tid = threadIdx.x, nth = blockDim.x;
    if (((((uintptr_t) src) | ((uintptr_t) dst)) & 15) == 0 && (n & 3) == 0 && (ld & 3) == 0) {
        const int n4 = n >> 2, tot = rows * n4;
        for (int q0 = tid; q0 < tot; q0 += 4 * nth) {
            float4 t[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int q = q0 + u * nth;
                if (q < tot) t[u] = *(const float4 *) (src + (size_t) (q / n4) * ld + 4 * (q % n4));
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int q = q0 + u * nth;
                if (q < tot) ((float4 *) dst)[q] = t[u];
            }
        }
    } else {
        const int tot = rows * n;
        for (int q0 = tid; q0 < tot; q0 += 4 * nth) {
            float t[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int q = q0 + u * nth;
                if (q < tot) t[u] = src[(size_t) (q / n) * ld + q % n];
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int q = q0 + u * nth;
                if (q < tot) dst[q] = t[u];
            }
        }
    }
}

__device__ __forceinline__ double block_sum_d(double v, double * red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    double r = lane < nw ? red[lane] : 0.0;
#pragma unroll
    for (int o = 16; o; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    return r;
}

__global__ __launch_bounds__(256) void prep_act_kernel(
        const float * __restrict__ x, int ldx, int K, const float * __restrict__ g,
        const float * __restrict__ b, float eps, int qmode,
        int8_t * __restrict__ xq, float * __restrict__ xd, int * __restrict__ xs,
        __half * __restrict__ xh) {
    extern __shared__ __align__(16) float row[];
    __shared__ double redd[32];
    const int m = blockIdx.x, tid = threadIdx.x;
    rows_to_smem(row, x + (size_t) m * ldx, ldx, 1, K);
    __syncthreads();
    if (g) {
        double s = 0.0;
        for (int i = tid; i < K; i += blockDim.x) s += (double) row[i];
        s = block_sum_d(s, redd);
        const float mean = (float) (s / K);
        double s2 = 0.0;
        for (int i = tid; i < K; i += blockDim.x) {
            const float v = __fsub_rn(row[i], mean);
            s2 += (double) __fmul_rn(v, v);
        }
        s2 = block_sum_d(s2, redd);
        const float var = (float) (s2 / K);
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll 4
        for (int i = tid; i < K; i += blockDim.x) {   // unrolled: the g / b loads of 4 iterations in flight
            const float v = __fsub_rn(row[i], mean);
            row[i] = __fadd_rn(__fmul_rn(__fmul_rn(v, scale), g[i]), b[i]);
        }
        __syncthreads();
    }
    if (qmode == 1) {
        const int lane = tid & 31, w = tid >> 5, nw = blockDim.x >> 5;
        for (int blk = w; blk < K / 32; blk += nw) {
            const float v = row[blk * 32 + lane];
            const float amax = warp_max(fabsf(v));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            const int q = (int) roundf(__fmul_rn(v, id));
            xq[(size_t) m * K + blk * 32 + lane] = (int8_t) q;
            const int s = warp_sum_i(q);
            if (lane == 0) {
                xd[(size_t) m * (K / 32) + blk] = __half2float(__float2half_rn(d));
                xs[(size_t) m * (K / 32) + blk] = s;
            }
        }
    } else {
        for (int i = tid; i < K; i += blockDim.x) xh[(size_t) m * K + i] = __float2half_rn(row[i]);
    }
}

// ---------------------------------------------------------------------------
// Quantised GEMV (Q4_0 / Q8_0 weights x Q8_0 activations), integer dot per
// 32-block with dp4a, float accumulation of sumi * d_w * d_x per block.
// CTA = 8 warps; warp w owns RPW consecutive output rows; lanes stride the
// K/32 blocks.  grid = (ceil(N / (8*RPW)), ceil(M / MT)).
// dynamic smem: MT*K int8 + MT*(K/32)*(4+4).
// ---------------------------------------------------------------------------
template <int WT, int MT, int RPW>
__global__ __launch_bounds__(256) void gemv_q_kernel(
        const uint8_t * __restrict__ W, int N, int K, int rb,
        const int8_t * __restrict__ xq, const float * __restrict__ xd, const int * __restrict__ xs,
        int M, GemvEpi e) {
    extern __shared__ __align__(16) uint8_t sm[];
    const int nb = K / 32;
    int8_t * sq = (int8_t *) sm;
    float * sd = (float *) (sm + MT * K);
    int * ss = (int *) (sd + MT * nb);
    const int m0 = blockIdx.y * MT;
    const int mt = min(MT, M - m0);
    const int tid = threadIdx.x;
    for (int i = tid; i < mt * K / 16; i += blockDim.x)
        ((uint4 *) sq)[i] = ((const uint4 *) (xq + (size_t) m0 * K))[i];
    for (int i = tid; i < mt * nb; i += blockDim.x) {
        sd[i] = xd[(size_t) m0 * nb + i];
        ss[i] = xs[(size_t) m0 * nb + i];
    }
    __syncthreads();
    const int lane = tid & 31, warp = tid >> 5;
    const int row0 = (blockIdx.x * 8 + warp) * RPW;
    float acc[RPW][MT];
#pragma unroll
    for (int i = 0; i < RPW; ++i)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[i][m] = 0.0f;

    for (int b = lane; b < nb; b += 32) {
#pragma unroll
        for (int i = 0; i < RPW; ++i) {
            const int r = row0 + i;
            if (r >= N) continue;
            const uint8_t * wr = W + (size_t) r * rb;
            if (WT == T3B_Q4_0) {
                const uint4 qv = __ldg((const uint4 *) (wr + b * 16));
                const float dw = __half2float(__ldg((const __half *) (wr + K / 2 + b * 2)));
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m >= mt) break;
                    const int * xv = (const int *) (sq + m * K + b * 32);
                    int si = 0;
                    si = __dp4a((int) (qv.x & 0x0F0F0F0Fu), xv[0], si);
                    si = __dp4a((int) ((qv.x >> 4) & 0x0F0F0F0Fu), xv[4], si);
                    si = __dp4a((int) (qv.y & 0x0F0F0F0Fu), xv[1], si);
                    si = __dp4a((int) ((qv.y >> 4) & 0x0F0F0F0Fu), xv[5], si);
                    si = __dp4a((int) (qv.z & 0x0F0F0F0Fu), xv[2], si);
                    si = __dp4a((int) ((qv.z >> 4) & 0x0F0F0F0Fu), xv[6], si);
                    si = __dp4a((int) (qv.w & 0x0F0F0F0Fu), xv[3], si);
                    si = __dp4a((int) ((qv.w >> 4) & 0x0F0F0F0Fu), xv[7], si);
                    si -= 8 * ss[m * nb + b];
                    acc[i][m] = __fadd_rn(acc[i][m], __fmul_rn(__fmul_rn((float) si, dw), sd[m * nb + b]));
                }
            } else {
                const uint4 q0 = __ldg((const uint4 *) (wr + b * 32));
                const uint4 q1 = __ldg((const uint4 *) (wr + b * 32 + 16));
                const float dw = __half2float(__ldg((const __half *) (wr + K + b * 2)));
#pragma unroll
                for (int m = 0; m < MT; ++m) {
                    if (m >= mt) break;
                    const int * xv = (const int *) (sq + m * K + b * 32);
                    int si = 0;
                    si = __dp4a((int) q0.x, xv[0], si);
                    si = __dp4a((int) q0.y, xv[1], si);
                    si = __dp4a((int) q0.z, xv[2], si);
                    si = __dp4a((int) q0.w, xv[3], si);
                    si = __dp4a((int) q1.x, xv[4], si);
                    si = __dp4a((int) q1.y, xv[5], si);
                    si = __dp4a((int) q1.z, xv[6], si);
                    si = __dp4a((int) q1.w, xv[7], si);
                    acc[i][m] = __fadd_rn(acc[i][m], __fmul_rn(__fmul_rn((float) si, dw), sd[m * nb + b]));
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
        const int r = row0 + i;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const float v = warp_sum(acc[i][m]);
            if (lane == 0 && r < N && m < mt) epi_store(e, m0 + m, r, v);
        }
    }
}

// ---------------------------------------------------------------------------
// Quantised skinny GEMM for many activation rows (batched decode, M >= 16):
// int8 tensor-core MMAs, mma.sync m16n8k32 — one instruction is exactly one
// 32-element block's integer dot products for a 16 x 8 tile — followed by the
// same per-block rescale as the GEMV, sumf += ((float) sumi * d_w) * d_x,
// accumulated in registers in block order.  Per-32 f16 scales force a
// rescale after every K = 32 step, which is why the accumulators live in
// registers rather than in tensor memory.
// CTA tile BM (64 or 32) activation rows x 32 weight rows; WARPS warps, two
// along M and WARPS / 2 along N: 4 warps with 32 x 16 / 16 x 16 warp tiles,
// or 8 warps with 16 x 8 ones (one MMA tile each, for the 32-row tile when
// one CTA per SM would leave the schedulers idle).  K is staged four blocks
// (128 elements) at a time in NS cp.async buffers; smem rows are padded by
// 16 bytes so the fragment loads of a warp hit 32 distinct banks.
// grid = (ceil(N / 32), ceil(M / BM)).
// ---------------------------------------------------------------------------
#define GQ_BM 64
#define GQ_BN 32
#define GQ_KB 4                       // 32-element blocks per stage
#define GQ_AROW (GQ_KB * 32 + 16)     // bytes per staged activation row
#define GQ_BROW (GQ_KB * 32 + 16)     // bytes per staged weight row (Q4_0 uses half)

__device__ __forceinline__ void cp_async16(void * smem, const void * gmem, bool pred) {
    const unsigned s = (unsigned) __cvta_generic_to_shared(smem);
    const int sz = pred ? 16 : 0;     // 0: fill with zeros, read nothing
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async8(void * smem, const void * gmem, bool pred) {
    const unsigned s = (unsigned) __cvta_generic_to_shared(smem);
    const int sz = pred ? 8 : 0;
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(s), "l"(gmem), "r"(sz) : "memory");
}

template <int WT>
__device__ __forceinline__ void mma_s8(int (&c)[4], const int (&a)[4], int b0, int b1) {
    if (WT == T3B_Q4_0)   // unsigned nibbles x signed activations
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                     "{%10,%11,%12,%13};"
                     : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
    else
        asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                     "{%10,%11,%12,%13};"
                     : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
                     : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

template <int WT, int BM, int WARPS>
__global__ __launch_bounds__(32 * WARPS) void gemm_q_mma_kernel(
        const uint8_t * __restrict__ W, int N, int K, int rb,
        const int8_t * __restrict__ xq, const float * __restrict__ xd, const int * __restrict__ xs,
        int M, GemvEpi e) {
    constexpr int QB = WT == T3B_Q4_0 ? 16 : 32;          // weight bytes per block
    constexpr int MT = BM / 32;                           // 16-row MMA tiles per warp (2 warps along M)
    constexpr int WN = WARPS / 2;                         // warps along N
    constexpr int NT = GQ_BN / (8 * WN);                  // 8-column MMA tiles per warp
    constexpr int NTHR = 32 * WARPS;
    constexpr int NS = BM == 32 ? 4 : 3;                  // cp.async stages in flight (static smem <= 48 KB)
    __shared__ __align__(16) int8_t As[NS][BM][GQ_AROW];
    __shared__ __align__(16) uint8_t Bs[NS][GQ_BN][GQ_BROW];
    __shared__ __align__(16) float Ds[NS][BM][GQ_KB];   // activation block scales
    __shared__ __align__(16) int Ss[NS][BM][GQ_KB];     // activation block sums (Q4_0)
    __shared__ __align__(16) __half Dw[NS][GQ_BN][GQ_KB];  // weight block scales
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int wm = warp / WN, wn = warp % WN;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * GQ_BN;
    const int nb = K / 32;
    const int nstage = nb / GQ_KB;

    auto load_stage = [&](int s, int st) {
        const int kb = st * GQ_KB;                         // first block of the stage
        // activations: BM rows x 128 bytes = 8 BM chunks of 16 bytes
#pragma unroll
        for (int u = 0; u < (8 * BM + NTHR - 1) / NTHR; ++u) {
            const int c = tid + u * NTHR;
            if (c < 8 * BM) {
                const int r = c >> 3, q = c & 7;
                const bool ok = m0 + r < M;
                cp_async16(&As[s][r][q * 16], xq + (size_t) (ok ? m0 + r : 0) * K + kb * 32 + q * 16, ok);
            }
        }
        // activation scales and sums: BM rows x 16 bytes each
        if (tid < BM) {
            const bool ok = m0 + tid < M;
            const size_t o = (size_t) (ok ? m0 + tid : 0) * nb + kb;
            cp_async16(&Ds[s][tid][0], xd + o, ok);
            if (WT == T3B_Q4_0) cp_async16(&Ss[s][tid][0], xs + o, ok);
        }
        // weights: 32 rows x (4 * QB) bytes
        constexpr int CPR = GQ_KB * QB / 16;              // chunks per row
#pragma unroll
        for (int u = 0; u < (GQ_BN * CPR + NTHR - 1) / NTHR; ++u) {
            const int c = tid + u * NTHR;
            if (c < GQ_BN * CPR) {
                const int r = c / CPR, q = c % CPR;
                const bool ok = n0 + r < N;
                cp_async16(&Bs[s][r][q * 16], W + (size_t) (ok ? n0 + r : 0) * rb + kb * QB + q * 16, ok);
            }
        }
        if (tid < GQ_BN) {
            const bool ok = n0 + tid < N;
            const uint8_t * sc = W + (size_t) (ok ? n0 + tid : 0) * rb + (size_t) nb * QB + kb * 2;
            cp_async8(&Dw[s][tid][0], sc, ok);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };

    float acc[MT][NT][4];
#pragma unroll
    for (int i = 0; i < MT; ++i)
#pragma unroll
        for (int j = 0; j < NT; ++j)
#pragma unroll
            for (int k = 0; k < 4; ++k) acc[i][j][k] = 0.0f;

    // NS - 1 stages in flight ahead of the one being consumed; every
    // iteration commits one group (empty at the tail), so "all but the
    // newest NS - 1 groups" is always the current stage
#pragma unroll
    for (int p = 0; p < NS - 1; ++p) {
        if (p < nstage) load_stage(p, p);
        else asm volatile("cp.async.commit_group;" ::: "memory");
    }
    for (int st = 0; st < nstage; ++st) {
        const int s = st % NS;
        if (st + NS - 1 < nstage) load_stage((st + NS - 1) % NS, st + NS - 1);
        else asm volatile("cp.async.commit_group;" ::: "memory");
        if (NS == 4) asm volatile("cp.async.wait_group 3;" ::: "memory");
        else asm volatile("cp.async.wait_group 2;" ::: "memory");
        __syncthreads();
#pragma unroll
        for (int bb = 0; bb < GQ_KB; ++bb) {
            int a[MT][4];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const int r = wm * (16 * MT) + mt * 16 + g;
                a[mt][0] = *(const int *) &As[s][r][bb * 32 + t * 4];
                a[mt][1] = *(const int *) &As[s][r + 8][bb * 32 + t * 4];
                a[mt][2] = *(const int *) &As[s][r][bb * 32 + 16 + t * 4];
                a[mt][3] = *(const int *) &As[s][r + 8][bb * 32 + 16 + t * 4];
            }
            int b[NT][2];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int r = wn * (8 * NT) + nt * 8 + g;
                if (WT == T3B_Q4_0) {
                    // block byte j holds elements j (low nibble) and j + 16 (high)
                    const unsigned wv = *(const unsigned *) &Bs[s][r][bb * 16 + t * 4];
                    b[nt][0] = (int) (wv & 0x0F0F0F0Fu);
                    b[nt][1] = (int) ((wv >> 4) & 0x0F0F0F0Fu);
                } else {
                    b[nt][0] = *(const int *) &Bs[s][r][bb * 32 + t * 4];
                    b[nt][1] = *(const int *) &Bs[s][r][bb * 32 + 16 + t * 4];
                }
            }
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const int r0 = wm * (16 * MT) + mt * 16 + g;
                const float dx0 = Ds[s][r0][bb], dx1 = Ds[s][r0 + 8][bb];
                int sx0 = 0, sx1 = 0;
                if (WT == T3B_Q4_0) { sx0 = 8 * Ss[s][r0][bb]; sx1 = 8 * Ss[s][r0 + 8][bb]; }
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    int c[4];
                    mma_s8<WT>(c, a[mt], b[nt][0], b[nt][1]);
                    const int cn = wn * (8 * NT) + nt * 8 + 2 * t;
                    const float dw0 = __half2float(Dw[s][cn][bb]), dw1 = __half2float(Dw[s][cn + 1][bb]);
                    // c0, c1: row g, columns 2t, 2t+1; c2, c3: row g + 8
                    acc[mt][nt][0] = __fadd_rn(acc[mt][nt][0], __fmul_rn(__fmul_rn((float) (c[0] - sx0), dw0), dx0));
                    acc[mt][nt][1] = __fadd_rn(acc[mt][nt][1], __fmul_rn(__fmul_rn((float) (c[1] - sx0), dw1), dx0));
                    acc[mt][nt][2] = __fadd_rn(acc[mt][nt][2], __fmul_rn(__fmul_rn((float) (c[2] - sx1), dw0), dx1));
                    acc[mt][nt][3] = __fadd_rn(acc[mt][nt][3], __fmul_rn(__fmul_rn((float) (c[3] - sx1), dw1), dx1));
                }
            }
        }
        __syncthreads();   // the buffer is refilled by the next stage's load
    }
    if (e.qx) {
        // bias + GELU, then Q8_0 of each row's 32-wide block (this CTA's
        // columns are exactly one block): the tile goes through shared memory
        float (*Tt)[GQ_BN + 1] = (float (*)[GQ_BN + 1]) & As[0][0][0];   // BM x 33 floats fit in As[0]
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int ml = wm * (16 * MT) + mt * 16 + g + (i >> 1) * 8;
                    const int nl = wn * (8 * NT) + nt * 8 + 2 * t + (i & 1);
                    const float b = e.bias ? e.bias[n0 + nl] : 0.0f;
                    Tt[ml][nl] = gelu_ggml(e.bias ? __fadd_rn(acc[mt][nt][i], b) : acc[mt][nt][i]);
                }
        __syncthreads();
        const int nbk = e.qK / 32;
        for (int ml = warp * (BM / WARPS); ml < warp * (BM / WARPS) + BM / WARPS; ++ml) {
            const int m = m0 + ml;
            if (m >= M) break;   // uniform over the warp
            const float v = Tt[ml][lane];
            const float amax = warp_max(fabsf(v));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            const int q = (int) roundf(__fmul_rn(v, id));
            e.qx[(size_t) m * e.qK + n0 + lane] = (int8_t) q;
            const int sq = warp_sum_i(q);
            if (lane == 0) {
                e.qd[(size_t) m * nbk + n0 / 32] = __half2float(__float2half_rn(d));
                e.qs[(size_t) m * nbk + n0 / 32] = sq;
            }
        }
        return;
    }
    // plain epilogue through the same tile: each warp then stores 32
    // consecutive columns of a row (coalesced), with one copy of the
    // epilogue's code instead of sixteen unrolled ones
    float (*Tt)[GQ_BN + 1] = (float (*)[GQ_BN + 1]) & As[0][0][0];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i)
                Tt[wm * (16 * MT) + mt * 16 + g + (i >> 1) * 8][wn * (8 * NT) + nt * 8 + 2 * t + (i & 1)] = acc[mt][nt][i];
    __syncthreads();
    const int rows = min(BM, M - m0);
#pragma unroll 1
    for (int q = threadIdx.x; q < rows * GQ_BN; q += blockDim.x) {
        const int r = q / GQ_BN, c = q % GQ_BN;
        if (n0 + c < N) epi_store(e, m0 + r, n0 + c, Tt[r][c]);
    }
}

// F16 weights x f16-rounded activations, f32 accumulation (each f16*f16
// product is exact in f32).  Lanes stride 8-element chunks.
template <int MT, int RPW>
__global__ __launch_bounds__(256) void gemv_f16_kernel(
        const __half * __restrict__ W, int N, int K, const __half * __restrict__ xh, int M, GemvEpi e) {
    extern __shared__ __align__(16) uint8_t sm[];
    __half * sx = (__half *) sm;
    const int m0 = blockIdx.y * MT;
    const int mt = min(MT, M - m0);
    const int tid = threadIdx.x;
    for (int i = tid; i < mt * K / 8; i += blockDim.x)
        ((uint4 *) sx)[i] = ((const uint4 *) (xh + (size_t) m0 * K))[i];
    __syncthreads();
    const int lane = tid & 31, warp = tid >> 5;
    const int row0 = (blockIdx.x * 8 + warp) * RPW;
    float acc[RPW][MT];
#pragma unroll
    for (int i = 0; i < RPW; ++i)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[i][m] = 0.0f;
    // unrolled: the weight loads of four chunks per row are in flight at once
    // (K = 4096 is 16 chunks per lane; one at a time they were 16 round trips)
#pragma unroll 4
    for (int c = lane; c < K / 8; c += 32) {
#pragma unroll
        for (int i = 0; i < RPW; ++i) {
            const int r = row0 + i;
            if (r >= N) continue;
            const uint4 wv = __ldg((const uint4 *) (W + (size_t) r * K + c * 8));
            const __half2 * wp = (const __half2 *) &wv;
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                if (m >= mt) break;
                const uint4 xv = *(const uint4 *) (sx + m * K + c * 8);
                const __half2 * xp = (const __half2 *) &xv;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 wf = __half22float2(wp[j]), xf = __half22float2(xp[j]);
                    acc[i][m] = fmaf(wf.x, xf.x, acc[i][m]);
                    acc[i][m] = fmaf(wf.y, xf.y, acc[i][m]);
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
        const int r = row0 + i;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const float v = warp_sum(acc[i][m]);
            if (lane == 0 && r < N && m < mt) epi_store(e, m0 + m, r, v);
        }
    }
}

// ---------------------------------------------------------------------------
// Few-row matrix-vector product in ONE launch (M <= 4): the activation prep
// of prep_act_kernel (optional LayerNorm, then Q8_0 blocks or f16 rounding,
// the same arithmetic in the same order) runs in every CTA over its MT rows
// in shared memory, followed by the dot of gemv_q_kernel / gemv_f16_kernel
// (same lane order, so the result is identical to the two-launch path).
// Before it reads the activations, each thread issues the loads of the first
// GP_PF weight blocks (Q4_0/Q8_0: 32 elements) or chunks (F16: 8 elements) of
// its rows, so the weight stream from HBM overlaps the prep.
// CTA = 8 warps, warp w owns RPW consecutive rows; grid = (ceil(N /
// (8 RPW)), ceil(M / MT)); dynamic smem = gemv_prep_smem(WT, MT, K).
// ---------------------------------------------------------------------------
#define GP_PF 4
__host__ __device__ constexpr size_t gemv_prep_smem(int wt, int mt, int K) {
    return (size_t) mt * K * 4 + (wt == T3B_F16 ? (size_t) mt * K * 2 : (size_t) mt * K + (size_t) mt * (K / 32) * 8);
}

template <int WT, int MT, int RPW>
__global__ __launch_bounds__(256) void gemv_prep_kernel(
        const uint8_t * __restrict__ W, int N, int K, int rb, const float * __restrict__ x, int ldx,
        const float * __restrict__ g, const float * __restrict__ b, float eps, int M, GemvEpi e) {
    extern __shared__ __align__(16) uint8_t sm[];
    constexpr int NW = 8;                                       // warps
    constexpr int QW = WT == T3B_Q8_0 ? 2 : 1;                  // 16-byte words per prefetched unit
    constexpr int PF = WT == T3B_F16 ? 2 * GP_PF : GP_PF;       // units prefetched per row and lane
    __shared__ double red[MT][NW];
    const int nb = K / 32;
    const int nu = WT == T3B_F16 ? K / 8 : nb;                  // units per row
    float * rows = (float *) sm;                                // [MT][K] f32
    int8_t * sq = (int8_t *) (rows + (size_t) MT * K);          // [MT][K]  (Q4_0 / Q8_0)
    float * sd = (float *) (sq + (size_t) MT * K);              // [MT][nb]
    int * ss = (int *) (sd + (size_t) MT * nb);                 // [MT][nb]
    __half * sx = (__half *) (rows + (size_t) MT * K);          // [MT][K]  (F16)
    const int m0 = blockIdx.y * MT;
    const int mt = min(MT, M - m0);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int row0 = (blockIdx.x * NW + warp) * RPW;

    // (1) weight prefetch
    uint4 pw[RPW][PF][QW];
    float pd[RPW][PF];
#pragma unroll
    for (int i = 0; i < RPW; ++i)
#pragma unroll
        for (int j = 0; j < PF; ++j) {
            const int u = lane + 32 * j, r = row0 + i;
            pd[i][j] = 0.0f;
            if (r < N && u < nu) {
                const uint8_t * wr = W + (size_t) r * rb;
                if (WT == T3B_Q4_0) {
                    pw[i][j][0] = __ldg((const uint4 *) (wr + u * 16));
                    pd[i][j] = __half2float(__ldg((const __half *) (wr + K / 2 + u * 2)));
                } else if (WT == T3B_Q8_0) {
                    pw[i][j][0] = __ldg((const uint4 *) (wr + u * 32));
                    pw[i][j][QW - 1] = __ldg((const uint4 *) (wr + u * 32 + 16));
                    pd[i][j] = __half2float(__ldg((const __half *) (wr + K + u * 2)));
                } else {
                    pw[i][j][0] = __ldg((const uint4 *) (wr + u * 16));
                }
            }
        }

    // launched with programmatic stream serialization: the weight loads above
    // overlap the previous kernel's tail; everything it writes (x, the
    // residual, the caches) is read only after this wait.  The next kernel
    // may start its own prologue now.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

    // (2) activation prep of rows m0 .. m0 + mt - 1 (prep_act_kernel per row)
    rows_to_smem(rows, x + (size_t) m0 * ldx, ldx, mt, K);
    __syncthreads();
    if (g) {
        double s[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            s[m] = 0.0;
            if (m < mt)
                for (int i = tid; i < K; i += blockDim.x) s[m] += (double) rows[(size_t) m * K + i];
        }
        // block_sum_d for every row at once (same order per row)
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
            for (int o = 16; o; o >>= 1) s[m] += __shfl_xor_sync(0xffffffffu, s[m], o);
        if (lane == 0)
#pragma unroll
            for (int m = 0; m < MT; ++m) red[m][warp] = s[m];
        __syncthreads();
        float mean[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            double r = lane < NW ? red[m][lane] : 0.0;
#pragma unroll
            for (int o = 16; o; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
            mean[m] = (float) (r / K);
        }
        __syncthreads();   // red is reused
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            s[m] = 0.0;
            if (m < mt)
#pragma unroll 4
                for (int i = tid; i < K; i += blockDim.x) {   // the g / b loads of 4 iterations in flight
                    const float v = __fsub_rn(rows[(size_t) m * K + i], mean[m]);
                    s[m] += (double) __fmul_rn(v, v);
                }
        }
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
            for (int o = 16; o; o >>= 1) s[m] += __shfl_xor_sync(0xffffffffu, s[m], o);
        if (lane == 0)
#pragma unroll
            for (int m = 0; m < MT; ++m) red[m][warp] = s[m];
        __syncthreads();
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            double r = lane < NW ? red[m][lane] : 0.0;
#pragma unroll
            for (int o = 16; o; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
            const float var = (float) (r / K);
            const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
            if (m < mt)
                for (int i = tid; i < K; i += blockDim.x) {
                    const float v = __fsub_rn(rows[(size_t) m * K + i], mean[m]);
                    rows[(size_t) m * K + i] = __fadd_rn(__fmul_rn(__fmul_rn(v, scale), g[i]), b[i]);
                }
        }
        __syncthreads();
    }
    if (WT != T3B_F16) {
        // Q8_0 blocks, eight lanes per block (four elements each), every
        // group of the CTA on its own block at once: the same maximum,
        // scale, rounding and integer sum as prep_act_kernel's warp per block.
        // K % 256 == 0 (the launcher's condition): mt * nb is a multiple of 8,
        // so each warp's four groups are all in or all out of an iteration
        // and every lane takes the full-mask shuffles.
        const int grp = tid >> 3, sub = tid & 7;
#pragma unroll 4
        for (int q = grp; q < mt * nb; q += 32) {
            const int m = q / nb, blk = q % nb;
            const float4 v = *(const float4 *) (rows + (size_t) m * K + blk * 32 + sub * 4);
            float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            const float d = __fdiv_rn(mx, 127.0f);
            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            const int q0 = (int) roundf(__fmul_rn(v.x, id)), q1 = (int) roundf(__fmul_rn(v.y, id));
            const int q2 = (int) roundf(__fmul_rn(v.z, id)), q3 = (int) roundf(__fmul_rn(v.w, id));
            *(int *) (sq + (size_t) m * K + blk * 32 + sub * 4) =
                (q0 & 0xff) | ((q1 & 0xff) << 8) | ((q2 & 0xff) << 16) | ((q3 & 0xff) << 24);
            int sum = q0 + q1 + q2 + q3;
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            if (sub == 0) {
                sd[m * nb + blk] = __half2float(__float2half_rn(d));
                ss[m * nb + blk] = sum;
            }
        }
    } else {
        for (int i = tid; i < mt * K; i += blockDim.x) sx[i] = __float2half_rn(rows[i]);
    }
    __syncthreads();

    // (3) the dot, lanes striding the units in increasing order
    float acc[RPW][MT];
#pragma unroll
    for (int i = 0; i < RPW; ++i)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[i][m] = 0.0f;
    auto unit = [&](int i, int u, const uint4 (&w)[QW], float dw) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            if (m >= mt) break;
            if (WT == T3B_Q4_0) {
                const int * xv = (const int *) (sq + (size_t) m * K + u * 32);
                const uint4 qv = w[0];
                int si = 0;
                si = __dp4a((int) (qv.x & 0x0F0F0F0Fu), xv[0], si);
                si = __dp4a((int) ((qv.x >> 4) & 0x0F0F0F0Fu), xv[4], si);
                si = __dp4a((int) (qv.y & 0x0F0F0F0Fu), xv[1], si);
                si = __dp4a((int) ((qv.y >> 4) & 0x0F0F0F0Fu), xv[5], si);
                si = __dp4a((int) (qv.z & 0x0F0F0F0Fu), xv[2], si);
                si = __dp4a((int) ((qv.z >> 4) & 0x0F0F0F0Fu), xv[6], si);
                si = __dp4a((int) (qv.w & 0x0F0F0F0Fu), xv[3], si);
                si = __dp4a((int) ((qv.w >> 4) & 0x0F0F0F0Fu), xv[7], si);
                si -= 8 * ss[m * nb + u];
                acc[i][m] = __fadd_rn(acc[i][m], __fmul_rn(__fmul_rn((float) si, dw), sd[m * nb + u]));
            } else if (WT == T3B_Q8_0) {
                const int * xv = (const int *) (sq + (size_t) m * K + u * 32);
                const uint4 q0 = w[0], q1 = w[QW - 1];
                int si = 0;
                si = __dp4a((int) q0.x, xv[0], si);
                si = __dp4a((int) q0.y, xv[1], si);
                si = __dp4a((int) q0.z, xv[2], si);
                si = __dp4a((int) q0.w, xv[3], si);
                si = __dp4a((int) q1.x, xv[4], si);
                si = __dp4a((int) q1.y, xv[5], si);
                si = __dp4a((int) q1.z, xv[6], si);
                si = __dp4a((int) q1.w, xv[7], si);
                acc[i][m] = __fadd_rn(acc[i][m], __fmul_rn(__fmul_rn((float) si, dw), sd[m * nb + u]));
            } else {
                const __half2 * wp = (const __half2 *) &w[0];
                const uint4 xw = *(const uint4 *) (sx + (size_t) m * K + u * 8);
                const __half2 * xp = (const __half2 *) &xw;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float2 wf = __half22float2(wp[j]), xf = __half22float2(xp[j]);
                    acc[i][m] = fmaf(wf.x, xf.x, acc[i][m]);
                    acc[i][m] = fmaf(wf.y, xf.y, acc[i][m]);
                }
            }
        }
    };
    // units lane + 32 j: the prefetched ones, then the rest from global memory
    // (for each unit all rows, as in the two-launch kernels)
#pragma unroll
    for (int j = 0; j < PF; ++j) {
        const int u = lane + 32 * j;
        if (u >= nu) break;
#pragma unroll
        for (int i = 0; i < RPW; ++i)
            if (row0 + i < N) unit(i, u, pw[i][j], pd[i][j]);
    }
    for (int u = lane + 32 * PF; u < nu; u += 32) {
#pragma unroll
        for (int i = 0; i < RPW; ++i) {
            const int r = row0 + i;
            if (r >= N) continue;
            const uint8_t * wr = W + (size_t) r * rb;
            uint4 w[QW];
            float dw = 0.0f;
            if (WT == T3B_Q4_0) {
                w[0] = __ldg((const uint4 *) (wr + u * 16));
                dw = __half2float(__ldg((const __half *) (wr + K / 2 + u * 2)));
            } else if (WT == T3B_Q8_0) {
                w[0] = __ldg((const uint4 *) (wr + u * 32));
                w[QW - 1] = __ldg((const uint4 *) (wr + u * 32 + 16));
                dw = __half2float(__ldg((const __half *) (wr + K + u * 2)));
            } else {
                w[0] = __ldg((const uint4 *) (wr + u * 16));
            }
            unit(i, u, w, dw);
        }
    }
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
        const int r = row0 + i;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            const float v = warp_sum(acc[i][m]);
            if (lane == 0 && r < N && m < mt) epi_store(e, m0 + m, r, v);
        }
    }
}

// ---------------------------------------------------------------------------
// F16-weight GEMM on the 5th-generation tensor cores (tcgen05), M >= 16
// activation rows (batched decode, prefill): Y = W . xh with f16 weights and
// f16-rounded activations (ggml's F16 mul_mat arithmetic: every f16 x f16
// product is exact in f32), f32 accumulation in tensor memory.
//
// * Operands reach shared memory by TMA (cp.async.bulk.tensor, 2-D tensor
//   maps, no multicast) in the canonical K-major layout with the 128-byte
//   swizzle: one box of 64 halves x R rows per operand and stage, rows of
//   128 bytes, 8-row atoms of 1024 bytes whose 16-byte chunks the TMA unit
//   permutes by row (chunk ^ row % 8) and the MMA unit reads back the same
//   way.  The MMA for K columns 16 j .. 16 j + 15 starts 32 j bytes into the
//   atom.
// * A 4-stage ring with full/empty mbarriers: one thread issues the TMA
//   loads, waits for a stage, issues its four K = 16 MMAs (M = 128,
//   N = TF_BN) and commits them to the stage's empty barrier; a slot is
//   refilled once the MMAs that read it have completed.
// * Split-K over gridDim.z when the tiles alone do not fill the GPU: each
//   CTA writes its partial tile to a workspace and the last CTA of a tile
//   (completion counter) adds the partials in split order, so the result is
//   the same for every run.  The epilogue (bias / GELU / residual / K-V
//   append) runs once per output element.
// grid = (ceil(N / TF_BN), ceil(M / 128), splits), 128 threads: after the
// MMAs, thread t reads row t's accumulators with tcgen05.ld.
// ---------------------------------------------------------------------------
#define TF_BM 128
#define TF_BN 64
#define TF_BK 64                             // K elements per stage
#define TF_NS 4                              // stages in the ring
#define TF_A_STAGE (TF_BM * TF_BK * 2)       // 16 KB
#define TF_B_STAGE (TF_BN * TF_BK * 2)       // 8 KB
#define TF_SMEM (TF_NS * (TF_A_STAGE + TF_B_STAGE) + 256 + 1024)   // + alignment of the ring to 1024 bytes
#define TF_SPIN (1u << 26)   // polls before a wait gives up (well above a second of polling)

struct TfArgs {
    int M, N, K;
    int kchunk;           // K elements per split (a multiple of TF_BK)
    int splits;
    GemvEpi e;
    float * ws;           // splits > 1: [splits][M][N rounded up to TF_BN] partial tiles
    unsigned * cnt;       // splits > 1: per-tile completion counters (zero; reset by the last CTA)
};

// UMMA shared-memory descriptor, K-major, 128-byte swizzle (sm_100 version
// 1): 8-row groups 1024 bytes apart (SBO), leading offset unused (1)
__device__ __forceinline__ unsigned long long tf_desc(unsigned saddr) {
    return (unsigned long long) ((saddr >> 4) & 0x3FFFu) | (1ull << 16) | ((unsigned long long) (1024u >> 4) << 32) |
           (1ull << 46) | (2ull << 61);
}
// instruction descriptor: kind::f16, A = B = f16, D = f32, both K-major, M = 128, N = TF_BN
#define TF_IDESC ((1u << 4) | ((unsigned) (TF_BN >> 3) << 17) | ((unsigned) (TF_BM >> 4) << 24))

// bounded wait for phase `parity` of an mbarrier: non-blocking test_wait
// polls (the producer polls without sleeping; waiters in other warps back off)
__device__ __forceinline__ bool tf_wait(unsigned addr, unsigned parity, bool backoff = false) {
    for (unsigned spins = 0;; ++spins) {
        unsigned done;
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                     : "=r"(done) : "r"(addr), "r"(parity) : "memory");
        if (done) return true;
        if (spins >= TF_SPIN) return false;
        if (backoff) __nanosleep(64);
    }
}
__device__ __forceinline__ void tf_tma(unsigned dst, const void * tmap, int x, int y, unsigned mbar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(dst), "l"(tmap), "r"(x), "r"(y), "r"(mbar) : "memory");
}

__global__ __launch_bounds__(128, 1) void gemm_f16_tc_kernel(const __grid_constant__ CUtensorMap ta,
                                                             const __grid_constant__ CUtensorMap tb, TfArgs p) {
    extern __shared__ __align__(1024) unsigned char tf_raw[];
    // swizzle atoms need 1024-byte aligned stage buffers
    unsigned char * tf_sm = tf_raw + ((1024u - ((unsigned) __cvta_generic_to_shared(tf_raw) & 1023u)) & 1023u);
    unsigned char * As = tf_sm;                                   // [TF_NS][TF_A_STAGE]
    unsigned char * Bs = tf_sm + TF_NS * TF_A_STAGE;              // [TF_NS][TF_B_STAGE]
    unsigned long long * full = (unsigned long long *) (Bs + TF_NS * TF_B_STAGE);
    unsigned long long * empty = full + TF_NS;
    unsigned long long * done = empty + TF_NS;
    unsigned * tslot = (unsigned *) (done + 1);
    __shared__ int tf_ok, tf_last;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.y * TF_BM, n0 = blockIdx.x * TF_BN, split = blockIdx.z;
    const int kbeg = split * p.kchunk, nk = p.kchunk / TF_BK;

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"((unsigned) __cvta_generic_to_shared(tslot)), "r"((unsigned) TF_BN) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int i = 0; i < 2 * TF_NS + 1; ++i)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"((unsigned) __cvta_generic_to_shared(full + i)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        tf_ok = 1;
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const unsigned tbase = *tslot;

    // lane 0 of warp 0 drives the loads and MMAs; the rest of its warp waits
    // at __syncwarp (a spin of theirs would share the warp's issue with it)
    if (tid == 0) {
        const unsigned a0 = (unsigned) __cvta_generic_to_shared(As), b0 = (unsigned) __cvta_generic_to_shared(Bs);
        // stage i: the A box (64 halves x 128 rows) and the B box (64 x
        // TF_BN) of K columns kbeg + 64 i ..
        auto load = [&](int i) {
            const int sl = i % TF_NS, k = kbeg + i * TF_BK;
            const unsigned fb = (unsigned) __cvta_generic_to_shared(full + sl);
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(fb),
                         "r"((unsigned) (TF_A_STAGE + TF_B_STAGE)) : "memory");
            tf_tma(a0 + sl * TF_A_STAGE, &ta, k, m0, fb);
            tf_tma(b0 + sl * TF_B_STAGE, &tb, k, n0, fb);
        };
        for (int i = 0; i < TF_NS && i < nk; ++i) load(i);
        bool ok = true;
        for (int i = 0; i < nk && ok; ++i) {
            const int sl = i % TF_NS;
            ok = tf_wait((unsigned) __cvta_generic_to_shared(full + sl), (unsigned) (i / TF_NS) & 1u);
            if (!ok) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
            for (int j = 0; j < TF_BK / 16; ++j) {   // MMA j: K columns 16 j .. 16 j + 15, 32 j bytes into each row
                const unsigned long long da = tf_desc(a0 + sl * TF_A_STAGE + 32 * j);
                const unsigned long long db = tf_desc(b0 + sl * TF_B_STAGE + 32 * j);
                const unsigned acc = (i > 0 || j > 0) ? 1u : 0u;
                asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                             "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
                             ::"r"(tbase), "l"(da), "l"(db), "r"((unsigned) TF_IDESC), "r"(acc) : "memory");
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         ::"r"((unsigned) __cvta_generic_to_shared(empty + sl)) : "memory");
            // refill the slot of stage i - 1 once its MMAs are done
            if (i >= 1 && i - 1 + TF_NS < nk) {
                const int ps = (i - 1) % TF_NS;
                ok = tf_wait((unsigned) __cvta_generic_to_shared(empty + ps), (unsigned) ((i - 1) / TF_NS) & 1u);
                if (ok) load(i - 1 + TF_NS);
            }
        }
        if (!ok) { tf_ok = 0; if (p.e.err) atomicOr(p.e.err, T3B_DEVERR_TIMEOUT); }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     ::"r"((unsigned) __cvta_generic_to_shared(done)) : "memory");
    }
    if (warp == 0) __syncwarp();
    // every MMA of this CTA complete (a commit tracks all earlier MMAs)
    if (!tf_wait((unsigned) __cvta_generic_to_shared(done), 0u, true)) tf_ok = 0;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    float v[TF_BN];
#pragma unroll
    for (int c = 0; c < TF_BN / 32; ++c) {
        unsigned r[32];
        const unsigned ta_ = tbase + ((unsigned) (warp * 32) << 16) + (unsigned) (c * 32);
        asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
                     "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
                     : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                       "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
                       "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
                       "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                     : "r"(ta_) : "memory");
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < 32; ++j) v[c * 32 + j] = __uint_as_float(r[j]);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tbase), "r"((unsigned) TF_BN) : "memory");
    }
    // the accumulator row of this thread goes into a padded shared tile (the
    // ring is free: the MMAs that read it completed before the accumulator
    // was read); the split partials and the epilogue are then written and
    // read from it in coalesced order
    const int rows = min(TF_BM, p.M - m0);
    float * tile_s = (float *) As;   // [TF_BM][TF_BN + 1]
#pragma unroll
    for (int j = 0; j < TF_BN; ++j) tile_s[tid * (TF_BN + 1) + j] = v[j];
    __syncthreads();
    if (p.splits > 1) {
        // partial tile of this split: [split][M][ldw] with the row padded to
        // a multiple of TF_BN columns; a warp moves two rows of 64 columns
        // per float4 instruction (256 contiguous bytes each)
        constexpr int C4 = TF_BN / 4;                       // float4 per tile row
        constexpr int PT = TF_BM * C4 / TF_BM;              // float4 per thread (16)
        const int ldw = (p.N + TF_BN - 1) / TF_BN * TF_BN;
        if (tf_ok) {
#pragma unroll
            for (int j = 0; j < PT; ++j) {
                const int q = tid + j * TF_BM, r = q / C4, c = (q % C4) * 4;
                if (r < rows) {
                    const float * t = tile_s + r * (TF_BN + 1) + c;
                    *(float4 *) (p.ws + ((size_t) split * p.M + m0 + r) * ldw + n0 + c) = make_float4(t[0], t[1], t[2], t[3]);
                }
            }
        }
        __threadfence();
        __syncthreads();
        const int tile = blockIdx.y * gridDim.x + blockIdx.x;
        if (tid == 0) tf_last = atomicAdd(&p.cnt[tile], 1u) == (unsigned) (p.splits - 1);
        __syncthreads();
        if (!tf_last) return;
        __threadfence();
        // splits added in split order (0 + s0 + s1 + ...), each thread's 16
        // float4 of a split in flight at once
        float4 a4[PT];
#pragma unroll
        for (int j = 0; j < PT; ++j) a4[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int sp = 0; sp < p.splits; ++sp) {
            float4 t4[PT];
#pragma unroll
            for (int j = 0; j < PT; ++j) {
                const int q = tid + j * TF_BM, r = q / C4, c = (q % C4) * 4;
                t4[j] = r < rows ? __ldcg((const float4 *) (p.ws + ((size_t) sp * p.M + m0 + r) * ldw + n0 + c))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int j = 0; j < PT; ++j) {
                a4[j].x += t4[j].x; a4[j].y += t4[j].y; a4[j].z += t4[j].z; a4[j].w += t4[j].w;
            }
        }
        if (tid == 0) p.cnt[tile] = 0u;
#pragma unroll
        for (int j = 0; j < PT; ++j) {
            const int q = tid + j * TF_BM, r = q / C4, c = (q % C4) * 4;
            float * t = tile_s + r * (TF_BN + 1) + c;
            t[0] = a4[j].x; t[1] = a4[j].y; t[2] = a4[j].z; t[3] = a4[j].w;
        }
        __syncthreads();
    }
    // epilogue: each warp stores 32 consecutive columns of a row at a time,
    // with one copy of the epilogue's code rather than 64 unrolled ones,
    // which the CTA would fetch cold exactly once
    if (!tf_ok) return;              // CTA-uniform
#pragma unroll 1
    for (int q = tid; q < rows * TF_BN; q += TF_BM) {
        const int r = q / TF_BN, c = q % TF_BN;
        if (n0 + c < p.N) epi_store(p.e, m0 + r, n0 + c, tile_s[r * (TF_BN + 1) + c]);
    }
}

// Plain f32 matvec for the speaker projection (cond_spkr: K = 256).
__global__ void matvec_f32_kernel(const float * __restrict__ W, int N, int K, const float * __restrict__ x,
                                  const float * __restrict__ b, float * __restrict__ y) {
    const int lane = threadIdx.x & 31;
    const int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (r >= N) return;
    float acc = 0.0f;
    for (int k = lane; k < K; k += 32) acc = fmaf(W[(size_t) r * K + k], x[k], acc);
    acc = warp_sum(acc);
    if (lane == 0) y[r] = b ? __fadd_rn(acc, b[r]) : acc;
}

// ---------------------------------------------------------------------------
// Embeddings
// ---------------------------------------------------------------------------
// Decode: x[row] = speech_emb[tok[slot(row)]] + wpe[pos[row]]
// (build_step_graph, main.cpp:625-627).
__global__ void embed_step_kernel(const __half * __restrict__ semb, const float * __restrict__ wpe,
                                  const int * __restrict__ tok, const int * __restrict__ row_slot,
                                  const int * __restrict__ pos, int D, int V, int n_pos,
                                  float * __restrict__ x, unsigned * err) {
    const int row = blockIdx.x;
    const int t = tok[row_slot[row]];
    const int p = pos[row];
    if (t < 0 || t >= V || p < 0 || p >= n_pos) {
        if (threadIdx.x == 0) atomicOr(err, (t < 0 || t >= V) ? T3B_DEVERR_TOKEN : T3B_DEVERR_POS);
        return;
    }
    for (int i = threadIdx.x; i < D; i += blockDim.x)
        x[(size_t) row * D + i] = __fadd_rn(__half2float(semb[(size_t) t * D + i]), wpe[(size_t) p * D + i]);
}

// Prompt rows (build_prompt_graph, main.cpp:588-616): kind 0 = speaker
// projection row (spk), 1 = speech_emb[id], 2 = text_emb[id], 3 = zeros
// (text row of the CFG unconditional prompt); plus wpe[pos0 + r].
__global__ void embed_prompt_kernel(const __half * __restrict__ semb, const __half * __restrict__ temb,
                                    const float * __restrict__ wpe, const float * __restrict__ spk,
                                    const int * __restrict__ kind, const int * __restrict__ id, int pos0,
                                    int D, float * __restrict__ x) {
    const int r = blockIdx.x;
    const int k = kind[r], t = id[r];
    const float * wp = wpe + (size_t) (pos0 + r) * D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) {
        float v;
        if (k == 0) v = spk[i];
        else if (k == 1) v = __half2float(semb[(size_t) t * D + i]);
        else if (k == 2) v = __half2float(temb[(size_t) t * D + i]);
        else v = 0.0f;
        x[(size_t) r * D + i] = __fadd_rn(v, wp[i]);
    }
}

// ---------------------------------------------------------------------------
// Decode attention over per-row f16 caches (ggml_flash_attn_ext, N query
// rows, no mask: each row attends its own positions 0..len-1).
// grid = (n_head, M, s_max), 128 threads, one key per thread per CTA for the
// scores; for P.V the threads form 16 groups of 8 lanes, a group takes every
// 16th key and a lane 8 of its 64 dims (one 16-byte load per key).  Each
// thread issues its V loads before the K loads, so both reads of the chunk
// are in flight together; the 16 group sums are added in group order.  The
// last CTA of a (row, head) merges the split partials (m, l, o[64]).
// ---------------------------------------------------------------------------
struct AttnArgs {
    const float * q; int ldq;
    const __half * kv; size_t row_elems; size_t layer_off; size_t v_off;
    const int * row_of;      // nullable: row m uses cache row m
    const int * len; int len_add;
    int max_ctx, n_head;
    float * out; int ldo;
    float * part; unsigned * cnt; int s_max;
    unsigned * err;
    // attn_rows_kernel only (nullable): also write the output re-quantised
    // to Q8_0 blocks (the out-projection's activation prep), row stride ldo
    int8_t * qx; float * qd; int * qs;
};

__global__ __launch_bounds__(T3B_ATTN_CHUNK) void attn_decode_kernel(AttnArgs a) {
    constexpr int NG = T3B_ATTN_CHUNK / 8;          // lane groups for P.V
    constexpr int KPG = T3B_ATTN_CHUNK / NG;        // keys per group
    __shared__ float qs[T3B_HD];
    __shared__ float ps[T3B_ATTN_CHUNK];
    __shared__ float red[32];
    __shared__ __align__(16) float oacc[NG][T3B_HD];
    __shared__ int last;
    const int h = blockIdx.x, m = blockIdx.y, sp = blockIdx.z, tid = threadIdx.x;
    const int L = a.len[m] + a.len_add;
    if (L <= 0 || L > a.max_ctx) {
        if (tid == 0 && sp == 0) atomicOr(a.err, T3B_DEVERR_POS);
        return;
    }
    const int ns = (L + T3B_ATTN_CHUNK - 1) / T3B_ATTN_CHUNK;
    if (sp >= ns) return;
    const int crow = a.row_of ? a.row_of[m] : m;
    const __half * kb = a.kv + (size_t) crow * a.row_elems + a.layer_off + (size_t) h * a.max_ctx * T3B_HD;
    const __half * vb = kb + a.v_off;
    const int j0 = sp * T3B_ATTN_CHUNK;
    const int nk = min(T3B_ATTN_CHUNK, L - j0);
    const int g = tid >> 3, e = tid & 7;
    uint4 vr[KPG];
#pragma unroll
    for (int i = 0; i < KPG; ++i) {
        const int t = g + NG * i;
        vr[i] = t < nk ? __ldg((const uint4 *) (vb + (size_t) (j0 + t) * T3B_HD + e * 8)) : make_uint4(0, 0, 0, 0);
    }
    if (tid < T3B_HD) qs[tid] = a.q[(size_t) m * a.ldq + h * T3B_HD + tid];
    __syncthreads();
    float sc = -INFINITY;
    if (tid < nk) {
        const uint4 * kp = (const uint4 *) (kb + (size_t) (j0 + tid) * T3B_HD);
        float dot = 0.0f;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const uint4 u = kp[c];
            const __half2 * hp = (const __half2 *) &u;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float2 f = __half22float2(hp[t]);
                dot = fmaf(qs[c * 8 + 2 * t], f.x, dot);
                dot = fmaf(qs[c * 8 + 2 * t + 1], f.y, dot);
            }
        }
        sc = dot * 0.125f;
    }
    const float mx = block_max(sc, red);
    const float p = tid < nk ? expf(sc - mx) : 0.0f;
    ps[tid] = p;
    const float l = block_sum(p, red);
    __syncthreads();
    {
        float o[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < KPG; ++i) {
            const int t = g + NG * i;
            const float pt = t < nk ? ps[t] : 0.0f;
            const __half2 * hp = (const __half2 *) &vr[i];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 f = __half22float2(hp[k]);
                o[2 * k] = fmaf(pt, f.x, o[2 * k]);
                o[2 * k + 1] = fmaf(pt, f.y, o[2 * k + 1]);
            }
        }
        float4 * dst = (float4 *) &oacc[g][e * 8];
        dst[0] = make_float4(o[0], o[1], o[2], o[3]);
        dst[1] = make_float4(o[4], o[5], o[6], o[7]);
    }
    __syncthreads();
    float osum = 0.0f;
    if (tid < T3B_HD) {
#pragma unroll
        for (int gg = 0; gg < NG; ++gg) osum += oacc[gg][tid];
    }
    if (ns == 1) {
        if (tid < T3B_HD) a.out[(size_t) m * a.ldo + h * T3B_HD + tid] = osum / l;
        return;
    }
    float * P = a.part + (((size_t) m * a.n_head + h) * a.s_max + sp) * (T3B_HD + 2);
    if (tid < T3B_HD) P[2 + tid] = osum;
    if (tid == 0) { P[0] = mx; P[1] = l; }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned prev = atomicAdd(&a.cnt[(size_t) m * a.n_head + h], 1u);
        last = (prev == (unsigned) (ns - 1));
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    if (tid < T3B_HD) {
        const float * P0 = a.part + ((size_t) m * a.n_head + h) * a.s_max * (T3B_HD + 2);
        float gm = -INFINITY;
        for (int s = 0; s < ns; ++s) gm = fmaxf(gm, __ldcg(P0 + (size_t) s * (T3B_HD + 2)));
        float lt = 0.0f, ot = 0.0f;
        for (int s = 0; s < ns; ++s) {
            const float * Ps = P0 + (size_t) s * (T3B_HD + 2);
            const float w = expf(__ldcg(Ps) - gm);
            lt = fmaf(__ldcg(Ps + 1), w, lt);
            ot = fmaf(__ldcg(Ps + 2 + tid), w, ot);
        }
        a.out[(size_t) m * a.ldo + h * T3B_HD + tid] = ot / lt;
    }
    if (tid == 0) a.cnt[(size_t) m * a.n_head + h] = 0u;
}

// ---------------------------------------------------------------------------
// Decode attention for many rows (batched decode, prefill): one CTA of 4
// warps per (row, head) walks all L keys.  Lanes form groups of 8; a group
// holds one key's 64 halves of K and of V (16 bytes per lane), so a warp
// takes 4 keys and the CTA 16 keys per step, two steps per iteration to
// keep four 16-byte loads in flight per lane.  Each group keeps an online
// softmax (running max, sum and 8 output dims per lane); the 16 groups are
// merged at the end.  Scores are q.k / 8 as in attn_decode_kernel.
// grid = (n_head, M), 128 threads.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void attn_merge(float & mx, float & l, float (&o)[8], float om, float ol, const float (&oo)[8]) {
    const float nm = fmaxf(mx, om);
    const float a1 = mx == -INFINITY ? 0.0f : expf(mx - nm);
    const float a2 = om == -INFINITY ? 0.0f : expf(om - nm);
    l = l * a1 + ol * a2;
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = o[i] * a1 + oo[i] * a2;
    mx = nm;
}

__global__ __launch_bounds__(128) void attn_rows_kernel(AttnArgs a) {
    __shared__ float wmx[4], wl[4];
    __shared__ float wo[4][T3B_HD];
    const int h = blockIdx.x, m = blockIdx.y, tid = threadIdx.x;
    const int lane = tid & 31, w = tid >> 5, grp = lane >> 3, c = lane & 7;
    const int L = a.len[m] + a.len_add;
    if (L <= 0 || L > a.max_ctx) {
        if (tid == 0) atomicOr(a.err, T3B_DEVERR_POS);
        return;
    }
    const int crow = a.row_of ? a.row_of[m] : m;
    const __half * kb = a.kv + (size_t) crow * a.row_elems + a.layer_off + (size_t) h * a.max_ctx * T3B_HD + c * 8;
    const __half * vb = kb + a.v_off;
    float q[8];
    {
        const float * qp = a.q + (size_t) m * a.ldq + h * T3B_HD + c * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = qp[i];
    }
    float mx = -INFINITY, l = 0.0f, o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = 0.0f;
    // the loop bound is uniform over the warp (every lane reaches every
    // shuffle); a group whose key is past L contributes nothing.  Each group
    // takes keys j, j+16, j+32, j+48: eight 16-byte loads per lane, and the
    // next iteration's eight are issued before this one's arithmetic, so the
    // memory latency overlaps the dots, the softmax and the P.V update.
    constexpr int U = 4;
    uint4 kk[U], vv[U];
    auto fetch = [&](int jn, uint4 (&kd)[U], uint4 (&vd)[U]) {
#pragma unroll
        for (int u = 0; u < U; ++u) {
            kd[u] = make_uint4(0u, 0u, 0u, 0u);
            vd[u] = kd[u];
            if (jn + 16 * u < L) {
                kd[u] = __ldg((const uint4 *) (kb + (size_t) (jn + 16 * u) * T3B_HD));
                vd[u] = __ldg((const uint4 *) (vb + (size_t) (jn + 16 * u) * T3B_HD));
            }
        }
    };
    fetch(w * 4 + grp, kk, vv);
    for (int jb = w * 4; jb < L; jb += 16 * U) {
        const int j = jb + grp;
        uint4 kn[U], vn[U];
        fetch(j + 16 * U, kn, vn);
        float d[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const __half2 * kh = (const __half2 *) &kk[u];
            float t = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(kh[i]);
                t = fmaf(q[2 * i], f.x, t);
                t = fmaf(q[2 * i + 1], f.y, t);
            }
            d[u] = t;
        }
#pragma unroll
        for (int off = 1; off < 8; off <<= 1)
#pragma unroll
            for (int u = 0; u < U; ++u) d[u] += __shfl_xor_sync(0xffffffffu, d[u], off);
        float sc[U], nm = mx;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            sc[u] = j + 16 * u < L ? d[u] * 0.125f : -INFINITY;
            nm = fmaxf(nm, sc[u]);
        }
        const float corr = mx == -INFINITY ? 0.0f : expf(mx - nm);
        float p[U], ps = 0.0f;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            p[u] = j + 16 * u < L ? expf(sc[u] - nm) : 0.0f;
            ps += p[u];
        }
        l = l * corr + ps;
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] *= corr;
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const __half2 * vh = (const __half2 *) &vv[u];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(vh[i]);
                o[2 * i] = fmaf(p[u], f.x, o[2 * i]);
                o[2 * i + 1] = fmaf(p[u], f.y, o[2 * i + 1]);
            }
        }
        mx = nm;
#pragma unroll
        for (int u = 0; u < U; ++u) { kk[u] = kn[u]; vv[u] = vn[u]; }
    }
    // merge the four groups of the warp (lanes c, c+8, c+16, c+24 hold the same dims)
#pragma unroll
    for (int off = 8; off <= 16; off <<= 1) {
        float oo[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) oo[i] = __shfl_xor_sync(0xffffffffu, o[i], off);
        const float om = __shfl_xor_sync(0xffffffffu, mx, off), ol = __shfl_xor_sync(0xffffffffu, l, off);
        attn_merge(mx, l, o, om, ol, oo);
    }
    if (grp == 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) wo[w][c * 8 + i] = o[i];
        if (c == 0) { wmx[w] = mx; wl[w] = l; }
    }
    __syncthreads();
    if (tid < T3B_HD) {
        float gm = -INFINITY;
#pragma unroll
        for (int u = 0; u < 4; ++u) gm = fmaxf(gm, wmx[u]);
        float lt = 0.0f, ot = 0.0f;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (wmx[u] == -INFINITY) continue;
            const float f = expf(wmx[u] - gm);
            lt = fmaf(wl[u], f, lt);
            ot = fmaf(wo[u][tid], f, ot);
        }
        const float v = ot / lt;
        a.out[(size_t) m * a.ldo + h * T3B_HD + tid] = v;
        if (a.qx) {   // warps 0 and 1: Q8_0 blocks 2h and 2h + 1 of row m
            const float amax = warp_max(fabsf(v));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            const int q = (int) roundf(__fmul_rn(v, id));
            a.qx[(size_t) m * a.ldo + h * T3B_HD + tid] = (int8_t) q;
            const int sq = warp_sum_i(q);
            if (lane == 0) {
                const int blk = (size_t) m * (a.ldo / 32) + h * 2 + w;
                a.qd[blk] = __half2float(__float2half_rn(d));
                a.qs[blk] = sq;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Causal attention over a prompt chunk (eval_prompt's ggml_flash_attn_ext
// with the causal mask, main.cpp:663-677): the M query rows are consecutive
// positions of ONE cache row (row m at position len[m], attending keys
// 0 .. len[m] + len_add - 1).  Flash-attention tiling: a CTA takes 64 query
// rows of one head and walks the keys in tiles of 64 staged in shared
// memory, so every K/V row is read once per query tile instead of once per
// query row.  Online softmax per query row; f32 arithmetic on f16 K/V, the
// score q.k / 8 as in the decode kernels.  Thread (ty, tx) of 16 x 16 holds
// a 4 x 4 block: queries 4ty.., keys 4tx.. for the scores, dims 4tx.. of the
// output.  Optional Q8_0 output (the out-projection's input) as in
// attn_rows_kernel.
// grid = (n_head, ceil(M / 64)), 256 threads, T3B_PREFILL_SMEM dynamic smem.
// ---------------------------------------------------------------------------
#define T3B_PF_T 64
#define T3B_PF_LD (T3B_PF_T + 4)   // padded rows (floats), 16-byte aligned
#define T3B_PREFILL_SMEM (4 * T3B_PF_T * T3B_PF_LD * 4)
__global__ __launch_bounds__(256) void attn_prefill_kernel(AttnArgs a, int M) {
    extern __shared__ __align__(16) float pf_sm[];
    float * qT = pf_sm;                           // [d][q]
    float * kT = qT + T3B_PF_T * T3B_PF_LD;       // [d][k]
    float * vS = kT + T3B_PF_T * T3B_PF_LD;       // [k][d]
    float * pT = vS + T3B_PF_T * T3B_PF_LD;       // [k][q]
    __shared__ int lmax_s;
    const int h = blockIdx.x, m0 = blockIdx.y * T3B_PF_T, tid = threadIdx.x;
    const int ty = tid >> 4, tx = tid & 15;
    if (tid == 0) lmax_s = 0;
    __syncthreads();
    int Lq[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + 4 * ty + i;
        Lq[i] = 0;
        if (m < M) {
            const int L = a.len[m] + a.len_add;
            if (L <= 0 || L > a.max_ctx) { if (tx == 0) atomicOr(a.err, T3B_DEVERR_POS); }
            else Lq[i] = L;
        }
        if (tx == 0 && Lq[i] > 0) atomicMax(&lmax_s, Lq[i]);
    }
    // Q tile, transposed
    for (int e = tid; e < T3B_PF_T * T3B_HD; e += 256) {
        const int qi = e >> 6, d = e & 63, m = m0 + qi;
        qT[d * T3B_PF_LD + qi] = m < M ? a.q[(size_t) m * a.ldq + h * T3B_HD + d] : 0.0f;
    }
    __syncthreads();
    const int Lmax = lmax_s;
    const int crow = a.row_of ? a.row_of[m0] : m0;
    const __half * kb = a.kv + (size_t) crow * a.row_elems + a.layer_off + (size_t) h * a.max_ctx * T3B_HD;
    const __half * vb = kb + a.v_off;
    float mrun[4], lrun[4], o[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        mrun[i] = -INFINITY; lrun[i] = 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) o[i][j] = 0.0f;
    }
    for (int k0 = 0; k0 < Lmax; k0 += T3B_PF_T) {
        // K (transposed) and V tiles: thread -> key tid / 4, dims 16 (tid % 4) ..
        {
            const int kk = tid >> 2, c = (tid & 3) * 16, j = k0 + kk;
            uint4 k2[2], v2[2];
            if (j < Lmax) {
                k2[0] = __ldg((const uint4 *) (kb + (size_t) j * T3B_HD + c));
                k2[1] = __ldg((const uint4 *) (kb + (size_t) j * T3B_HD + c + 8));
                v2[0] = __ldg((const uint4 *) (vb + (size_t) j * T3B_HD + c));
                v2[1] = __ldg((const uint4 *) (vb + (size_t) j * T3B_HD + c + 8));
            } else {
                k2[0] = k2[1] = v2[0] = v2[1] = make_uint4(0u, 0u, 0u, 0u);
            }
            const __half * kh = (const __half *) k2;
            const __half * vh = (const __half *) v2;
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                kT[(c + e) * T3B_PF_LD + kk] = __half2float(kh[e]);
                vS[kk * T3B_PF_LD + c + e] = __half2float(vh[e]);
            }
        }
        __syncthreads();
        float sc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) sc[i][j] = 0.0f;
#pragma unroll 8
        for (int d = 0; d < T3B_HD; ++d) {
            const float4 qa = *(const float4 *) (qT + d * T3B_PF_LD + 4 * ty);
            const float4 ka = *(const float4 *) (kT + d * T3B_PF_LD + 4 * tx);
            const float qv[4] = {qa.x, qa.y, qa.z, qa.w}, kv[4] = {ka.x, ka.y, ka.z, ka.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) sc[i][j] = fmaf(qv[i], kv[j], sc[i][j]);
        }
        float corr[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float rm = -INFINITY;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                sc[i][j] = k0 + 4 * tx + j < Lq[i] ? sc[i][j] * 0.125f : -INFINITY;
                rm = fmaxf(rm, sc[i][j]);
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) rm = fmaxf(rm, __shfl_xor_sync(0xffffffffu, rm, off));
            const float mn = fmaxf(mrun[i], rm);
            corr[i] = mrun[i] == -INFINITY ? 0.0f : expf(mrun[i] - mn);
            float ps = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float p = sc[i][j] == -INFINITY ? 0.0f : expf(sc[i][j] - mn);
                pT[(4 * tx + j) * T3B_PF_LD + 4 * ty + i] = p;
                ps += p;
            }
#pragma unroll
            for (int off = 1; off < 16; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
            lrun[i] = lrun[i] * corr[i] + ps;
            mrun[i] = mn;
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) o[i][j] *= corr[i];
        const int kn = min(T3B_PF_T, Lmax - k0);
#pragma unroll 4
        for (int k = 0; k < kn; ++k) {
            const float4 pa = *(const float4 *) (pT + k * T3B_PF_LD + 4 * ty);
            const float4 va = *(const float4 *) (vS + k * T3B_PF_LD + 4 * tx);
            const float pv[4] = {pa.x, pa.y, pa.z, pa.w}, vv[4] = {va.x, va.y, va.z, va.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) o[i][j] = fmaf(pv[i], vv[j], o[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int m = m0 + 4 * ty + i;
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = Lq[i] > 0 ? o[i][j] / lrun[i] : 0.0f;
        if (m < M && Lq[i] > 0)
            *(float4 *) (a.out + (size_t) m * a.ldo + h * T3B_HD + 4 * tx) = make_float4(v[0], v[1], v[2], v[3]);
        if (a.qx) {   // Q8_0 block (tx / 8) of the head: eight lanes hold its 32 dims
            float amax = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
            for (int off = 1; off < 8; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
            const float d = __fdiv_rn(amax, 127.0f);
            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            int q[4], sq = 0;
#pragma unroll
            for (int j = 0; j < 4; ++j) { q[j] = (int) roundf(__fmul_rn(v[j], id)); sq += q[j]; }
#pragma unroll
            for (int off = 1; off < 8; off <<= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
            if (m < M && Lq[i] > 0) {
                *(int *) (a.qx + (size_t) m * a.ldo + h * T3B_HD + 4 * tx) =
                    (q[0] & 0xff) | ((q[1] & 0xff) << 8) | ((q[2] & 0xff) << 16) | ((q[3] & 0xff) << 24);
                if ((tx & 7) == 0) {
                    const size_t blk = (size_t) m * (a.ldo / 32) + h * 2 + (tx >> 3);
                    a.qd[blk] = __half2float(__float2half_rn(d));
                    a.qs[blk] = sq;
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// Fused sampler
// ---------------------------------------------------------------------------
struct ExpFix { const unsigned long long * tab; int bits; int n; };   // n = fix-up entries (0: none)

// 2^(i/32) words of t3_expf_core (device copy)
__device__ const unsigned long long g_t3_exp2_tab[32] = T3_EXP2_TAB_INIT;

// exp with the host libm's rounding: t3_expf_core + fix-up table lookup
// (two 32-byte buckets, read together) when the build found differences.
__device__ __forceinline__ float t3_expf_fix(float x, float y, uint4 a0, uint4 a1, uint4 b0, uint4 b1) {
    const uint32_t key = __float_as_uint(x);
    const uint32_t w[16] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w,
                            b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k)   // slot = (key << 32) | value: little-endian words (value, key)
        if ((w[2 * k] | w[2 * k + 1]) != 0u && w[2 * k + 1] == key) y = __uint_as_float(w[2 * k]);
    return y;
}
__device__ __forceinline__ float t3_expf_dev(float x, const ExpFix & f, const unsigned long long * e2) {
    const float y = t3_expf_core(x, e2);
    if (f.n == 0 || !(x >= -104.0f && x <= 0.0f)) return y;
    const uint32_t key = __float_as_uint(x);
    const uint4 * b1 = (const uint4 *) (f.tab + (size_t) t3_expf_hash1(key, f.bits) * T3_EXPF_SLOTS);
    const uint4 * b2 = (const uint4 *) (f.tab + (size_t) t3_expf_hash2(key, f.bits) * T3_EXPF_SLOTS);
    return t3_expf_fix(x, y, __ldg(b1), __ldg(b1 + 1), __ldg(b2), __ldg(b2 + 1));
}

// float -> 32-bit key whose ascending order is the float's DEScending order.
__device__ __forceinline__ uint32_t desc_key(float x) {
    const uint32_t u = __float_as_uint(x);
    const uint32_t asc = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ~asc;
}
__device__ __forceinline__ float desc_key_inv(uint32_t k) {
    const uint32_t asc = ~k;
    const uint32_t u = (asc & 0x80000000u) ? (asc & 0x7fffffffu) : ~asc;
    return __uint_as_float(u);
}

// std::mt19937 regeneration (libstdc++ _M_gen_rand), block-parallel in the
// three dependency phases of the recurrence.  All threads must call it.
__device__ void mt_twist(uint32_t * x) {
    const uint32_t UP = 0x80000000u, LO = 0x7fffffffu, A = 0x9908b0dfu;
    const int t = threadIdx.x;
    uint32_t nv = 0;
    // k in [0, 227): x[k+397] not yet rewritten
    if (t < 227) { const uint32_t y = (x[t] & UP) | (x[t + 1] & LO); nv = x[t + 397] ^ (y >> 1) ^ ((y & 1u) ? A : 0u); }
    __syncthreads();
    if (t < 227) x[t] = nv;
    __syncthreads();
    // k in [227, 454): x[k-227] from the first phase
    if (t < 227) { const int k = 227 + t; const uint32_t y = (x[k] & UP) | (x[k + 1] & LO); nv = x[k - 227] ^ (y >> 1) ^ ((y & 1u) ? A : 0u); }
    __syncthreads();
    if (t < 227) x[227 + t] = nv;
    __syncthreads();
    // k in [454, 623): x[k-227] from the second phase
    if (t < 169) { const int k = 454 + t; const uint32_t y = (x[k] & UP) | (x[k + 1] & LO); nv = x[k - 227] ^ (y >> 1) ^ ((y & 1u) ? A : 0u); }
    __syncthreads();
    if (t < 169) x[454 + t] = nv;
    __syncthreads();
    if (t == 0) { const uint32_t y = (x[623] & UP) | (x[0] & LO); x[623] = x[396] ^ (y >> 1) ^ ((y & 1u) ? A : 0u); }
    __syncthreads();
}
__device__ __forceinline__ uint32_t mt_temper(uint32_t z) {
    z ^= (z >> 11);
    z ^= (z << 7) & 0x9d2c5680u;
    z ^= (z << 15) & 0xefc60000u;
    z ^= (z >> 18);
    return z;
}

__device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = __umulhi(0xD2511F53u, c[0]), lo0 = 0xD2511F53u * c[0];
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c[2]), lo1 = 0xCD9E8D57u * c[2];
        const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
        c[0] = n0; c[1] = lo1; c[2] = n2; c[3] = lo0;
        k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
    }
}

// Sequential float / double chains the reference evaluates left to right.
// One thread walks them; operands come in as float4 loads, eight at a time,
// so the only serial dependency left is the add itself.
__device__ __forceinline__ float seq_sum_f32(const float * a, int n) {
    // operands for the next 16 adds are loaded while the current 16 run
    float s = 0.0f;
    int j = 0;
    if (n >= 16) {
        float4 c0 = *(const float4 *) (a), c1 = *(const float4 *) (a + 4), c2 = *(const float4 *) (a + 8),
               c3 = *(const float4 *) (a + 12);
        for (; j + 32 <= n; j += 16) {
            const float4 n0 = *(const float4 *) (a + j + 16), n1 = *(const float4 *) (a + j + 20);
            const float4 n2 = *(const float4 *) (a + j + 24), n3 = *(const float4 *) (a + j + 28);
            s = __fadd_rn(s, c0.x); s = __fadd_rn(s, c0.y); s = __fadd_rn(s, c0.z); s = __fadd_rn(s, c0.w);
            s = __fadd_rn(s, c1.x); s = __fadd_rn(s, c1.y); s = __fadd_rn(s, c1.z); s = __fadd_rn(s, c1.w);
            s = __fadd_rn(s, c2.x); s = __fadd_rn(s, c2.y); s = __fadd_rn(s, c2.z); s = __fadd_rn(s, c2.w);
            s = __fadd_rn(s, c3.x); s = __fadd_rn(s, c3.y); s = __fadd_rn(s, c3.z); s = __fadd_rn(s, c3.w);
            c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        }
        s = __fadd_rn(s, c0.x); s = __fadd_rn(s, c0.y); s = __fadd_rn(s, c0.z); s = __fadd_rn(s, c0.w);
        s = __fadd_rn(s, c1.x); s = __fadd_rn(s, c1.y); s = __fadd_rn(s, c1.z); s = __fadd_rn(s, c1.w);
        s = __fadd_rn(s, c2.x); s = __fadd_rn(s, c2.y); s = __fadd_rn(s, c2.z); s = __fadd_rn(s, c2.w);
        s = __fadd_rn(s, c3.x); s = __fadd_rn(s, c3.y); s = __fadd_rn(s, c3.z); s = __fadd_rn(s, c3.w);
        j += 16;
    }
    for (; j < n; ++j) s = __fadd_rn(s, a[j]);
    return s;
}
__device__ __forceinline__ double seq_sum_f64(const float * a, int n) {
    double s = 0.0;
    int j = 0;
    for (; j + 8 <= n; j += 8) {
        const float4 u = *(const float4 *) (a + j), v = *(const float4 *) (a + j + 4);
        s = __dadd_rn(s, (double) u.x); s = __dadd_rn(s, (double) u.y);
        s = __dadd_rn(s, (double) u.z); s = __dadd_rn(s, (double) u.w);
        s = __dadd_rn(s, (double) v.x); s = __dadd_rn(s, (double) v.y);
        s = __dadd_rn(s, (double) v.z); s = __dadd_rn(s, (double) v.w);
    }
    for (; j < n; ++j) s = __dadd_rn(s, (double) a[j]);
    return s;
}
// First j with fl(fl(...(a[0]) + a[1]) ... + a[j]) >= target; n if none.
__device__ __forceinline__ int seq_cut_f32(const float * a, int n, float target) {
    float c = 0.0f;
    int j = 0;
    for (; j + 8 <= n; j += 8) {
        const float4 u = *(const float4 *) (a + j), v = *(const float4 *) (a + j + 4);
        const float w[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
#pragma unroll
        for (int t = 0; t < 8; ++t) {
            c = __fadd_rn(c, w[t]);
            if (c >= target) return j + t;
        }
    }
    for (; j < n; ++j) {
        c = __fadd_rn(c, a[j]);
        if (c >= target) return j;
    }
    return n;
}

struct SampArgs {
    const float * cond; long long cond_stride;
    const float * uncond; long long uncond_stride;   // nullable
    int V;
    const int * slot_of;                              // nullable: slot = row
    int * hist; int hist_stride; int * hist_len; int hist_append;
    const t3b_sample_params * params; int params_per_row;
    const int * rng_mode;                             // per slot; nullable = Philox
    uint32_t * mt;                                    // [slot][625]
    const unsigned long long * ph_seed; unsigned long long * ph_ctr;
    int * tok_out;                                    // [row]
    int * step_tok;                                   // nullable: [slot] next-step token
    int * done; int stop_token;                       // nullable
    ExpFix fx;
    unsigned long long * tl;                          // nullable: stage stamps of row 0 (debug)
    int mt_resident;                                  // mt19937 words already in shared memory (persistent kernel)
};

#define T3B_SAMPLER_THREADS 1024
#define T3B_SAMPLER_TL 22   // debug stage stamps of row 0
#define T3B_SAMPLER_VMAX 8192
// dynamic smem: s[VMAX] f32 | keys[VMAX] u64 | e[VMAX] f32
#define T3B_SAMPLER_SMEM (T3B_SAMPLER_VMAX * (4 + 8 + 4))

// exp(x) with the host libm's rounding for N values at once: every bucket
// read is issued before any result is needed, so a batch costs one memory
// round trip.
template <int N>
__device__ __forceinline__ void t3_expf_batch(float (&x)[N], const ExpFix & f, const unsigned long long * e2) {
    if (f.n == 0) {
#pragma unroll
        for (int n = 0; n < N; ++n) x[n] = t3_expf_core(x[n], e2);
        return;
    }
    uint4 a0[N], a1[N], b0[N], b1[N];
#pragma unroll
    for (int n = 0; n < N; ++n) {
        if (x[n] >= -104.0f && x[n] <= 0.0f) {   // fix-ups exist only in [-104, 0]
            const uint32_t key = __float_as_uint(x[n]);
            const uint4 * p1 = (const uint4 *) (f.tab + (size_t) t3_expf_hash1(key, f.bits) * T3_EXPF_SLOTS);
            const uint4 * p2 = (const uint4 *) (f.tab + (size_t) t3_expf_hash2(key, f.bits) * T3_EXPF_SLOTS);
            a0[n] = __ldg(p1); a1[n] = __ldg(p1 + 1); b0[n] = __ldg(p2); b1[n] = __ldg(p2 + 1);
        } else {
            a0[n] = a1[n] = b0[n] = b1[n] = make_uint4(0u, 0u, 0u, 0u);
        }
    }
#pragma unroll
    for (int n = 0; n < N; ++n) x[n] = t3_expf_fix(x[n], t3_expf_core(x[n], e2), a0[n], a1[n], b0[n], b1[n]);
}

// Block-wide exclusive scan of doubles (blockDim.x multiple of 32, <= 1024).
__device__ __forceinline__ double block_excl_scan_d(double v, double * red, double * total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    double incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    __syncthreads();
    if (lane == 31) red[w] = incl;
    __syncthreads();
    if (w == 0) {
        const double x = lane < nw ? red[lane] : 0.0;
        double xi = x;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double n = __shfl_up_sync(0xffffffffu, xi, o);
            if (lane >= o) xi += n;
        }
        if (lane < nw) red[lane] = xi - x;
        if (lane == 31) red[32] = xi;
    }
    __syncthreads();
    const double r = red[w] + (incl - v);
    *total = red[32];
    return r;
}

// Index of the first element whose running sum reaches `target`, for values
// a[0..n) (float or double via the loader), split in per-thread contiguous
// chunks.  The running sum is evaluated exactly enough (double) to locate the
// crossing; *margin_ok tells whether both neighbours of the crossing are at
// least eps away from target, so that any evaluation order that keeps its
// error below eps crosses at the same index.  Returns n when the total stays
// below target.
template <class LoadF>
__device__ int block_first_crossing(int n, double target, double eps, LoadF load, double * red, int * shi, bool * margin_ok) {
    const int tid = threadIdx.x, nth = blockDim.x;
    const int per = (n + nth - 1) / nth;
    const int c0 = min(n, tid * per), c1 = min(n, c0 + per);
    double sum = 0.0;
    for (int j = c0; j < c1; ++j) sum += load(j);
    double total;
    const double excl = block_excl_scan_d(sum, red, &total);
    if (tid == 0) { shi[0] = n; shi[1] = 1; }
    __syncthreads();
    if (c0 < c1 && excl < target && excl + sum >= target) {
        double run = excl, prev = excl;
        int j = c0;
        for (; j < c1; ++j) {
            prev = run;
            run += load(j);
            if (run >= target) break;
        }
        if (j >= c1) j = c1 - 1;
        shi[0] = j;
        shi[1] = (run >= target + eps) && (j == 0 || prev < target - eps);
    }
    __syncthreads();
    const int idx = shi[0];
    if (idx == n) *margin_ok = total < target - eps;
    else *margin_ok = shi[1] != 0;
    __syncthreads();
    return idx;
}

// Block-wide exclusive scan of ints in thread order (blockDim.x a multiple
// of 32); *total receives the sum.
__device__ __forceinline__ int block_excl_scan_i(int v, int * red, int * total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    __syncthreads();
    if (lane == 31) red[w] = incl;
    __syncthreads();
    if (w == 0) {
        const int x = lane < nw ? red[lane] : 0;
        int xi = x;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, xi, o);
            if (lane >= o) xi += n;
        }
        if (lane < nw) red[lane] = xi - x;
        if (lane == 31) red[32] = xi;
    }
    __syncthreads();
    const int r = red[w] + incl - v;
    *total = red[32];
    return r;
}

// Linear value bins of the sampler's fast top-k/top-p path, highest score
// first: floor((v - smin) * scale) never decreases as v grows.
#define SAMP_NBIN 2048
#define SAMP_BIN_MAX 32
__device__ __forceinline__ int samp_dbin(float v, float smin, float scale) {
    int b = (int) __fmul_rn(__fsub_rn(v, smin), scale);
    b = min(max(b, 0), SAMP_NBIN - 1);
    return SAMP_NBIN - 1 - b;
}

// The two 32-bit draws of the row's generator (block-wide: the mt19937
// state is loaded and twisted by every thread).  The stream advances by two
// words / one Philox counter, as in the reference's discrete_distribution.
__device__ __forceinline__ void samp_rng_bits(const SampArgs & a, int slot, int rmode, uint32_t * mtx, uint32_t & x1,
                                              uint32_t & x2) {
    const int tid = threadIdx.x, nth = blockDim.x;
    if (rmode == T3B_RNG_MT19937) {
        uint32_t * st = a.mt + (size_t) slot * 625;
        if (!a.mt_resident) {        // else mtx still holds this slot's state
            for (int i = tid; i < 625; i += nth) mtx[i] = st[i];
            __syncthreads();
        }
        int idx = (int) mtx[624];
        bool tw = false;
        if (idx >= 624) { mt_twist(mtx); idx = 0; tw = true; }
        x1 = mt_temper(mtx[idx]); ++idx;
        if (idx >= 624) { mt_twist(mtx); idx = 0; tw = true; }
        x2 = mt_temper(mtx[idx]); ++idx;
        __syncthreads();          // every thread has read the index word
        if (tw) for (int i = tid; i < 624; i += nth) st[i] = mtx[i];
        if (tid == 0) { st[624] = (uint32_t) idx; mtx[624] = (uint32_t) idx; }
    } else {
        const unsigned long long sd = a.ph_seed[slot];
        const unsigned long long ct = a.ph_ctr[slot];
        uint32_t c4[4] = {(uint32_t) ct, (uint32_t) (ct >> 32), (uint32_t) slot, 0u};
        philox4x32_10(c4, (uint32_t) sd, (uint32_t) (sd >> 32));
        x1 = c4[0]; x2 = c4[1];
        __syncthreads();
        if (tid == 0) a.ph_ctr[slot] = ct + 1ull;
    }
}

// std::generate_canonical<double, 53> of two 32-bit draws
__device__ __forceinline__ double samp_canonical(uint32_t x1, uint32_t x2) {
    double sum = (double) x1;
    sum += (double) x2 * 4294967296.0;
    double u = sum / 18446744073709551616.0;
    if (u >= 1.0) u = nextafter(1.0, 0.0);
    return u;
}

// Ascending bitonic sort of one 64-bit key per lane.
__device__ __forceinline__ unsigned long long warp_sort_u64(unsigned long long k) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1)
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, stride);
            const bool keep_min = ((lane & size) == 0) == ((lane & stride) == 0);
            k = keep_min ? (o < k ? o : k) : (o > k ? o : k);
        }
    return k;
}

// The row's outputs: token, next-step token, history append, stop flag.
__device__ __forceinline__ int samp_finish(const SampArgs & a, int r, int slot, int hl, int tok) {
    if (threadIdx.x == 0) {
        if (a.tok_out) a.tok_out[r] = tok;
        if (a.step_tok) a.step_tok[slot] = tok;
        if (a.hist_append && a.hist && a.hist_len) {
            if (hl < a.hist_stride) {
                a.hist[(size_t) slot * a.hist_stride + hl] = tok;
                a.hist_len[slot] = hl + 1;
            }
        }
        if (a.done && tok == a.stop_token) a.done[slot] = 1;
    }
    __syncthreads();
    return tok;
}

// Warp scratch of the few-survivor path (shared memory)
struct SampWarpBuf { float f[32]; float q[32]; double d[32]; int i[32]; };

// Steps (2)-(5) of the row when at most 32 scores are finite (after min-p),
// by one warp: lane j holds survivor j.  Orders come from ranks (each lane
// counts the lanes ahead of it over 32 shuffles) and a pass through shared
// memory; each sequential float chain of the reference (top-p sum and
// running sum, softmax sum) is walked in the reference's order by every lane
// over values read back from shared memory, whose loads do not wait on the
// chain.  sml: the finite scores' indices (any order); seen: history bit
// set.  Writes the n survivors in index order to lst and their
// probabilities to pr (0 for the ones dropped on the way); returns false
// when every probability is 0 (the reference returns token 0 undrawn).
__device__ bool samp_small_probs(const t3b_sample_params & P, int V, const float * s, const int * sml, int n,
                                 const unsigned * seen, const ExpFix & fx, const unsigned long long * e2tab,
                                 int * lst, float * pr, SampWarpBuf * wb, unsigned long long * tls) {
    const unsigned FULL = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    // survivors in index order: rank of each index among the n (distinct)
    {
        const int raw = lane < n ? sml[lane] : 0x7fffffff;
        int rk = 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) rk += __shfl_sync(FULL, raw, j) < raw ? 1 : 0;
        if (lane < n) wb->i[rk] = raw;
        __syncwarp();
    }
    const int idx = lane < n ? wb->i[lane] : -1;
    bool alive = lane < n;
    float v = alive ? s[idx] : -INFINITY;
    // (2) top-k: with n <= k the reference's threshold is -inf (no change);
    // else the score at descending rank k, nudged by 1e-10f when fewer than
    // k scores are above it, and every score <= it dropped
    if (P.top_k > 0 && P.top_k < V && n > P.top_k) {
        const unsigned long long kd = warp_sort_u64(alive ? ((unsigned long long) desc_key(v) << 32) | (unsigned) idx : ~0ull);
        const float thr = desc_key_inv((uint32_t) (__shfl_sync(FULL, kd, P.top_k) >> 32));
        const int above = __popc(__ballot_sync(FULL, alive && v > thr));
        const float thr2 = above < P.top_k ? __fsub_rn(thr, 1e-10f) : thr;
        alive = alive && v > thr2;
    }
    // (3) top-p: descending score (ties by index: lanes are in index
    // order), e = exp(s - max), psum = sequential sum, keep up to the first
    // rank whose running sum of e / psum reaches top_p
    if (P.top_p < 1.0f) {
        const int c = __popc(__ballot_sync(FULL, alive));
        if (c > 0) {
            const float vv = alive ? v : -INFINITY;
            int rk = 0;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const float o = __shfl_sync(FULL, vv, j);
                rk += (o > vv || (o == vv && j < lane)) ? 1 : 0;
            }
            float mx = vv;
#pragma unroll
            for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
            const float ej = alive ? t3_expf_dev(__fsub_rn(vv, mx), fx, e2tab) : 0.0f;
            if (alive) wb->f[rk] = ej;
            __syncwarp();
            float psum = 0.0f;
#pragma unroll 4
            for (int r = 0; r < c; ++r) psum = __fadd_rn(psum, wb->f[r]);
            if (alive) wb->q[rk] = __fdiv_rn(ej, psum);
            __syncwarp();
            float cum = 0.0f;
            int cut = c;
#pragma unroll 4
            for (int r = 0; r < c; ++r) {
                cum = __fadd_rn(cum, wb->q[r]);
                if (cum >= P.top_p) { cut = r + 1; break; }
            }
            alive = alive && rk < cut;
            __syncwarp();
        }
    }
    if (tls && lane == 0) { unsigned long long t_; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_)); tls[8] = t_; }
    // (4) repetition penalty on surviving history ids (each id once)
    if (P.repeat_penalty != 1.0f && alive && ((seen[idx >> 5] >> (idx & 31)) & 1u))
        v = v > 0.0f ? __fdiv_rn(v, P.repeat_penalty) : __fmul_rn(v, P.repeat_penalty);
    // (5) softmax over the survivors in index order (lane order)
    float mx = alive ? v : -INFINITY;
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, o));
    const float pe = alive ? t3_expf_dev(__fsub_rn(v, mx), fx, e2tab) : 0.0f;
    wb->f[lane] = pe;
    __syncwarp();
    float psum = 0.0f;
#pragma unroll 4
    for (int j = 0; j < n; ++j) psum = __fadd_rn(psum, wb->f[j]);
    if (lane < n) {
        lst[lane] = idx;
        pr[lane] = psum != 0.0f ? __fdiv_rn(pe, psum) : 0.0f;
    }
    __syncwarp();
    return psum != 0.0f;
}

// Steps (6)/(7) over the list of samp_small_probs, by one warp: the first
// maximum in index order (temp <= 0), or discrete_distribution's draw:
// dsum = sequential double sum, running sum of p / dsum with the last index
// (V - 1) forced to 1, first entry >= u.
__device__ int samp_small_pick(const t3b_sample_params & P, int V, const int * lst, const float * pr, int n,
                               uint32_t x1, uint32_t x2, SampWarpBuf * wb) {
    const unsigned FULL = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const float p = lane < n ? pr[lane] : 0.0f;
    const int idx = lane < n ? lst[lane] : 0;
    if (P.temp <= 0.0f) {
        float bp = p;
        int bl = lane < n ? lane : 32;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float op = __shfl_xor_sync(FULL, bp, o);
            const int ol = __shfl_xor_sync(FULL, bl, o);
            if (op > bp || (op == bp && ol < bl)) { bp = op; bl = ol; }
        }
        // the reference starts at index 0: with every p = 0 index 0 stays
        const int ib = __shfl_sync(FULL, idx, bl < 32 ? bl : 0);
        return bp > 0.0f ? ib : 0;
    }
    double dsum = 0.0;
#pragma unroll 4
    for (int j = 0; j < n; ++j) dsum = __dadd_rn(dsum, (double) pr[j]);
    const double u = samp_canonical(x1, x2);
    if (u <= 0.0) return 0;
    wb->d[lane] = (double) p / dsum;   // each term divided once, in parallel
    __syncwarp();
    // running sum: every lane walks the chain in the reference's order
    double cc = 0.0;
    int pick = V - 1;
#pragma unroll 4
    for (int j = 0; j < n; ++j) {
        cc = __dadd_rn(cc, wb->d[j]);
        const double ci = lst[j] == V - 1 ? 1.0 : cc;
        if (ci >= u) { pick = lst[j]; break; }
    }
    __syncwarp();
    return pick;
}

// One row of sample_next_token_ex by the whole block (any blockDim.x that
// is a multiple of 32 and >= 256).  smraw: T3B_SAMPLER_SMEM bytes of shared
// memory.  Returns the token (every thread), or -1 for a finished stream.
//
// Every value the reference computes is reproduced bit for bit: its
// sequential float sums are either evaluated sequentially (one thread) or,
// where the reference only compares a running sum with a threshold, located
// with a double-precision parallel prefix and accepted only when the
// crossing is farther from the threshold than the sequential rounding error
// can reach; otherwise the sequential chain runs.
__device__ __noinline__ int sample_row_block(const SampArgs & a, int r, unsigned char * smraw) {
    float * s = (float *) smraw;
    unsigned long long * keys = (unsigned long long *) (smraw + T3B_SAMPLER_VMAX * 4);
    float * e = (float *) (smraw + T3B_SAMPLER_VMAX * 12);
    int * lst = (int *) keys;   // index list, reused after the sort
    __shared__ float redf[32];
    __shared__ int redi[33];
    __shared__ double redd[33];
    __shared__ unsigned seen[T3B_SAMPLER_VMAX / 32];
    __shared__ unsigned surv[T3B_SAMPLER_VMAX / 32];   // survivor bit set (list mode)
    __shared__ float redf2[32];
    __shared__ int shi[8];
    __shared__ float shf[4];
    __shared__ uint32_t mtx[625];
    __shared__ unsigned long long e2tab[32];   // t3_expf_core's table (first use is after several barriers)
    __shared__ int sml[32];                    // indices kept by min-p while they are at most 32
    __shared__ int sml_n;
    __shared__ SampWarpBuf swb;                // few-survivor path scratch

    const int tid = threadIdx.x, nth = blockDim.x, lane = tid & 31;
    unsigned long long t_entry = 0;   // debug: the row's first instruction
    if (a.tl && tid == 0) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_entry));
    const int slot = a.slot_of ? a.slot_of[r] : r;
    if (a.done && a.done[slot]) return -1;
    if (tid < 32) e2tab[tid] = g_t3_exp2_tab[tid];
    if (tid == 0) sml_n = 0;
    unsigned long long * tls = (a.tl && r == 0) ? a.tl : nullptr;
#define SAMP_STAMP(i) do { if (tls && tid == 0) { unsigned long long t_; asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_)); tls[i] = t_; } } while (0)
    if (tls && tid == 0) tls[T3B_SAMPLER_TL - 2] = t_entry;
    SAMP_STAMP(0);
    const t3b_sample_params P = a.params[a.params_per_row ? r : 0];
    const int V = a.V;
    const float * cond = a.cond + (long long) slot * a.cond_stride;
    const float * unc = a.uncond ? a.uncond + (long long) slot * a.uncond_stride : nullptr;
    const int hl = a.hist_len ? min(a.hist_len[slot], a.hist_stride) : 0;
    const int rmode = a.rng_mode ? a.rng_mode[slot] : T3B_RNG_PHILOX;   // loaded early: used at the draw
    const int * hist = a.hist ? a.hist + (size_t) slot * a.hist_stride : nullptr;
    // first history id of this thread, loaded now: the min-p stage needs it
    const int hist0 = (P.repeat_penalty != 1.0f && tid < hl) ? __ldg(hist + tid) : -1;

    // (0) CFG mix, (1) temperature  (main.cpp:735-738).  Each thread issues
    // its loads eight at a time (through L2: the persistent kernel passes
    // logits other CTAs have just written); the max and the count of finite
    // scores are gathered on the way for min-p and the top-k skip.
    const bool cfg = unc != nullptr && P.cfg_weight != 0.0f;
    const bool use_t = P.temp > 0.0f && P.temp != 1.0f;
    const float inv_t = use_t ? __fdiv_rn(1.0f, P.temp) : 1.0f;
    float lmx = -INFINITY, lmn = INFINITY;
    int lfin = 0;
    auto take = [&](int i, float v, float uv) {
        if (cfg) v = __fadd_rn(v, __fmul_rn(P.cfg_weight, __fsub_rn(v, uv)));
        if (use_t) v = __fmul_rn(v, inv_t);
        s[i] = v;
        if (v != -INFINITY) { lmx = fmaxf(lmx, v); lmn = fminf(lmn, v); ++lfin; }
    };
    const int mis = (int) (((uintptr_t) cond >> 2) & 3u);
    const bool vec = !cfg || mis == (int) (((uintptr_t) unc >> 2) & 3u);
    if (vec) {
        // 16-byte loads over the aligned body (both rows share the alignment),
        // the first `head` and the last few elements one by one; two 16-byte
        // loads per row and thread in flight (one round trip for V <= 8 nth)
        const int head = min((4 - mis) & 3, V), nq = (V - head) >> 2, tail0 = head + 4 * nq;
        const float4 * c4 = (const float4 *) (cond + head);
        const float4 * u4 = cfg ? (const float4 *) (unc + head) : nullptr;
        if (tid < head) take(tid, __ldcg(cond + tid), cfg ? __ldcg(unc + tid) : 0.0f);
        if (tid < V - tail0) take(tail0 + tid, __ldcg(cond + tail0 + tid), cfg ? __ldcg(unc + tail0 + tid) : 0.0f);
        for (int q0 = 0; q0 < nq; q0 += 2 * nth) {
            float4 cv[2], uv[2];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int q = q0 + k * nth + tid;
                cv[k] = q < nq ? __ldcg(c4 + q) : make_float4(0.f, 0.f, 0.f, 0.f);
                uv[k] = (cfg && q < nq) ? __ldcg(u4 + q) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int q = q0 + k * nth + tid;
                if (q < nq) {
                    const int i = head + 4 * q;
                    take(i, cv[k].x, uv[k].x); take(i + 1, cv[k].y, uv[k].y);
                    take(i + 2, cv[k].z, uv[k].z); take(i + 3, cv[k].w, uv[k].w);
                }
            }
        }
    } else {   // CFG rows of different alignment: eight loads per row and thread in flight
        for (int i0 = 0; i0 < V; i0 += 8 * nth) {
            float cv[8], uv[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int i = i0 + q * nth + tid;
                cv[q] = i < V ? __ldcg(cond + i) : 0.0f;
                uv[q] = i < V ? __ldcg(unc + i) : 0.0f;
            }
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int i = i0 + q * nth + tid;
                if (i < V) take(i, cv[q], uv[q]);
            }
        }
    }
    // count, max and min in one exchange; before its barrier, one thread
    // evaluates log(min_p) for the min-p stage (a double log in every thread
    // costs microseconds of FP64 issue) and the history bit set is cleared
    const int nw = nth >> 5, w = tid >> 5;
    const int nwords0 = (V + 31) / 32;
    if (tid == 0 && P.min_p > 0.0f) {
        // (double) d <= lg - 1e-5  <=>  d <= largest float not above it;
        // (double) d >= lg + 1e-5  <=>  d >= smallest float not below it
        const double lg = log((double) P.min_p);
        shf[2] = __double2float_rd(lg - 1e-5);
        shf[3] = __double2float_ru(lg + 1e-5);
    }
    for (int i = tid; i < nwords0; i += nth) seen[i] = 0u;
    lfin = warp_sum_i(lfin);
    lmx = warp_max(lmx);
    lmn = -warp_max(-lmn);
    if (lane == 0) { redi[w] = lfin; redf[w] = lmx; redf2[w] = lmn; }
    __syncthreads();
    int nfin = warp_sum_i(lane < nw ? redi[lane] : 0);
    const float smax = warp_max(lane < nw ? redf[lane] : -INFINITY);
    const float smin = -warp_max(lane < nw ? -redf2[lane] : -INFINITY);

    SAMP_STAMP(1);
    // (1b) min-p: drop exp(s - max) < min_p.  The host expf is within one ulp
    // of exp, so for results in the normal range exp(d) < min_p is decided by
    // d against log(min_p) except within 1e-5 of it (a relative gap of 1e-5 in
    // exp, far above one ulp); only that window evaluates expf exactly.
    if (P.min_p > 0.0f && nfin > 0) {
        const bool fast = P.min_p >= 1e-30f;
        const float flo = shf[2], fhi = shf[3];
        int kept = 0;
        // history ids into the bit set (published by the count's barrier):
        // the few-survivor path below uses it as is
        if (P.repeat_penalty != 1.0f)
            for (int j = tid; j < hl; j += nth) {
                const int t = j == tid ? hist0 : hist[j];
                if (t >= 0 && t < V) atomicOr(&seen[t >> 5], 1u << (t & 31));
            }
        for (int i0 = 0; i0 < V; i0 += nth) {   // warp-uniform trip count (the ballot below)
            const int i = i0 + tid;
            bool keep = false;
            if (i < V) {
                const float v = s[i];
                if (v != -INFINITY) {
                    const float d = __fsub_rn(v, smax);
                    bool drop;
                    if (fast && d <= flo) drop = true;
                    else if (fast && d >= fhi) drop = false;
                    else drop = t3_expf_dev(d, a.fx, e2tab) < P.min_p;
                    if (drop) s[i] = -INFINITY;
                    else { ++kept; keep = true; }
                }
            }
            // the first 32 kept indices (any order), one atomic per warp
            const unsigned bk = __ballot_sync(0xffffffffu, keep);
            if (bk) {
                int base = 0;
                if (lane == 0) base = atomicAdd(&sml_n, __popc(bk));
                base = __shfl_sync(0xffffffffu, base, 0) + __popc(bk & ((1u << lane) - 1u));
                if (keep && base < 32) sml[base] = i;
            }
        }
        nfin = block_sum_i(kept, redi);
        if (nfin > 0 && nfin <= 32) {
            // Few survivors: steps (2)-(7) by one warp over the list (the
            // history bit set is complete: block_sum_i's barrier)
            SAMP_STAMP(2);
            int tok = 0;
            if (rmode != T3B_RNG_MT19937) {
                // Philox: the draw is computed by the warp itself, no barrier
                if (tid < 32) {
                    const bool ok = samp_small_probs(P, V, s, sml, nfin, seen, a.fx, e2tab, lst, e, &swb, tls);
                    uint32_t x1 = 0u, x2 = 0u;
                    if (ok && P.temp > 0.0f) {
                        const unsigned long long sd = a.ph_seed[slot];
                        const unsigned long long ct = a.ph_ctr[slot];
                        uint32_t c4[4] = {(uint32_t) ct, (uint32_t) (ct >> 32), (uint32_t) slot, 0u};
                        philox4x32_10(c4, (uint32_t) sd, (uint32_t) (sd >> 32));
                        x1 = c4[0]; x2 = c4[1];
                        if (lane == 0) a.ph_ctr[slot] = ct + 1ull;
                    }
                    const int t = ok ? samp_small_pick(P, V, lst, e, nfin, x1, x2, &swb) : 0;
                    if (lane == 0) shi[6] = t;
                }
                __syncthreads();
                tok = shi[6];
            } else {
                if (tid < 32) {
                    const bool ok = samp_small_probs(P, V, s, sml, nfin, seen, a.fx, e2tab, lst, e, &swb, tls);
                    if (lane == 0) shi[7] = ok;
                }
                __syncthreads();
                SAMP_STAMP(12);
                if (shi[7]) {
                    uint32_t x1 = 0u, x2 = 0u;
                    if (P.temp > 0.0f) samp_rng_bits(a, slot, rmode, mtx, x1, x2);
                    SAMP_STAMP(13);
                    if (tid < 32) {
                        const int t = samp_small_pick(P, V, lst, e, nfin, x1, x2, &swb);
                        if (lane == 0) shi[6] = t;
                    }
                    __syncthreads();
                    tok = shi[6];
                }
            }
            SAMP_STAMP(15);
            const int tk = samp_finish(a, r, slot, hl, tok);
            SAMP_STAMP(T3B_SAMPLER_TL - 1);
            return tk;
        }
    }

    SAMP_STAMP(2);
    // (2) top-k (main.cpp:740-748): radix-select the value at descending
    // rank k, then keep s > thr (thr nudged by 1e-10f if fewer than k).  With
    // k or fewer finite scores the reference's threshold is -inf and nothing
    // changes, so the stage is skipped.
    bool topk_pending = false;   // drop of s <= thr_k not yet applied
    float thr_k = -INFINITY;
    // Fast path of (2) and (3): linear value bins order the scores, so a
    // histogram finds the bin of rank k; the scores of that bin and above are
    // scattered into their bins and each bin (at most SAMP_BIN_MAX scores) is
    // insertion-sorted by (value desc, index asc), which is the order top-p
    // needs.  fastc = number of sorted survivors in keys[] (-1: not taken;
    // the radix path below then runs on the untouched scores).
    int fastc = -1;
    {
        const bool need_k = P.top_k > 0 && P.top_k < V && nfin > P.top_k;
        const bool need_p = P.top_p < 1.0f;
        const float span = __fsub_rn(smax, smin);
        if ((need_k || need_p) && nfin > 256 && span > 0.0f && span < INFINITY) {   // few scores: gather + bitonic is cheaper
            const float scale = __fdiv_rn((float) SAMP_NBIN, span);
            int * hist = (int *) e;            // e[] is free until the top-p exps
            int * start = hist + SAMP_NBIN;
            int * cur = start + SAMP_NBIN;
            for (int d = tid; d < SAMP_NBIN; d += nth) { hist[d] = 0; cur[d] = 0; }
            __syncthreads();
            for (int i = tid; i < V; i += nth) {
                const float v = s[i];
                if (v != -INFINITY) atomicAdd(&hist[samp_dbin(v, smin, scale)], 1);
            }
            __syncthreads();
            SAMP_STAMP(16);
            // bins [b0, b0 + bpt) per thread in thread order: warp scan, then
            // every warp scans the warp totals itself (one barrier); the
            // thread holding rank k names its bin; max bin count up to it
            const int b0 = min(SAMP_NBIN, tid * ((SAMP_NBIN + nth - 1) / nth));
            const int bpt = min((SAMP_NBIN + nth - 1) / nth, SAMP_NBIN - b0);
            int tot = 0;
            for (int d = 0; d < bpt; ++d) tot += hist[b0 + d];
            int incl = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += n;
            }
            if (lane == 31) redi[w] = incl;
            if (tid == 0) shi[0] = SAMP_NBIN - 1;
            __syncthreads();
            int wt = lane < nw ? redi[lane] : 0, wi = wt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, wi, o);
                if (lane >= o) wi += n;
            }
            const int excl = __shfl_sync(0xffffffffu, wi - wt, w) + incl - tot;
            {
                int run = excl;
                for (int d = 0; d < bpt; ++d) { start[b0 + d] = run; run += hist[b0 + d]; }
            }
            if (need_k && excl <= P.top_k && P.top_k < excl + tot) {
                for (int d = 0; d < bpt; ++d)
                    if (P.top_k < start[b0 + d] + hist[b0 + d]) { shi[0] = b0 + d; break; }
            }
            __syncthreads();
            const int dsel = shi[0];
            int lmaxb = 0;
            for (int d = 0; d < bpt && b0 + d <= dsel; ++d) lmaxb = max(lmaxb, hist[b0 + d]);
            lmaxb = (int) warp_max((float) lmaxb);
            if (lane == 0) redi[w] = lmaxb;
            __syncthreads();
            const int maxb = (int) warp_max(lane < nw ? (float) redi[lane] : 0.0f);
            if (maxb <= SAMP_BIN_MAX) {
                for (int i = tid; i < V; i += nth) {
                    const float v = s[i];
                    if (v == -INFINITY) continue;
                    const int d = samp_dbin(v, smin, scale);
                    if (d > dsel) continue;
                    const int pos = start[d] + atomicAdd(&cur[d], 1);
                    keys[pos] = ((unsigned long long) desc_key(v) << 32) | (unsigned) i;
                }
                __syncthreads();
                SAMP_STAMP(18);
                const int nsb = start[dsel] + hist[dsel];   // scattered scores, bins 0..dsel
                if (nsb <= 2 * nth) {
                    // each score counts the smaller keys of its bin (<= SAMP_BIN_MAX
                    // reads) and moves to that rank once every count is known
                    unsigned long long kq[2];
                    int pq[2];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const int q = tid + u * nth;
                        pq[u] = -1;
                        if (q < nsb) {
                            const unsigned long long key = keys[q];
                            const int d = samp_dbin(s[(int) (key & 0xffffffffu)], smin, scale);
                            const int b = start[d], n = hist[d];
                            int rk = 0;
                            for (int j = 0; j < n; ++j) rk += keys[b + j] < key ? 1 : 0;
                            kq[u] = key;
                            pq[u] = b + rk;
                        }
                    }
                    __syncthreads();
#pragma unroll
                    for (int u = 0; u < 2; ++u)
                        if (pq[u] >= 0) keys[pq[u]] = kq[u];
                } else {
                    for (int d = tid; d <= dsel; d += nth) {   // insertion sort per bin
                        unsigned long long * kp = keys + start[d];
                        const int n = hist[d];
                        for (int x = 1; x < n; ++x) {
                            const unsigned long long t = kp[x];
                            int y = x - 1;
                            while (y >= 0 && kp[y] > t) { kp[y + 1] = kp[y]; --y; }
                            kp[y + 1] = t;
                        }
                    }
                }
                __syncthreads();
                SAMP_STAMP(19);
                const int ns = start[dsel] + hist[dsel];
                if (need_k) {
                    // threshold = the score at descending rank k; scores in
                    // higher bins are strictly above it, equal scores share its bin
                    if (tid == 0) {
                        const float thr = desc_key_inv((uint32_t) (keys[P.top_k] >> 32));
                        int above = start[dsel];
                        for (int j = start[dsel]; j < ns; ++j) {
                            if (desc_key_inv((uint32_t) (keys[j] >> 32)) > thr) ++above;
                            else break;
                        }
                        const float thr2 = above < P.top_k ? __fsub_rn(thr, 1e-10f) : thr;
                        shf[2] = thr;
                        shi[5] = above;
                        shi[6] = thr2 == thr;   // a nudge that moves thr can admit scores below this bin
                    }
                    __syncthreads();
                    if (shi[6]) {
                        thr_k = shf[2];
                        topk_pending = true;      // applied by the pass below
                        fastc = shi[5];
                    }
                } else {
                    fastc = ns;
                }
                __syncthreads();
            }
        }
    }
    // List mode: with the fast path the survivors of top-k (and below, of
    // top-p) are keys[0 .. nsurv) and s[] is not masked; a bit set marks them
    // for the penalty and the index-order compaction.
    bool listmode = fastc >= 0;
    int nsurv = fastc;
    if (listmode) topk_pending = false;
    if (fastc < 0 && P.top_k > 0 && P.top_k < V && nfin > P.top_k) {
        // digits of 11, 11 and 10 bits: the first already spreads the scores
        // over their exponent and leading mantissa bits, so few keys share a
        // bin and plain shared-memory atomics stay cheap
        // The first pass runs over all scores; the keys of the bin holding rank
        // k are then gathered, and the other two passes run over that list only.
        int * hist = (int *) keys;                    // 2048 bins, free until the top-p gather
        uint32_t * cand = (uint32_t *) keys + 2048;   // keys of the selected first-digit bin
        uint32_t prefix = 0u, maskb = 0u;
        int rank = P.top_k;
        int nc = 0;
        for (int pass = 0; pass < 3; ++pass) {
            const int sh = pass == 0 ? 21 : (pass == 1 ? 10 : 0);
            const int nb = pass == 2 ? 1024 : 2048;
            for (int i = tid; i < nb; i += nth) hist[i] = 0;
            __syncthreads();
            if (pass == 0) {
                for (int i = tid; i < V; i += nth) atomicAdd(&hist[desc_key(s[i]) >> 21], 1);
            } else {
                for (int i = tid; i < nc; i += nth) {
                    const uint32_t k = cand[i];
                    if ((k & maskb) == prefix) atomicAdd(&hist[(k >> sh) & (uint32_t) (nb - 1)], 1);
                }
            }
            __syncthreads();
            // block scan over the bins: thread t owns bins [t*bpt, (t+1)*bpt)
            const int bpt = (nb + nth - 1) / nth;
            const int b0 = min(nb, tid * bpt), b1 = min(nb, b0 + bpt);
            int tot = 0;
            for (int b = b0; b < b1; ++b) tot += hist[b];
            int inc = tot;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += n;
            }
            if (lane == 31) redi[tid >> 5] = inc;
            __syncthreads();
            if (tid < 32) {
                const int nw = nth >> 5;
                const int v = lane < nw ? redi[lane] : 0;
                int vi = v;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int n = __shfl_up_sync(0xffffffffu, vi, o);
                    if (lane >= o) vi += n;
                }
                if (lane < nw) redi[lane] = vi - v;
            }
            __syncthreads();
            const int excl = redi[tid >> 5] + inc - tot;
            if (excl <= rank && rank < excl + tot) {
                int run = excl;
                for (int b = b0; b < b1; ++b) {
                    if (rank < run + hist[b]) { shi[0] = b; shi[1] = run; break; }
                    run += hist[b];
                }
            }
            __syncthreads();
            rank -= shi[1];
            prefix |= ((uint32_t) shi[0]) << sh;
            maskb |= ((uint32_t) (nb - 1)) << sh;
            if (pass == 0) {
                if (tid == 0) shi[3] = 0;
                __syncthreads();
                const uint32_t bsel = (uint32_t) shi[0];
                for (int i0 = 0; i0 < V; i0 += nth) {      // warp-aggregated gather (order irrelevant)
                    const int i = i0 + tid;
                    const uint32_t k = i < V ? desc_key(s[i]) : 0u;
                    const bool take = i < V && (k >> 21) == bsel;
                    const unsigned bal = __ballot_sync(0xffffffffu, take);
                    int base = 0;
                    if (lane == 0 && bal) base = atomicAdd(&shi[3], __popc(bal));
                    base = __shfl_sync(0xffffffffu, base, 0);
                    if (take) cand[base + __popc(bal & ((1u << lane) - 1u))] = k;
                }
                __syncthreads();
                nc = shi[3];
            }
            __syncthreads();
        }
        float thr = desc_key_inv(prefix);
        int above;
        if (thr != 0.0f) {
            above = P.top_k - rank;   // keys before the selected one = scores strictly above thr
        } else {                      // +0 and -0 have distinct keys but compare equal
            int ab = 0;
            for (int i = tid; i < V; i += nth) ab += s[i] > thr ? 1 : 0;
            above = block_sum_i(ab, redi);
        }
        if (above < P.top_k) thr = __fsub_rn(thr, 1e-10f);
        thr_k = thr;
        topk_pending = true;
    }

    SAMP_STAMP(3);
    // (3) top-p (main.cpp:750-772): survivors sorted by score descending
    // (ties by ascending index), sequential float sums in that order.
    if (P.top_p < 1.0f) {
        if (tid == 0) shi[2] = fastc >= 0 ? fastc : 0;
        __syncthreads();
        for (int i0 = 0; fastc < 0 && i0 < V; i0 += nth) {   // warp-aggregated gather (+ top-k drop)
            const int i = i0 + tid;
            float v = i < V ? s[i] : -INFINITY;
            if (topk_pending && i < V && v <= thr_k) { s[i] = -INFINITY; v = -INFINITY; }
            const bool keep = v != -INFINITY;
            const unsigned b = __ballot_sync(0xffffffffu, keep);
            int base = 0;
            if (lane == 0 && b) base = atomicAdd(&shi[2], __popc(b));
            base = __shfl_sync(0xffffffffu, base, 0);
            if (keep) keys[base + __popc(b & ((1u << lane) - 1u))] = ((unsigned long long) desc_key(v) << 32) | (unsigned) i;
        }
        topk_pending = false;
        __syncthreads();
        const int c = shi[2];
        SAMP_STAMP(4);
        if (c > 0 && fastc < 0) {
            int n2 = 2;
            while (n2 < c) n2 <<= 1;
            for (int i = c + tid; i < n2; i += nth) keys[i] = ~0ull;
            __syncthreads();
            // bitonic sort on compare-exchange pairs: pair p touches elements of
            // the 64-element segment p/32 whenever the stride j <= 32, so those
            // stages need only a warp barrier
            for (int k = 2; k <= n2; k <<= 1)
                for (int j = k >> 1; j > 0; j >>= 1) {
                    for (int p = tid; p < n2 / 2; p += nth) {
                        const int i = ((p & ~(j - 1)) << 1) | (p & (j - 1));
                        const unsigned long long x0 = keys[i], x1 = keys[i + j];
                        const bool up = (i & k) == 0;
                        if ((x0 > x1) == up) { keys[i] = x1; keys[i + j] = x0; }
                    }
                    const int jn = j > 1 ? j >> 1 : k;          // next stage's stride
                    if (j >= 64 || (jn >= 64 && k < n2)) __syncthreads();
                    else __syncwarp();
                }
        }
        if (c > 0) {
            __syncthreads();
            SAMP_STAMP(5);
            const float mx = s[(int) (keys[0] & 0xffffffffu)];
            for (int j0 = 0; j0 < c; j0 += 4 * nth) {
                float x[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int j = j0 + u * nth + tid;
                    x[u] = j < c ? __fsub_rn(s[(int) (keys[j] & 0xffffffffu)], mx) : -INFINITY;
                }
                t3_expf_batch<4>(x, a.fx, e2tab);
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int j = j0 + u * nth + tid;
                    if (j < c) e[j] = x[u];
                }
            }
            __syncthreads();
            SAMP_STAMP(6);
            if (tid == 0) shf[0] = seq_sum_f32(e, c);
            __syncthreads();
            SAMP_STAMP(7);
            const float psum = shf[0];
            for (int j = tid; j < c; j += nth) e[j] = __fdiv_rn(e[j], psum);
            __syncthreads();
            // cut = 1 + first j with fl(...fl(e0 + e1)... + ej) >= top_p
            bool ok;
            const double eps = (double) (c + 2) * 0x1p-24 * 1.01 + 1e-12;
            int j = block_first_crossing(c, (double) P.top_p, eps, [&](int q) { return (double) e[q]; }, redd, shi, &ok);
            SAMP_STAMP(20);
            if (!ok) {
                if (tid == 0) shi[3] = seq_cut_f32(e, c, P.top_p);
                __syncthreads();
                j = shi[3];
                __syncthreads();
            }
            SAMP_STAMP(21);
            // the survivors are keys[0 .. cut): list mode from here on (the
            // top-k drop was applied by the gather or is implied by the list)
            listmode = true;
            nsurv = j < c ? j + 1 : c;
        } else {
            listmode = true;   // nothing survived
            nsurv = 0;
        }
    }
    if (topk_pending) {
        for (int i = tid; i < V; i += nth) if (s[i] <= thr_k) s[i] = -INFINITY;
        __syncthreads();
    }

    SAMP_STAMP(8);
    const int nwords = (V + 31) / 32;
    if (listmode) {
        for (int i = tid; i < nwords; i += nth) surv[i] = 0u;
        __syncthreads();
        for (int q = tid; q < nsurv; q += nth) {
            const int i = (int) (keys[q] & 0xffffffffu);
            atomicOr(&surv[i >> 5], 1u << (i & 31));
        }
    }
    // (4) repetition penalty over distinct history ids (main.cpp:774-781)
    if (P.repeat_penalty != 1.0f && hl > 0) {
        for (int i = tid; i < nwords; i += nth) seen[i] = 0u;
        __syncthreads();
        for (int j = tid; j < hl; j += nth) {
            const int t = hist[j];
            if (t < 0 || t >= V) continue;
            const unsigned bit = 1u << (t & 31);
            const unsigned old = atomicOr(&seen[t >> 5], bit);
            if (old & bit) continue;
            const float v = s[t];
            if (listmode ? (surv[t >> 5] & bit) == 0u : v == -INFINITY) continue;
            s[t] = v > 0.0f ? __fdiv_rn(v, P.repeat_penalty) : __fmul_rn(v, P.repeat_penalty);
        }
    }
    __syncthreads();

    SAMP_STAMP(9);
    // (5) softmax over survivors in index order (main.cpp:783-793).  Dropped
    // entries have p = 0 and add nothing to any later sum, so only the
    // survivors are compacted (index order: thread t owns [t*per, (t+1)*per))
    // and exponentiated; one whose exp underflows stays in the list with 0.
    // (list mode: thread t owns bit-set words [t*wper, (t+1)*wper), the
    // same index order)
    const int per = (V + nth - 1) / nth;
    const int i0 = min(V, tid * per), i1 = min(V, i0 + per);
    const int wper = (nwords + nth - 1) / nth;
    const int w0 = min(nwords, tid * wper), w1 = min(nwords, w0 + wper);
    float lm = -INFINITY;
    int cnt = 0;
    if (listmode) {
        for (int q = w0; q < w1; ++q)
            for (unsigned m = surv[q]; m; m &= m - 1u) { lm = fmaxf(lm, s[q * 32 + __ffs(m) - 1]); ++cnt; }
    } else {
        for (int i = i0; i < i1; ++i) { const float v = s[i]; if (v != -INFINITY) { lm = fmaxf(lm, v); ++cnt; } }
    }
    const float mx = block_max(lm, redf);
    int incl = cnt;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
    }
    if (lane == 31) redi[w] = incl;
    __syncthreads();
    if (w == 0) {
        const int nw = nth >> 5;
        int v = lane < nw ? redi[lane] : 0;
        int vi = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int n = __shfl_up_sync(0xffffffffu, vi, o);
            if (lane >= o) vi += n;
        }
        if (lane < nw) redi[lane] = vi - v;
        if (lane == nw - 1) shi[4] = vi;
    }
    __syncthreads();
    {
        int o = redi[w] + incl - cnt;
        if (listmode) {
            for (int q = w0; q < w1; ++q)
                for (unsigned m = surv[q]; m; m &= m - 1u) { const int i = q * 32 + __ffs(m) - 1; lst[o] = i; e[o] = s[i]; ++o; }
        } else {
            for (int i = i0; i < i1; ++i) { const float v = s[i]; if (v != -INFINITY) { lst[o] = i; e[o] = v; ++o; } }
        }
    }
    __syncthreads();
    const int cf = shi[4];
    SAMP_STAMP(10);
    for (int j0 = 0; j0 < cf; j0 += 4 * nth) {
        float x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int j = j0 + u * nth + tid;
            x[u] = j < cf ? __fsub_rn(e[j], mx) : -INFINITY;
        }
        t3_expf_batch<4>(x, a.fx, e2tab);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int j = j0 + u * nth + tid;
            if (j < cf) e[j] = x[u];
        }
    }
    __syncthreads();
    SAMP_STAMP(11);
    if (tid == 0) shf[1] = seq_sum_f32(e, cf);
    __syncthreads();
    SAMP_STAMP(12);
    const float psum = shf[1];
    int tok = 0;
    if (psum != 0.0f) {
        for (int j = tid; j < cf; j += nth) e[j] = __fdiv_rn(e[j], psum);
        __syncthreads();
        if (P.temp <= 0.0f) {
            // (6) first maximum in index order
            const int per2 = (cf + nth - 1) / nth;
            const int c0 = min(cf, tid * per2), c1 = min(cf, c0 + per2);
            float bp = -1.0f; int bi = 0x7fffffff;
            for (int j = c0; j < c1; ++j) if (e[j] > bp) { bp = e[j]; bi = lst[j]; }
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const float op = __shfl_xor_sync(0xffffffffu, bp, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (op > bp || (op == bp && oi < bi)) { bp = op; bi = oi; }
            }
            if (lane == 0) { redf[w] = bp; redi[w] = bi; }
            __syncthreads();
            if (tid == 0) {
                float b = -1.0f; int ix = 0x7fffffff;
                for (int q = 0; q < (nth >> 5); ++q)
                    if (redf[q] > b || (redf[q] == b && redi[q] < ix)) { b = redf[q]; ix = redi[q]; }
                shi[5] = ix;
            }
            __syncthreads();
            tok = shi[5];
        } else {
            // (7) discrete_distribution draw
            uint32_t x1, x2;
            samp_rng_bits(a, slot, rmode, mtx, x1, x2);
            SAMP_STAMP(13);
            const double u = samp_canonical(x1, x2);
            // dsum = sequential double sum of the p (std::accumulate).  When
            // every nonzero p >= 2^-29 all partial sums (< 2) are exact in
            // double, so any order gives the same value.
            float pmin = INFINITY;
            double ls = 0.0;
            for (int j = tid; j < cf; j += nth) { const float pj = e[j]; if (pj > 0.0f) pmin = fminf(pmin, pj); ls += (double) pj; }
            pmin = -block_max(-pmin, redf);
            double dsum;
            if (pmin >= 0x1p-29f) {
                double tot;
                block_excl_scan_d(ls, redd, &tot);
                dsum = tot;
            } else {
                if (tid == 0) redd[32] = seq_sum_f64(e, cf);
                __syncthreads();
                dsum = redd[32];
                __syncthreads();
            }
            SAMP_STAMP(14);
            // lower_bound(cp, u) with cp_j = cp_{j-1} + p_j / dsum and the last
            // entry (index V-1) forced to 1
            int pick;
            if (u <= 0.0) pick = 0;
            else {
                bool ok;
                const double eps = (double) (cf + 16) * 0x1p-52;
                const int j = block_first_crossing(cf, u, eps, [&](int q) { return (double) e[q] / dsum; }, redd, shi, &ok);
                if (ok) pick = j < cf ? lst[j] : V - 1;
                else {
                    if (tid == 0) {
                        int pk = V - 1;
                        double c = 0.0;
                        for (int q = 0; q < cf; ++q) {
                            c = __dadd_rn(c, (double) e[q] / dsum);
                            const double ci = lst[q] == V - 1 ? 1.0 : c;
                            if (ci >= u) { pk = lst[q]; break; }
                        }
                        shi[6] = pk;
                    }
                    __syncthreads();
                    pick = shi[6];
                }
            }
            tok = pick;
        }
    }
    SAMP_STAMP(15);
#undef SAMP_STAMP
    return samp_finish(a, r, slot, hl, tok);
}

__global__ __launch_bounds__(T3B_SAMPLER_THREADS, 1) void sampler_kernel(SampArgs a) {
    extern __shared__ __align__(16) unsigned char smraw[];
    sample_row_block(a, blockIdx.x, smraw);
}

// exp test hook
__global__ void expf_test_kernel(const float * in, float * out, int n, ExpFix fx) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = t3_expf_dev(in[i], fx, g_t3_exp2_tab);
}

// Advance per-row positions after a decode step (graph-captured loops).
__global__ void advance_pos_kernel(int * pos, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) pos[i] += 1;
}

// S3Gen's token input taken from a stream's history on the device, the
// preprocessing s3gen_synthesize_to_wav applies (src/chatterbox_tts.cpp:
// 1389-1398): ids in [0, s3_vocab) kept in order (the start and stop tokens
// drop out), then `sil` copies of the silence token.  One CTA of 1024
// threads compacts the history chunk by chunk (ballot + warp-total scan).
// *n_out = tokens written, or -1 when they do not fit `cap`.
__global__ __launch_bounds__(1024) void s3gen_tokens_kernel(const int * __restrict__ hist, const int * __restrict__ hist_len,
                                                            int s3_vocab, int sil_tok, int sil, int * __restrict__ out,
                                                            int cap, int * __restrict__ n_out) {
    __shared__ int wtot[32];
    __shared__ int base_s;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int n = *hist_len;
    int base = 0;
    for (int c0 = 0; c0 < n; c0 += 1024) {
        const int i = c0 + tid;
        const int t = i < n ? hist[i] : -1;
        const bool keep = t >= 0 && t < s3_vocab;
        const unsigned b = __ballot_sync(0xffffffffu, keep);
        const int in_warp = __popc(b & ((1u << lane) - 1u));
        if (lane == 0) wtot[w] = __popc(b);
        __syncthreads();
        if (w == 0) {
            const int v = wtot[lane];
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += u;
            }
            wtot[lane] = incl - v;                      // exclusive prefix of the warp totals
            if (lane == 31) base_s = base + incl;       // next chunk's base
        }
        __syncthreads();
        const int dst = base + wtot[w] + in_warp;
        if (keep && dst < cap) out[dst] = t;
        base = base_s;
        __syncthreads();
    }
    if (tid < sil && base + tid < cap) out[base + tid] = sil_tok;
    if (tid == 0) *n_out = base + sil <= cap ? base + sil : -1;
}
