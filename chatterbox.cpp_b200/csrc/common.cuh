// common.cuh — shared device helpers for the T3 decode kernels.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#define T3B_HD 64            // head dimension of T3 (n_embd / n_head = 1024 / 16)
#define T3B_ATTN_CHUNK 128   // keys per attention CTA (one key per thread)
#define T3B_ATTN_ROWS_MIN 8  // from this many query rows on, one CTA per (row, head) walks all keys

// S3Gen's token input (src/chatterbox_tts.cpp:1389-1398,
// include/tts-cpp/chatterbox/s3gen_pipeline.h:15): its speech vocabulary,
// the silence token and the lookahead silence appended to a final chunk.
#define T3B_S3_VOCAB 6561
#define T3B_S3_SILENCE 4299
#define T3B_S3_LOOKAHEAD 3

// Device-side error word bits (read back by the host after a launch).
#define T3B_DEVERR_TOKEN   1u   // token id outside the embedding table
#define T3B_DEVERR_POS     2u   // position outside the KV cache / wpe table
#define T3B_DEVERR_TIMEOUT 4u   // a bounded spin-wait gave up

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide reductions for blockDim.x a multiple of 32 (<= 1024).  `red`
// is a shared scratch of >= 32 words.  Every thread gets the result.
__device__ __forceinline__ float block_sum(float v, float * red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float r = lane < nw ? red[lane] : 0.0f;
    r = warp_sum(r);
    return r;
}
__device__ __forceinline__ float block_max(float v, float * red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    float r = lane < nw ? red[lane] : -INFINITY;
    r = warp_max(r);
    return r;
}
__device__ __forceinline__ int block_sum_i(int v, int * red) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum_i(v);
    __syncthreads();
    if (lane == 0) red[w] = v;
    __syncthreads();
    int r = lane < nw ? red[lane] : 0;
    r = warp_sum_i(r);
    return r;
}

// ggml GELU (tanh approximation) with the CPU backend's f16 lookup-table
// semantics: argument and result rounded through f16, |x| >= 10 short-cut.
__device__ __forceinline__ float gelu_ggml(float x) {
    if (x <= -10.0f) return 0.0f;
    if (x >= 10.0f) return x;
    const float xh = __half2float(__float2half_rn(x));
    const float c = 0.79788456080286535587989211986876f, a = 0.044715f;
    // 0.5*x*(1 + tanh(c*x*(1 + a*x*x))), evaluated left to right without
    // contraction.
    const float ax = __fmul_rn(a, xh), axx = __fmul_rn(ax, xh);
    const float inner = __fmul_rn(__fmul_rn(c, xh), __fadd_rn(1.0f, axx));
    const float g = __fmul_rn(__fmul_rn(0.5f, xh), __fadd_rn(1.0f, tanhf(inner)));
    return __half2float(__float2half_rn(g));
}

__device__ __forceinline__ uint32_t ld_nc_u32(const void * p) {
    return __ldg((const unsigned int *) p);
}
