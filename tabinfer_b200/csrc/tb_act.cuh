// tb_act.cuh -- activation preparation shared by the standalone quantizers and
// the GEMV prologues, so a fused GEMV sees bit-identical int8 activations to
// QUANTQ8 (models/qwen3.js:332-358) / RMSNORMQ (qwen3.js:569-612) run alone.
#pragma once
#include "tb_common.cuh"

// Sum of squares of xr[0..H) by a 256-thread block, in a fixed order
// (thread-strided fmaf, warp butterfly, then warp 0 over the 8 warp sums).
// Every thread returns the same value.  `red` is >= 32 floats of shared memory.
__device__ __forceinline__ float block256_sumsq(const float* __restrict__ xr, int H, float* red)
{
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < H; i += 256) { float v = xr[i]; ss = fmaf(v, v, ss); }
    ss = warp_sum(ss);
    __syncthreads();
    if (lane == 0) red[wid] = ss;
    __syncthreads();
    if (wid == 0) {
        float t = lane < 8 ? red[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) red[8] = t;
    }
    __syncthreads();
    return red[8];
}

// block256_sumsq for NB rows at once (same per-row order and result), reading
// element i of row b through `at(b, i)`.  out[b] valid in every thread.
template <int NB, typename At>
__device__ __forceinline__ void block256_sumsq_rows(At at, int H, float* red, float* out)
{
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    float ss[NB];
#pragma unroll
    for (int b = 0; b < NB; b++) ss[b] = 0.0f;
    for (int i = threadIdx.x; i < H; i += 256) {
#pragma unroll
        for (int b = 0; b < NB; b++) { const float v = at(b, i); ss[b] = fmaf(v, v, ss[b]); }
    }
#pragma unroll
    for (int b = 0; b < NB; b++) ss[b] = warp_sum(ss[b]);
    __syncthreads();
    if (lane == 0) {
#pragma unroll
        for (int b = 0; b < NB; b++) red[b * 8 + wid] = ss[b];
    }
    __syncthreads();
    if (wid == 0) {
#pragma unroll
        for (int b = 0; b < NB; b++) {
            float t = lane < 8 ? red[b * 8 + lane] : 0.0f;
            t = warp_sum(t);
            if (lane == 0) red[64 + b] = t;
        }
    }
    __syncthreads();
#pragma unroll
    for (int b = 0; b < NB; b++) out[b] = red[64 + b];
    __syncthreads();
}

__device__ __forceinline__ float rms_inv(float sumsq, int H, float eps)
{
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sumsq, (float)H), eps)));
}

// Per-32 int8 quantization of one group held one element per lane (WGSL f32
// semantics: scale = maxabs/127, q = clamp(round_half_even(x * (1/scale)))).
struct Q8Group {
    int q;        // this lane's int8 value
    float scale;  // group scale (maxabs/127)
};
__device__ __forceinline__ Q8Group q8_group(float v)
{
    const float m = warp_max(fabsf(v));
    const float scale = __fdiv_rn(m, 127.0f);
    const float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    int q = __float2int_rn(__fmul_rn(v, inv));
    return Q8Group{max(-127, min(127, q)), scale};
}
