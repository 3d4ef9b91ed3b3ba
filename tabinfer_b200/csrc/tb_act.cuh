// tb_act.cuh -- activation preparation shared by the standalone quantizers and
// the GEMV prologues, so a fused GEMV sees bit-identical int8 activations to
// QUANTQ8 (models/qwen3.js:332-358) / RMSNORMQ (qwen3.js:569-612) run alone.
#pragma once
#include "tb_common.cuh"

// Canonical RMSNorm reduction order, shared by every RMSNorm here (fused into a
// GEMV prologue or standalone) so they agree bit for bit.  In a 256-thread
// block, thread t accumulates, with fmaf, the float4s f = t, t+256, ... of the
// row (components x, y, z, w in turn); each warp reduces its 32 partials with
// an xor butterfly; every thread then adds the 8 warp sums in warp order.
__device__ __forceinline__ float sumsq_f4(float4 v, float ss)
{
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    return fmaf(v.w, v.w, ss);
}

// Block-reduce per-thread partial sums of NB rows (NB <= 8) in the canonical
// order; the total of row b is returned in out[b] by every thread.  One
// __syncthreads; `red` holds >= 64 floats and may be reused after the next
// __syncthreads.
template <int NB>
__device__ __forceinline__ void block256_reduce_rows(const float* part, float* red, float* out)
{
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int b = 0; b < NB; b++) {
        const float s = warp_sum(part[b]);
        if (lane == 0) red[b * 8 + wid] = s;
    }
    __syncthreads();
#pragma unroll
    for (int b = 0; b < NB; b++) {
        float t = red[b * 8];
#pragma unroll
        for (int w = 1; w < 8; w++) t = __fadd_rn(t, red[b * 8 + w]);
        out[b] = t;
    }
}

// Sum of squares of one row in the canonical order (H % 4 == 0, 16-byte aligned).
__device__ __forceinline__ float block256_sumsq(const float* __restrict__ xr, int H, float* red)
{
    float ss = 0.0f;
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    for (int f = threadIdx.x; f < (H >> 2); f += 256) ss = sumsq_f4(x4[f], ss);
    float out;
    block256_reduce_rows<1>(&ss, red, &out);
    __syncthreads();
    return out;
}

__device__ __forceinline__ float rms_inv(float sumsq, int H, float eps)
{
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sumsq, (float)H), eps)));
}

// WGSL f32 semantics of the per-32 quantization: scale = maxabs/127,
// q = clamp(round_half_even(x * (1/scale)), -127, 127).
__device__ __forceinline__ float q8_scale(float maxabs) { return __fdiv_rn(maxabs, 127.0f); }
__device__ __forceinline__ float q8_inv(float scale) { return scale > 0.0f ? __frcp_rn(scale) : 0.0f; }
__device__ __forceinline__ int q8_quant(float v, float inv)
{
    return max(-127, min(127, __float2int_rn(__fmul_rn(v, inv))));
}

// Per-32 quantization of one group held one element per lane.
struct Q8Group {
    int q;        // this lane's int8 value
    float scale;  // group scale (maxabs/127)
};
__device__ __forceinline__ Q8Group q8_group(float v)
{
    const float scale = q8_scale(warp_max(fabsf(v)));
    return Q8Group{q8_quant(v, q8_inv(scale)), scale};
}

// models/qwen3.js:3357-3374: f16 bits of an f32, mantissa rounded half-up.
__device__ __forceinline__ uint32_t js_f32_to_f16(float val)
{
    uint32_t x = __float_as_uint(val);
    uint32_t sign = (x >> 16) & 0x8000u, ex = (x >> 23) & 0xffu, mant = x & 0x7fffffu;
    if (ex == 0xffu) return sign | (mant ? 0x7e00u : 0x7c00u);
    int e = (int)ex - 127 + 15;
    if (e >= 31) return sign | 0x7c00u;
    if (e <= 0) {
        if (e < -10) return sign;
        uint32_t m = mant | 0x800000u;
        int shift = 14 - e;
        uint32_t half = (m >> shift) + ((m >> (shift - 1)) & 1u);
        return sign | half;
    }
    return sign | ((((uint32_t)e << 10) | (mant >> 13)) + ((mant >> 12) & 1u));
}
