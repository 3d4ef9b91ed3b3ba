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

// QUANTQ8 of one 32-group held by 8 consecutive lanes (lane & 7 = j4 holds
// elements 4*j4 .. 4*j4+3), stored in the permuted dp4a layout of the GEMV
// activation (act: xlo uint4 [G], xhi uint4 [G], s8 int [G] = 8*sum(q), sf float
// [G] = scale): the same bits as stage_q8<1, false>.  nat (warp-uniform): the
// natural-order layout of the ternary GEMVs instead (word j4 of the group holds
// elements 4*j4 .. 4*j4+3, s8 = sum(q)): the same bits as stage_q8<1, true>.
// Every lane of the warp calls it (shuffles); live: this lane's group is real
// and is stored.
__device__ __forceinline__ void q8_store_group4(const float e[4], int g, bool live, unsigned char* act, int G,
                                                bool nat = false)
{
    uint4* xlo = reinterpret_cast<uint4*>(act);
    uint4* xhi = xlo + G;
    int* xs8 = reinterpret_cast<int*>(xhi + G);
    float* xsf = reinterpret_cast<float*>(xs8 + G);
    float mx = fmaxf(fmaxf(fabsf(e[0]), fabsf(e[1])), fmaxf(fabsf(e[2]), fabsf(e[3])));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    const float scale = q8_scale(mx), is = q8_inv(scale);
    const int q0 = q8_quant(e[0], is), q1 = q8_quant(e[1], is), q2 = q8_quant(e[2], is), q3 = q8_quant(e[3], is);
    if (nat) {
        int sum = q0 + q1 + q2 + q3;
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        sum += __shfl_xor_sync(0xffffffffu, sum, 4);
        const int j4 = threadIdx.x & 7;
        if (live) {
            reinterpret_cast<uint32_t*>((j4 < 4 ? xlo : xhi) + g)[j4 & 3] =
                ((uint32_t)q0 & 0xffu) | (((uint32_t)q1 & 0xffu) << 8) | (((uint32_t)q2 & 0xffu) << 16) |
                ((uint32_t)q3 << 24);
            if (j4 == 0) { xs8[g] = sum; xsf[g] = scale; }
        }
        return;
    }
    // this lane's k = 4*j4 .. 4*j4+3 of the group: weight word j4/2, half j4&1
    const uint32_t ev = ((uint32_t)q0 & 0xffu) | (((uint32_t)q2 & 0xffu) << 8);
    const uint32_t od = ((uint32_t)q1 & 0xffu) | (((uint32_t)q3 & 0xffu) << 8);
    const uint32_t ev_p = __shfl_xor_sync(0xffffffffu, ev, 1), od_p = __shfl_xor_sync(0xffffffffu, od, 1);
    int sum = q0 + q1 + q2 + q3;
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    const int j4 = threadIdx.x & 7;
    if (live && !(j4 & 1)) {
        const int w = j4 >> 1;
        uint32_t* dst = reinterpret_cast<uint32_t*>((w < 2 ? xlo : xhi) + g) + 2 * (w & 1);
        *reinterpret_cast<uint2*>(dst) = make_uint2(ev | (ev_p << 16), od | (od_p << 16));
        if (j4 == 0) { xs8[g] = 8 * sum; xsf[g] = scale; }
    }
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

// ---- fragment-order activation of the tensor-core GEMVs (tb_gemv_mma.cu) ----
// Per 32-group and row slot, 32 bytes holding the k-slots t and 4+t of MMA thread
// t side by side: int4 slot i = k 8i+{0,2,4,6} (the low nibbles of word i), slot
// 4+i = k 8i+{1,3,5,7}; ternary slot s = k 4s..4s+3.  Beside it per (group, row)
// {scale bits, kc}, kc = 2^23 + 2^22 - F * sum(q) (F = 8 int4, 1 ternary): the
// accumulator seed that removes the weights' bias and converts the sum exactly.
constexpr uint32_t MMA_KC_MAGIC = 0x4B400000u;
__device__ __forceinline__ int mma_slot_pos(int k, bool tern)
{
    const int slot = tern ? (k >> 2) : ((k >> 3) + 4 * (k & 1));
    const int byte = tern ? (k & 3) : ((k & 7) >> 1);
    return 8 * (slot & 3) + 4 * (slot >> 2) + byte;
}
// QUANTQ8 of one 32-group held by 8 consecutive lanes (lane & 7 = j4 holds elements
// 4 j4 .. 4 j4 + 3; every lane of the warp calls it), stored in fragment order at row
// slot m of group g: the same int8 values and scale as q8_group on the elements.
__device__ __forceinline__ void mma_store_group4(const float e[4], int g, int m, int ts, bool tern,
                                                 unsigned char* xa, uint2* xk)
{
    float mx = fmaxf(fmaxf(fabsf(e[0]), fabsf(e[1])), fmaxf(fabsf(e[2]), fabsf(e[3])));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    const float scale = q8_scale(mx), is = q8_inv(scale);
    const int j4 = threadIdx.x & 7;
    unsigned char* row = xa + ((size_t)g * ts + m) * 32;
    int sum = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int q = q8_quant(e[i], is);
        sum += q;
        row[mma_slot_pos(4 * j4 + i, tern)] = (unsigned char)(q & 0xff);
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
    if (j4 == 0) xk[(size_t)g * ts + m] = make_uint2(__float_as_uint(scale), MMA_KC_MAGIC - (tern ? 1u : 8u) * (uint32_t)sum);
}

