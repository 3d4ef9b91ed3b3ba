// tb_int4.cu -- int4 G=32 quant-on-arrival and the per-32 int8 activation
// quantizers (QUANTQ8 / QUANTQ8T / RMSNORMQ).  The decode GEMVs live in
// tb_gemv.cu and reuse the same quantization code (tb_act.cuh), so the fused
// GEMV prologues produce bit-identical int8 activations.
//
// Layout (identical to models/qwen3.js:263-270, so packs made by the reference's
// loader or its quant cache are read unchanged): pack u32 [N][K/8], weight k of
// row n in word k/8 at bits 4*(k%8) as q+8; scales f16 [N][K/32].
#include "tb_act.cuh"
#include "tb_internal.h"

namespace {

// ---------------------------------------------------------------------------
// quant-on-arrival (bit-exact with quantizeInt4Bf16, models/qwen3.js:3405-3426)
// ---------------------------------------------------------------------------

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

// JavaScript Math.round on a double (ties toward +inf; NaN/Inf unchanged).
__device__ __forceinline__ double js_round(double v)
{
    if (isnan(v) || isinf(v)) return v;
    double f = floor(v);
    return __dsub_rn(v, f) >= 0.5 ? __dadd_rn(f, 1.0) : f;
}

// One thread per (row, 32-group).  The JS runs in doubles, so does this.
// Row n of the source starts ld elements after row n-1 (ld = K for a whole
// matrix; a column slice of a wider matrix for a row-split shard: the groups
// of a slice that starts at a multiple of 32 are the full matrix's groups).
__global__ void __launch_bounds__(256) k_quant_int4_g32(const uint16_t* __restrict__ w, uint32_t* __restrict__ pack,
                                                        uint16_t* __restrict__ scales, long long ngroups,
                                                        long long gpr, long long ld)
{
    tb_pdl_wait();
    for (long long gi = blockIdx.x * (long long)blockDim.x + threadIdx.x; gi < ngroups;
         gi += (long long)gridDim.x * blockDim.x) {
        const long long row = gi / gpr;
        const uint4* src = reinterpret_cast<const uint4*>(w + row * ld + (gi - row * gpr) * 32);
        uint32_t u[16];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint4 v = src[i];
            u[4 * i + 0] = v.x; u[4 * i + 1] = v.y; u[4 * i + 2] = v.z; u[4 * i + 3] = v.w;
        }
        double maxabs = 0.0;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            uint32_t b = (j & 1) ? (u[j >> 1] >> 16) : (u[j >> 1] & 0xffffu);
            double a = fabs((double)__uint_as_float(b << 16));
            if (a > maxabs) maxabs = a;
        }
        double scale = maxabs > 0.0 ? __ddiv_rn(maxabs, 7.0) : 1e-8;
        uint32_t sb = js_f32_to_f16(__double2float_rn(scale));
        double sval = (double)__half2float(__ushort_as_half((unsigned short)sb));
        double inv = __ddiv_rn(1.0, sval);
        uint32_t words[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int j = 0; j < 32; j++) {
            uint32_t b = (j & 1) ? (u[j >> 1] >> 16) : (u[j >> 1] & 0xffffu);
            double q = js_round(__dmul_rn((double)__uint_as_float(b << 16), inv));
            if (q < -8.0) q = -8.0; else if (q > 7.0) q = 7.0;
            uint32_t nib = isnan(q) ? 0u : (uint32_t)((int)q + 8) & 0xfu;
            words[j >> 3] |= nib << (4 * (j & 7));
        }
        reinterpret_cast<uint4*>(pack)[gi] = make_uint4(words[0], words[1], words[2], words[3]);
        scales[gi] = (uint16_t)sb;
    }
}

// bf16ToF16bits, models/qwen3.js:3386-3390: the loader's f16 copy of the
// embedding table and norm weights (bf16 -> f32 exactly -> f16 rounded half-up).
__global__ void __launch_bounds__(256) k_bf16_to_f16_js(const uint16_t* __restrict__ in, uint16_t* __restrict__ out,
                                                        long long n)
{
    tb_pdl_wait();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = (uint16_t)js_f32_to_f16(__uint_as_float((uint32_t)in[i] << 16));
}

// ---------------------------------------------------------------------------
// per-32 int8 activation quantization (QUANTQ8 / QUANTQ8T / RMSNORMQ)
// ---------------------------------------------------------------------------

// One warp per (row, 32-group); lane j owns element j (q8_group, tb_act.cuh).
__device__ __forceinline__ void q8_group_store(float v, int lane, int8_t* xq, float* xs, int32_t* xsum16)
{
    const Q8Group qg = q8_group(v);
    xq[lane] = (int8_t)qg.q;
    int s = qg.q;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);   // sums within each half-warp
    if (lane == 0) *xs = qg.scale;
    if (xsum16 && (lane & 15) == 0) xsum16[lane >> 4] = s;
}

__global__ void __launch_bounds__(256) k_quant_q8(const float* __restrict__ x, int8_t* __restrict__ xq,
                                                  float* __restrict__ xs, int32_t* __restrict__ xsum16,
                                                  long long ngroups)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    const int lane = threadIdx.x & 31;
    for (long long g = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; g < ngroups;
         g += ((long long)gridDim.x * blockDim.x) >> 5) {
        float v = x[g * 32 + lane];
        q8_group_store(v, lane, xq + g * 32, xs + g, xsum16 ? xsum16 + 2 * g : nullptr);
    }
}

// RMSNORMQ (qwen3.js:569-612): one 256-thread CTA per row.  inv = 1/sqrt(mean(x^2)+eps),
// normalized = (x*inv)*w, then the per-32 quantization above.
__global__ void __launch_bounds__(256) k_rmsnorm_q8(const float* __restrict__ x, const uint16_t* __restrict__ w16,
                                                    float eps, int H, int8_t* __restrict__ xq,
                                                    float* __restrict__ xs, int32_t* __restrict__ xsum16)
{
    __shared__ float red[80];
    tb_pdl_wait();
    tb_pdl_trigger();
    const int row = blockIdx.x, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const float* xr = x + (long long)row * H;
    const float inv = rms_inv(block256_sumsq(xr, H, red), H, eps);
    const int ng = H / 32;
    for (int g = wid; g < ng; g += 8) {
        int i = g * 32 + lane;
        float v = __fmul_rn(__fmul_rn(xr[i], inv), tb_h2f(w16[i]));
        q8_group_store(v, lane, xq + (long long)row * H + g * 32, xs + (long long)row * ng + g,
                       xsum16 ? xsum16 + (long long)row * (H / 16) + 2 * g : nullptr);
    }
}

}  // namespace

// N x K slice of a row-major bf16 matrix with row stride ld (elements; w and
// ld*2 bytes 16-byte aligned) -> int4 G32 pack [N][K/8] + f16 scales [N][K/32].
int tb_quant_int4_strided_impl(tb_ctx* ctx, const uint16_t* w, int64_t ld, uint32_t* pack, uint16_t* scales,
                               int64_t N, int64_t K)
{
    TB_REQUIRE(ctx, TB_ALIGNED(w, 16) && ld % 8 == 0 && ld >= K, "quant_int4: source must be 16-byte aligned rows");
    long long ng = N * (K / 32);
    int grid = (int)std::min<long long>((ng + 255) / 256, (long long)ctx->num_sms * 16);
    cudaError_t e = tb_launch(ctx, k_quant_int4_g32, dim3(grid), dim3(256), 0, w, pack, scales, ng,
                              (long long)(K / 32), (long long)ld);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "quant_int4 launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

int tb_quant_q8_impl(tb_ctx* ctx, const float* x, int8_t* xq, float* xs, int32_t* xsum16, int64_t T, int64_t K)
{
    TB_REQUIRE(ctx, x && xq && xs, "null pointer");
    TB_REQUIRE(ctx, T > 0 && K > 0 && K % 32 == 0, "bad shape T=%lld K=%lld", (long long)T, (long long)K);
    long long ng = T * (K / 32);
    int grid = (int)std::min<long long>((ng * 32 + 255) / 256, (long long)ctx->num_sms * 8);
    cudaError_t e = tb_launch(ctx, k_quant_q8, dim3(grid), dim3(256), 0, x, xq, xs, xsum16, ng);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "quant_q8 launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

extern "C" {

TB_API int tb_quant_int4_g32(tb_ctx* ctx, const uint16_t* w, uint32_t* pack, uint16_t* scales, int64_t N, int64_t K)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, w && pack && scales, "null pointer");
    TB_REQUIRE(ctx, N > 0 && K > 0 && K % 32 == 0, "bad shape N=%lld K=%lld (K%%32 must be 0)", (long long)N, (long long)K);
    TB_REQUIRE(ctx, TB_ALIGNED(w, 16) && TB_ALIGNED(pack, 16) && TB_ALIGNED(scales, 2), "misaligned pointer");
    return tb_quant_int4_strided_impl(ctx, w, K, pack, scales, N, K);
}

TB_API int tb_convert_bf16_f16(tb_ctx* ctx, const uint16_t* in, uint16_t* out, int64_t n)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, in && out && n >= 0, "null pointer or negative size");
    if (n == 0) return TB_OK;
    int grid = (int)std::min<long long>((n + 255) / 256, (long long)ctx->num_sms * 16);
    cudaError_t e = tb_launch(ctx, k_bf16_to_f16_js, dim3(grid), dim3(256), 0, in, out, (long long)n);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "bf16_to_f16 launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_quant_q8(tb_ctx* ctx, const float* x, int8_t* xq, float* xs, int32_t* xsum16, int64_t T, int64_t K)
{
    if (!ctx) return TB_ERR_INVALID;
    return tb_quant_q8_impl(ctx, x, xq, xs, xsum16, T, K);
}

TB_API int tb_rmsnorm_q8(tb_ctx* ctx, const float* x, const uint16_t* w16, float eps, int8_t* xq, float* xs,
                         int32_t* xsum16, int64_t T, int64_t H)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, x && w16 && xq && xs, "null pointer");
    TB_REQUIRE(ctx, T > 0 && T <= 65535 && H > 0 && H % 32 == 0, "bad shape T=%lld H=%lld", (long long)T, (long long)H);
    TB_REQUIRE(ctx, TB_ALIGNED(x, 16), "x must be 16-byte aligned");
    cudaError_t e = tb_launch(ctx, k_rmsnorm_q8, dim3((unsigned)T), dim3(256), 0, x, w16, eps, (int)H, xq, xs, xsum16);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "rmsnorm_q8 launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

}  // extern "C"
