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

// Ternary detection + pack of the WebGPU layout (quantizeTernaryBf16,
// models/qwen3.js:3435-3469).  A warp takes 64 consecutive weights of a row
// (two 32-groups), lane l the bf16 pair 2l, 2l+1.  Per group: mx = max of the
// magnitude bits (bits & 0x7fff); the matrix is not ternary when any nonzero
// magnitude sits more than TOL = 2 ulps below its group's mx (then *fail is
// set and the pack is not used); code = 1 for a zero magnitude, else 0 / 2 by
// sign; weight k lands at bits 8*(k%4) + 2*((k/4)%4) of word k/16 (OR-reduced
// over the 8 lanes of a word); scale = bf16ToF16bits(mx).  Source rows are ldw
// u32 (bf16 pairs) apart and cpr chunks long (a column slice of a wider matrix
// when ldw > 32 * cpr); pack == nullptr checks without writing.
__global__ void __launch_bounds__(256) k_quant_tern_wgsl(const uint32_t* __restrict__ w, long long ldw, long long cpr,
                                                         uint32_t* __restrict__ pack, uint16_t* __restrict__ scales,
                                                         long long nchunks, int* __restrict__ fail)
{
    tb_pdl_wait();
    constexpr uint32_t TOL = 2;
    const int lane = threadIdx.x & 31;
    const long long nwarps = (long long)gridDim.x * (blockDim.x >> 5);
    bool bad = false;
    for (long long c = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5); c < nchunks; c += nwarps) {
        const long long row = c / cpr;
        const uint32_t u = __ldg(w + row * ldw + (c - row * cpr) * 32 + lane);   // weights 64c .. 64c+63 of the slice
        const uint32_t lo = u & 0xffffu, hi = u >> 16;
        const uint32_t m0 = lo & 0x7fffu, m1 = hi & 0x7fffu;
        uint32_t mx = max(m0, m1);
#pragma unroll
        for (int o = 1; o < 16; o <<= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        bad |= (m0 != 0u && mx - m0 > TOL) || (m1 != 0u && mx - m1 > TOL);
        const uint32_t c0 = m0 == 0u ? 1u : ((lo & 0x8000u) ? 0u : 2u);
        const uint32_t c1 = m1 == 0u ? 1u : ((hi & 0x8000u) ? 0u : 2u);
        const int k0 = (2 * lane) & 15, k1 = k0 + 1;   // positions inside the 16-weight word
        uint32_t word = (c0 << (((k0 & 3) << 3) + ((k0 >> 2) & 3) * 2)) | (c1 << (((k1 & 3) << 3) + ((k1 >> 2) & 3) * 2));
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) word |= __shfl_xor_sync(0xffffffffu, word, o);
        if (pack && (lane & 7) == 0) pack[c * 4 + (lane >> 3)] = word;
        if (pack && (lane & 15) == 0) scales[c * 2 + (lane >> 4)] = (uint16_t)js_f32_to_f16(__uint_as_float(mx << 16));
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(fail, 1);
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

// The same QUANTQ8T with four elements a lane (8 lanes a 32-group, one 16-byte
// load each): the same group maximum (order-free), scale, rounding and sums as
// k_quant_q8, so the same bits, with four times the bytes in flight a warp.
// nq = element quads (T * K / 4); x 16-byte and xq 4-byte aligned.
__global__ void __launch_bounds__(256) k_quant_q8_v4(const float4* __restrict__ x, uint32_t* __restrict__ xq,
                                                     float* __restrict__ xs, int32_t* __restrict__ xsum16,
                                                     long long nq)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    const int lane = threadIdx.x & 31, j4 = lane & 7;
    const long long stride = (long long)gridDim.x * blockDim.x;
    // the loop bound is the warp's first quad, so every lane of a warp runs the
    // same iterations (shuffles); lanes past the end are not stored
    for (long long base = blockIdx.x * (long long)blockDim.x + threadIdx.x - lane; base < nq; base += stride) {
        const long long f = base + lane;
        const bool live = f < nq;
        const float4 v = live ? __ldg(x + f) : make_float4(0.f, 0.f, 0.f, 0.f);
        float mx = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        const float scale = q8_scale(mx), is = q8_inv(scale);
        const int q0 = q8_quant(v.x, is), q1 = q8_quant(v.y, is), q2 = q8_quant(v.z, is), q3 = q8_quant(v.w, is);
        const long long g = f >> 3;
        if (live) {
            xq[f] = ((uint32_t)q0 & 0xffu) | (((uint32_t)q1 & 0xffu) << 8) | (((uint32_t)q2 & 0xffu) << 16) |
                    ((uint32_t)q3 << 24);
            if (j4 == 0) xs[g] = scale;
        }
        if (xsum16) {   // warp-uniform: sums of each half-group (16 elements, 4 lanes)
            int sm = q0 + q1 + q2 + q3;
            sm += __shfl_xor_sync(0xffffffffu, sm, 1);
            sm += __shfl_xor_sync(0xffffffffu, sm, 2);
            if (live && (j4 & 3) == 0) xsum16[2 * g + (j4 >> 2)] = sm;
        }
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
    if (TB_ALIGNED(x, 16) && TB_ALIGNED(xq, 4)) {
        const long long nq = ng * 8;
        const int grid = (int)std::min<long long>((nq + 255) / 256, (long long)ctx->num_sms * 16);
        cudaError_t e = tb_launch(ctx, k_quant_q8_v4, dim3(grid), dim3(256), 0, reinterpret_cast<const float4*>(x),
                                  reinterpret_cast<uint32_t*>(xq), xs, xsum16, nq);
        if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "quant_q8 launch: %s", cudaGetErrorString(e));
        return TB_OK;
    }
    int grid = (int)std::min<long long>((ng * 32 + 255) / 256, (long long)ctx->num_sms * 8);
    cudaError_t e = tb_launch(ctx, k_quant_q8, dim3(grid), dim3(256), 0, x, xq, xs, xsum16, ng);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "quant_q8 launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

// flag (device int) |= 1 when the N x K slice (rows ld elements apart) is not
// ternary; it must be zero beforehand.  pack == nullptr: check only.
int tb_quant_tern_wgsl_strided_impl(tb_ctx* ctx, const uint16_t* w, int64_t ld, uint32_t* pack, uint16_t* scales,
                                    int64_t N, int64_t K, int* flag)
{
    TB_REQUIRE(ctx, w && flag && K % 64 == 0 && ld % 2 == 0 && ld >= K && N > 0, "quant_tern_wgsl: bad slice");
    const long long nchunks = N * (K / 64);
    int grid = (int)std::min<long long>((nchunks + 7) / 8, (long long)ctx->num_sms * 16);
    cudaError_t e = tb_launch(ctx, k_quant_tern_wgsl, dim3(grid), dim3(256), 0, reinterpret_cast<const uint32_t*>(w),
                              (long long)(ld / 2), (long long)(K / 64), pack, scales, nchunks, flag);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "quant_tern_wgsl launch: %s", cudaGetErrorString(e));
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

TB_API int tb_quant_tern_wgsl_bf16(tb_ctx* ctx, const uint16_t* w, uint32_t* pack, uint16_t* scales, int64_t N,
                                  int64_t K, int* nonternary)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, w && pack && scales && nonternary, "null pointer");
    TB_REQUIRE(ctx, N > 0 && K > 0, "bad shape N=%lld K=%lld", (long long)N, (long long)K);
    TB_REQUIRE(ctx, TB_ALIGNED(w, 4) && TB_ALIGNED(pack, 4) && TB_ALIGNED(scales, 2) && TB_ALIGNED(nonternary, 4),
               "misaligned pointer");
    // K % 64 != 0: not representable in this layout, the caller keeps int4 (qwen3.js:3436)
    cudaError_t e = cudaMemsetAsync(nonternary, K % 64 ? 1 : 0, sizeof(int), ctx->stream);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "memset: %s", cudaGetErrorString(e));
    if (K % 64) return TB_OK;
    return tb_quant_tern_wgsl_strided_impl(ctx, w, K, pack, scales, N, K, nonternary);
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
