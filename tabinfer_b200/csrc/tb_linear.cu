// tb_linear.cu -- the router-level entry points that quantize an f32
// activation into context scratch and run the matching GEMV:
// linearQ (models/qwen3.js:1588-1608, both weight kinds) and Model::linear
// (native/crates/n2-core/src/model.rs:316-339).
#include "tb_internal.h"

static inline size_t up256(size_t v) { return (v + 255) & ~size_t(255); }

extern "C" {

TB_API int tb_linear_int4(tb_ctx* ctx, float* y, const float* x, const uint32_t* pack, const uint16_t* scales,
                          int64_t T, int64_t N, int64_t K, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, T >= 1, "T must be >= 1");
    TB_REQUIRE(ctx, K > 0 && K % 32 == 0, "K must be a positive multiple of 32");
    if (T == 1 && N >= 16384) return tb_gemv_f32_impl(ctx, y, x, pack, scales, N, K, 1, acc);
    if (T >= 2 && T <= 16 && tb_gemv_mma_fits(K, &N, 1, (int)T)) {
        // the DP4A math on the tensor cores, every weight read once for all rows
        void* buf = tb_ctx_scratch(ctx, tb_gemv_mma_act_bytes(K, (int)T));
        if (!buf) return TB_ERR_NOMEM;
        return tb_gemv_mma_impl(ctx, 1, &y, &pack, &scales, &N, x, nullptr, 0.0f, K, (int)T, acc, false, false, buf);
    }
    if (T > 8) {
        // prefill: linearQ's default gemmDP4A (qwen3.js:1605-1607) -- QUANTQ8T rows
        // into context scratch, then the tensor-core GEMM on them
        if (T % 128 != 0 || N % 128 != 0 || K % 128 != 0)
            return tb_fail(ctx, TB_ERR_UNSUPPORTED,
                           "linear_int4: T=%lld > 8 needs T, N and K multiples of 128 (prefill GEMM)", (long long)T);
        const size_t xq_b = up256((size_t)T * K), xs_b = up256((size_t)T * (K / 32) * 4);
        unsigned char* scr = static_cast<unsigned char*>(tb_ctx_scratch(ctx, xq_b + xs_b));
        if (!scr) return TB_ERR_NOMEM;
        int8_t* xq = reinterpret_cast<int8_t*>(scr);
        float* xs = reinterpret_cast<float*>(scr + xq_b);
        int rc = tb_quant_q8_impl(ctx, x, xq, xs, nullptr, T, K);
        if (rc) return rc;
        return tb_gemm_dp4_impl(ctx, y, xq, xs, pack, scales, T, N, K, acc ? 1 : 0, false);
    }
    // quantQ8 / QUANTQ8T runs inside the GEMV prologue (bit-identical int8 rows)
    return tb_gemv_dp4a_impl(ctx, 1, &y, &pack, &scales, &N, x, nullptr, 0.0f, K, (int)T, acc);
}

// linearQ's ternary branch (qwen3.js:1594-1598).  T = 2..16 (K % 256 == 0, N % 8
// == 0) runs the tensor-core GEMV with the same exact group sums; other T <= 8 the
// ternary GEMV
// with quantQ8 in its prologue: per 32-group the same exact int32 sum and f32
// scaling as the reference's gemvTern (T = 1) and gemmTern tiles (T > 1).
// T > 8 quantizes the rows (QUANTQ8T) into context scratch and runs gemmTern
// with its exact group sums (tb_gemm_dp4).
TB_API int tb_linear_tern_wgsl(tb_ctx* ctx, float* y, const float* x, const uint32_t* pack, const uint16_t* scales,
                               int64_t T, int64_t N, int64_t K, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, T >= 1, "T must be >= 1");
    TB_REQUIRE(ctx, K > 0 && K % 64 == 0, "K must be a positive multiple of 64");
    if (T >= 2 && T <= 16 && tb_gemv_mma_fits(K, &N, 1, (int)T)) {
        void* buf = tb_ctx_scratch(ctx, tb_gemv_mma_act_bytes(K, (int)T));
        if (!buf) return TB_ERR_NOMEM;
        return tb_gemv_mma_impl(ctx, 1, &y, &pack, &scales, &N, x, nullptr, 0.0f, K, (int)T, acc, true, false, buf);
    }
    if (T <= 8) return tb_gemv_tern_wgsl_impl(ctx, 1, &y, &pack, &scales, &N, x, nullptr, 0.0f, K, (int)T, acc);
    if (T % 128 != 0 || N % 128 != 0 || K % 128 != 0)
        return tb_fail(ctx, TB_ERR_UNSUPPORTED,
                       "linear_tern_wgsl: T=%lld > 8 needs T, N and K multiples of 128 (prefill GEMM)", (long long)T);
    const size_t xq_b = up256((size_t)T * K), xs_b = up256((size_t)T * (K / 32) * 4);
    unsigned char* scr = static_cast<unsigned char*>(tb_ctx_scratch(ctx, xq_b + xs_b));
    if (!scr) return TB_ERR_NOMEM;
    int8_t* xq = reinterpret_cast<int8_t*>(scr);
    float* xs = reinterpret_cast<float*>(scr + xq_b);
    int rc = tb_quant_q8_impl(ctx, x, xq, xs, nullptr, T, K);
    if (rc) return rc;
    return tb_gemm_dp4_impl(ctx, y, xq, xs, pack, scales, T, N, K, acc ? 1 : 0, true);
}

TB_API int tb_linear_tern(tb_ctx* ctx, float* y, const float* x, const uint8_t* codes, const float* scales, int64_t T,
                          int64_t N, int64_t K)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, T >= 1 && T <= 8, "T must be 1..8");
    TB_REQUIRE(ctx, K > 0 && K % 64 == 0, "K must be a positive multiple of 64");
    size_t act_b = up256((size_t)T * K), xsum_b = up256((size_t)T * (K / 64) * 4), sc_b = up256((size_t)T * 4);
    unsigned char* scr = static_cast<unsigned char*>(tb_ctx_scratch(ctx, act_b + xsum_b + sc_b));
    if (!scr) return TB_ERR_NOMEM;
    int8_t* act = reinterpret_cast<int8_t*>(scr);
    int32_t* xsum = reinterpret_cast<int32_t*>(scr + act_b);
    float* sc = reinterpret_cast<float*>(scr + act_b + xsum_b);
    int rc = tb_quant_act_impl(ctx, x, act, xsum, sc, T, K);
    if (rc) return rc;
    return tb_gemv_tern_impl(ctx, y, codes, scales, act, xsum, N, K, (int)T, sc);
}

}  // extern "C"
