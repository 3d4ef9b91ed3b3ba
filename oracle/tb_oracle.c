/*
 * tb_oracle.c -- CPU restatement of TabInfer's quantized-GEMV hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * product in tabinfer_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference legs of bench.py may load it; the product never
 * calls it and has no CPU fallback.
 *
 * Every function restates the reference algorithm in plain C and cites the
 * reference file:line it follows (paths relative to the TabInfer checkout).
 * Floating-point semantics follow the reference's own language:
 *   - the int4 quantizer runs in JavaScript doubles (models/qwen3.js), with
 *     Float32Array stores and the hand-written f32->f16 rounding;
 *   - the WGSL kernels compute in f32 (WGSL round() = round-half-to-even,
 *     pack4x8snorm = floor(0.5 + 127*clamp(v,-1,1)));
 *   - the ternary kernels follow Rust f32 (no FMA contraction, f32::round =
 *     half away from zero) in native/crates/n2-kernels/src/tern.rs.
 * Floating outputs whose reference order is a parallel tree are returned as
 * f64 "exact-ish" sums; the tests compare those within stated tolerances.
 *
 * Parity pins: tests/test_oracle.py checks these functions against the
 * reference's own golden data (numpy pack_ternary from native/tools/pack_bin.py,
 * the tern.rs known-answer tests, and the qwen3.js self-test fixtures).
 *
 * Built by oracle/build.py with gcc -O2 (no -ffast-math, -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define TBO_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* f16 / bf16 helpers                                                        */
/* ------------------------------------------------------------------------ */

static inline uint32_t f32_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float bits_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* f32 -> f16 bits exactly as models/qwen3.js:3357-3374 (f32ToF16): the value is
 * first stored to a Float32Array (double->f32 round-to-nearest-even), then the
 * mantissa is truncated and incremented when the first dropped bit is set
 * (round-half-up on magnitude, not round-to-even). */
TBO_API uint16_t tbo_f32_to_f16_js(float val)
{
    uint32_t x = f32_bits(val);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ex = (x >> 23) & 0xffu;
    uint32_t mant = x & 0x7fffffu;
    if (ex == 0xffu) return (uint16_t)(sign | (mant ? 0x7e00u : 0x7c00u));
    int e = (int)ex - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        uint32_t m = mant | 0x800000u;
        int shift = 14 - e;
        uint32_t half = m >> shift;
        if ((m >> (shift - 1)) & 1u) half += 1;
        return (uint16_t)(sign | half);
    }
    uint32_t half = ((uint32_t)e << 10) | (mant >> 13);
    if ((mant >> 12) & 1u) half += 1;
    return (uint16_t)(sign | half);
}

/* f16 bits -> exact value, models/qwen3.js:3397-3400 (f16ToF32scalar, JS double). */
TBO_API double tbo_f16_to_f64(uint16_t h)
{
    int s = (h >> 15) & 1, e = (h >> 10) & 0x1f, f = h & 0x3ff;
    double sg = s ? -1.0 : 1.0;
    if (e == 0) return sg * ldexp((double)f, -24);
    if (e == 31) return f ? NAN : sg * INFINITY;
    return sg * ldexp(1.0 + f / 1024.0, e - 15);
}

static inline double bf16_to_f64(uint16_t u) { return (double)bits_f32((uint32_t)u << 16); }

/* JavaScript Math.round: nearest integer, ties toward +infinity; NaN/Inf pass. */
static inline double js_round(double x)
{
    if (isnan(x) || isinf(x)) return x;
    double f = floor(x);
    return (x - f) >= 0.5 ? f + 1.0 : f;
}

/* ------------------------------------------------------------------------ */
/* int4 G=32 quantizer -- models/qwen3.js:3405-3426 (quantizeInt4Bf16)       */
/* ------------------------------------------------------------------------ */

/* in: bf16 bits [N,K] row-major.  out: pack u32 [N,K/8] (k=8w+i at bits 4i,
 * nibble = q+8), scales f16 bits [N,K/32].  K % 32 == 0. */
TBO_API void tbo_quant_int4_g32(const uint16_t *w, int64_t N, int64_t K,
                                uint32_t *pack, uint16_t *scales)
{
    const int64_t G = 32, wpr = K / 8, gpr = K / G;
    memset(pack, 0, (size_t)(N * wpr) * sizeof(uint32_t));
    for (int64_t n = 0; n < N; n++) {
        for (int64_t g = 0; g < gpr; g++) {
            const uint16_t *src = w + n * K + g * G;
            double maxabs = 0.0;
            for (int j = 0; j < G; j++) {
                double v = fabs(bf16_to_f64(src[j]));
                if (v > maxabs) maxabs = v;              /* NaN never wins */
            }
            double scale = maxabs > 0 ? maxabs / 7.0 : 1e-8;
            uint16_t sb = tbo_f32_to_f16_js((float)scale);
            scales[n * gpr + g] = sb;
            double inv = 1.0 / tbo_f16_to_f64(sb);      /* 1/0 -> +Inf, as JS */
            for (int j = 0; j < G; j++) {
                int64_t k = g * G + j;
                double q = js_round(bf16_to_f64(src[j]) * inv);
                if (q < -8) q = -8; else if (q > 7) q = 7;
                /* (NaN + 8) & 0xF == 0 in JS (ToInt32(NaN) = 0) */
                uint32_t nib = isnan(q) ? 0u : ((uint32_t)((int)q + 8) & 0xFu);
                pack[n * wpr + (k >> 3)] |= nib << (4 * (k & 7));
            }
        }
    }
}

/* Dequantize as the self-test oracle does, models/qwen3.js:3073-3074
 * (w = (nib-8)*f16ToF32(scale), stored to a Float32Array). */
TBO_API void tbo_dequant_int4_g32(const uint32_t *pack, const uint16_t *scales,
                                  int64_t N, int64_t K, float *w)
{
    const int64_t wpr = K / 8, gpr = K / 32;
    for (int64_t n = 0; n < N; n++)
        for (int64_t k = 0; k < K; k++) {
            uint32_t word = pack[n * wpr + (k >> 3)];
            int nib = (int)((word >> (4 * (k & 7))) & 0xFu);
            w[n * K + k] = (float)((nib - 8) * tbo_f16_to_f64(scales[n * gpr + k / 32]));
        }
}

/* f32-activation int4 GEMV oracle: y[b,n] = sum_k x[b,k]*Wdq[n,k], accumulated
 * in double exactly as the JS self-test reference loop (qwen3.js:3089), which
 * is the math of gemvQ (qwen3.js:276-321) without its f32 reduction order. */
TBO_API void tbo_gemv_int4_f32act(const float *x, const uint32_t *pack,
                                  const uint16_t *scales, int64_t N, int64_t K,
                                  int64_t batch, double *y)
{
    const int64_t wpr = K / 8, gpr = K / 32;
    for (int64_t n = 0; n < N; n++) {
        for (int64_t b = 0; b < batch; b++) {
            double a = 0.0;
            for (int64_t g = 0; g < gpr; g++) {
                double s = tbo_f16_to_f64(scales[n * gpr + g]);
                for (int j = 0; j < 32; j++) {
                    int64_t k = g * 32 + j;
                    int nib = (int)((pack[n * wpr + (k >> 3)] >> (4 * (k & 7))) & 0xFu);
                    float wv = (float)((nib - 8) * s);
                    a += (double)x[b * K + k] * (double)wv;
                }
            }
            y[b * N + n] = a;
        }
    }
}

/* ------------------------------------------------------------------------ */
/* f16 prefill GEMM -- gemmqWgsl / gemmQ, qwen3.js:964-1026: the activation   */
/* tile is stored as f16 (vec4<f16>(X), round to nearest even), each weight as */
/* f16((nib - 8) * f32(scale)) (the product is exact in f32, one rounding),    */
/* and the f16 products are summed in f32 on the GPU; here in f64.             */
/* ------------------------------------------------------------------------ */

/* x [M,K] f32 (or bf16 bits when x_bf16), pack/scales of W [N,K] -> y [M,N]. */
TBO_API void tbo_gemm_int4_f16(const void *x, int x_bf16, const uint32_t *pack, const uint16_t *scales,
                               int64_t M, int64_t N, int64_t K, double *y)
{
    const int64_t wpr = K / 8, gpr = K / 32;
    double *wrow = (double *)malloc(sizeof(double) * (size_t)K);
    double *xf = (double *)malloc(sizeof(double) * (size_t)(M * K));
    for (int64_t i = 0; i < M * K; i++) {
        float v;
        if (x_bf16) {
            uint32_t b = (uint32_t)((const uint16_t *)x)[i] << 16;
            memcpy(&v, &b, 4);
        } else {
            v = ((const float *)x)[i];
        }
        xf[i] = (double)(_Float16)v;          /* round to nearest even */
    }
    for (int64_t n = 0; n < N; n++) {
        for (int64_t k = 0; k < K; k++) {
            const float s = (float)tbo_f16_to_f64(scales[n * gpr + k / 32]);
            const int nib = (int)((pack[n * wpr + (k >> 3)] >> (4 * (k & 7))) & 0xFu);
            wrow[k] = (double)(_Float16)((float)(nib - 8) * s);
        }
        for (int64_t m = 0; m < M; m++) {
            double a = 0.0;
            const double *xr = xf + m * K;
            for (int64_t k = 0; k < K; k++) a += xr[k] * wrow[k];
            y[m * N + n] = a;
        }
    }
    free(wrow);
    free(xf);
}

/* ------------------------------------------------------------------------ */
/* int8 per-32 activation quantizer -- QUANTQ8 qwen3.js:332-358 (one row),    */
/* QUANTQ8T qwen3.js:1210-1231 (T rows).  WGSL f32 semantics.                */
/* ------------------------------------------------------------------------ */

/* x [T,K] f32 -> xq int8 [T,K] (natural k order; the reference packs 4 per
 * u32 little-endian, which is the same bytes), xs f32 [T,K/32] = maxabs/127,
 * xsum i32 [T,K/16] (per-16 sums, QUANTQ8 only; may be NULL). */
TBO_API void tbo_quant_q8(const float *x, int64_t T, int64_t K,
                          int8_t *xq, float *xs, int32_t *xsum)
{
    const int64_t gpr = K / 32;
    for (int64_t t = 0; t < T; t++)
        for (int64_t g = 0; g < gpr; g++) {
            const float *src = x + t * K + g * 32;
            float m = 0.0f;
            for (int j = 0; j < 32; j++) m = fmaxf(m, fabsf(src[j]));
            float scale = m / 127.0f;
            float inv = scale > 0.0f ? 1.0f / scale : 0.0f;
            xs[t * gpr + g] = scale;
            int q[32];
            for (int j = 0; j < 32; j++) {
                float r = rintf(src[j] * inv);           /* WGSL round: half to even */
                int v = (int)r;
                q[j] = v < -127 ? -127 : (v > 127 ? 127 : v);
                xq[t * K + g * 32 + j] = (int8_t)q[j];
            }
            if (xsum) {
                int s0 = 0, s1 = 0;
                for (int j = 0; j < 16; j++) { s0 += q[j]; s1 += q[16 + j]; }
                xsum[t * (K / 16) + 2 * g] = s0;
                xsum[t * (K / 16) + 2 * g + 1] = s1;
            }
        }
}

/* Fused RMSNorm -> int8, RMSNORMQ qwen3.js:569-612 (one row per batch entry).
 * inv = 1/sqrt(mean(x^2)+eps) (sum of squares taken in double here; the WGSL
 * tree order differs by <1 ulp), then normalized = (x*inv)*w and the group
 * quantization of QUANTQ8.  Also returns inv per row for diagnostics. */
TBO_API void tbo_rmsnorm_q8(const float *x, const uint16_t *w16, int64_t T,
                            int64_t H, float eps, int8_t *xq, float *xs,
                            int32_t *xsum, float *inv_out)
{
    const int64_t ng = H / 32;
    for (int64_t t = 0; t < T; t++) {
        const float *xr = x + t * H;
        double ss = 0.0;
        for (int64_t i = 0; i < H; i++) ss += (double)xr[i] * (double)xr[i];
        float inv = 1.0f / sqrtf((float)ss / (float)H + eps);
        if (inv_out) inv_out[t] = inv;
        for (int64_t g = 0; g < ng; g++) {
            float mx = 0.0f;
            for (int j = 0; j < 32; j++) {
                int64_t i = g * 32 + j;
                float v = (xr[i] * inv) * (float)tbo_f16_to_f64(w16[i]);
                mx = fmaxf(mx, fabsf(v));
            }
            float scale = mx / 127.0f;
            float invs = scale > 0.0f ? 1.0f / scale : 0.0f;
            xs[t * ng + g] = scale;
            int s0 = 0, s1 = 0;
            for (int j = 0; j < 32; j++) {
                int64_t i = g * 32 + j;
                float v = ((xr[i] * inv) * (float)tbo_f16_to_f64(w16[i])) * invs;
                int q = (int)rintf(v);
                q = q < -127 ? -127 : (q > 127 ? 127 : q);
                xq[t * H + i] = (int8_t)q;
                if (j < 16) s0 += q; else s1 += q;
            }
            if (xsum) { xsum[t * (H / 16) + 2 * g] = s0; xsum[t * (H / 16) + 2 * g + 1] = s1; }
        }
    }
}

/* int8-activation int4 GEMV/GEMM math, GEMVDP4 qwen3.js:359-400 and
 * gemmdp4Wgsl qwen3.js:1326-1388: per (row, 32-group) an exact int32 dot of
 * (nib-8) with the int8 activation, scaled by f32(s16)*xs.  The per-group
 * products are summed in double (the WGSL order is a workgroup tree). */
TBO_API void tbo_gemv_int4_q8act(const int8_t *xq, const float *xs,
                                 const uint32_t *pack, const uint16_t *scales,
                                 int64_t N, int64_t K, int64_t batch, double *y)
{
    const int64_t wpr = K / 8, gpr = K / 32;
    for (int64_t n = 0; n < N; n++)
        for (int64_t b = 0; b < batch; b++) {
            double a = 0.0;
            for (int64_t g = 0; g < gpr; g++) {
                int32_t dot = 0;
                for (int j = 0; j < 32; j++) {
                    int64_t k = g * 32 + j;
                    int nib = (int)((pack[n * wpr + (k >> 3)] >> (4 * (k & 7))) & 0xFu);
                    dot += (nib - 8) * (int32_t)xq[b * K + k];
                }
                float s = (float)tbo_f16_to_f64(scales[n * gpr + g]) * xs[b * gpr + g];
                a += (double)s * (double)dot;
            }
            y[b * N + n] = a;
        }
}

/* Fused gate+up+SiLU, gateupDP4Wgsl qwen3.js:679-728: swi = silu(g)*u with
 * g,u from the int8-activation math above.  Returned in double. */
TBO_API void tbo_gateup_q8act(const int8_t *xq, const float *xs,
                              const uint32_t *gpack, const uint16_t *gscales,
                              const uint32_t *upack, const uint16_t *uscales,
                              int64_t I, int64_t H, int64_t batch, double *swi)
{
    double *g = (double *)malloc(sizeof(double) * (size_t)(I * batch));
    double *u = (double *)malloc(sizeof(double) * (size_t)(I * batch));
    tbo_gemv_int4_q8act(xq, xs, gpack, gscales, I, H, batch, g);
    tbo_gemv_int4_q8act(xq, xs, upack, uscales, I, H, batch, u);
    for (int64_t i = 0; i < I * batch; i++) swi[i] = g[i] / (1.0 + exp(-g[i])) * u[i];
    free(g); free(u);
}

/* ------------------------------------------------------------------------ */
/* Ternary, WebGPU layout -- models/qwen3.js                                 */
/* ------------------------------------------------------------------------ */

/* quantizeTernaryBf16, qwen3.js:3435-3469.  Returns 1 and fills pack u32
 * [N,K/16] + f16 scales [N,K/32] when every 32-group holds only {-s, 0, +s}
 * (nonzero magnitude bits at most TOL = 2 below the group's maximum mx);
 * returns 0 (the reference's null) otherwise or when K % 64 != 0.
 * Code w+1: 1 for a zero magnitude, 0 negative, 2 positive; weight k at bits
 * 8*(k&3) + 2*((k>>2)&3) of word k>>4; scale = bf16ToF16bits(mx)
 * (qwen3.js:3386-3390: bf16 -> f32 exactly, then f32ToF16). */
TBO_API int tbo_quant_tern_wgsl(const uint16_t *w, int64_t N, int64_t K,
                                uint32_t *pack, uint16_t *scales)
{
    const int TOL = 2;
    if (K % 64 != 0) return 0;
    const int64_t wpr = K / 16, gpr = K / 32;
    memset(pack, 0, (size_t)(N * wpr) * sizeof(uint32_t));
    for (int64_t n = 0; n < N; n++)
        for (int64_t g = 0; g < gpr; g++) {
            const uint16_t *src = w + n * K + g * 32;
            int mx = 0;
            for (int j = 0; j < 32; j++) { int m = src[j] & 0x7FFF; if (m > mx) mx = m; }
            scales[n * gpr + g] = tbo_f32_to_f16_js(bits_f32((uint32_t)mx << 16));
            for (int j = 0; j < 32; j++) {
                int64_t k = g * 32 + j;
                int m = src[j] & 0x7FFF;
                if (m != 0 && mx - m > TOL) return 0;
                uint32_t c = m == 0 ? 1u : ((src[j] & 0x8000) ? 0u : 2u);
                pack[n * wpr + (k >> 4)] |= c << (((k & 3) << 3) + ((k >> 2) & 3) * 2);
            }
        }
    return 1;
}

/* gemvTern2Wgsl / gemvTernWgsl, qwen3.js:449-546 (and the ternary tiles of the
 * prefill GEMM, gemmdp4Wgsl(tern) :1357-1359, whose QUANTQ8T rows equal
 * QUANTQ8's): per (row, 32-group) the exact int32 sum((c-1) * xq), scaled by
 * f32(s16) * xs (an f32 product, as the shader's f32(sc) * xsc).  Groups summed
 * in double. */
TBO_API void tbo_gemv_tern_wgsl_q8act(const int8_t *xq, const float *xs,
                                      const uint32_t *pack, const uint16_t *scales,
                                      int64_t N, int64_t K, int64_t batch, double *y)
{
    const int64_t wpr = K / 16, gpr = K / 32;
    for (int64_t n = 0; n < N; n++)
        for (int64_t b = 0; b < batch; b++) {
            double a = 0.0;
            for (int64_t g = 0; g < gpr; g++) {
                int32_t dot = 0;
                for (int j = 0; j < 32; j++) {
                    int64_t k = g * 32 + j;
                    int c = (int)((pack[n * wpr + (k >> 4)] >> (((k & 3) << 3) + ((k >> 2) & 3) * 2)) & 3u);
                    dot += (c - 1) * (int32_t)xq[b * K + k];
                }
                float s = (float)tbo_f16_to_f64(scales[n * gpr + g]) * xs[b * gpr + g];
                a += (double)s * (double)dot;
            }
            y[b * N + n] = a;
        }
}

/* gateupTern2Wgsl, qwen3.js:747-810: swi = silu(g) * u of the two ternary GEMVs. */
TBO_API void tbo_gateup_tern_wgsl_q8act(const int8_t *xq, const float *xs,
                                        const uint32_t *gpack, const uint16_t *gscales,
                                        const uint32_t *upack, const uint16_t *uscales,
                                        int64_t I, int64_t H, int64_t batch, double *swi)
{
    double *g = (double *)malloc(sizeof(double) * (size_t)(I * batch));
    double *u = (double *)malloc(sizeof(double) * (size_t)(I * batch));
    tbo_gemv_tern_wgsl_q8act(xq, xs, gpack, gscales, I, H, batch, g);
    tbo_gemv_tern_wgsl_q8act(xq, xs, upack, uscales, I, H, batch, u);
    for (int64_t i = 0; i < I * batch; i++) swi[i] = g[i] / (1.0 + exp(-g[i])) * u[i];
    free(g); free(u);
}

/* ------------------------------------------------------------------------ */
/* Ternary Q2_0_g64 -- native/crates/n2-kernels/src/tern.rs                  */
/* ------------------------------------------------------------------------ */

/* tern.rs:131-160 (pack_ternary) == native/tools/pack_bin.py:19-29.
 * s = max|w| per 64; code 1 if |w| < 0.5s, else 0 (negative) / 2 (positive);
 * code c of a group lives in byte c%16 at bit 2*(c/16). */
TBO_API void tbo_pack_ternary(const float *w, int64_t N, int64_t K,
                              uint8_t *codes, float *scales)
{
    const int64_t nb = K / 64;
    memset(codes, 0, (size_t)(N * K / 4));
    for (int64_t r = 0; r < N; r++)
        for (int64_t b = 0; b < nb; b++) {
            const float *g = w + r * K + b * 64;
            float s = 0.0f;
            for (int c = 0; c < 64; c++) { float a = fabsf(g[c]); s = a > s ? a : s; }
            scales[r * nb + b] = s;
            float thr = s * 0.5f;
            for (int c = 0; c < 64; c++) {
                uint8_t code = fabsf(g[c]) < thr ? 1 : (g[c] < 0.0f ? 0 : 2);
                codes[r * (K / 4) + b * 16 + (c & 15)] |= (uint8_t)(code << (2 * (c >> 4)));
            }
        }
}

/* tern.rs:206-222 (quantize_act_into): per-vector scale = 127/amax (1.0 when
 * amax == 0), act = round-half-away(x*scale) clamped to +-127, xsum per 64.
 * Returns the scale.  Applied to each of T rows independently. */
TBO_API void tbo_quantize_act(const float *x, int64_t T, int64_t K,
                              int8_t *act, int32_t *xsum, float *scale_out)
{
    for (int64_t t = 0; t < T; t++) {
        const float *xr = x + t * K;
        float amax = 0.0f;
        for (int64_t i = 0; i < K; i++) { float a = fabsf(xr[i]); amax = a > amax ? a : amax; }
        float scale = amax > 0.0f ? 127.0f / amax : 1.0f;
        for (int64_t i = 0; i < K; i++) {
            float v = roundf(xr[i] * scale);
            v = v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v);
            act[t * K + i] = (int8_t)v;
        }
        for (int64_t b = 0; b < K / 64; b++) {
            int32_t s = 0;
            for (int i = 0; i < 64; i++) s += act[t * K + b * 64 + i];
            xsum[t * (K / 64) + b] = s;
        }
        scale_out[t] = scale;
    }
}

/* The WASM CPU engine's quantize (cpu/kernel/src/lib.rs:566-606): per-vector
 * asc = amax/127 (1e-9 when amax == 0), inv = 1/asc, act = nearest-even(x*inv)
 * clamped to +-127 (f32x4_nearest then the saturating narrow), xsum per 64.
 * Returns asc -- the factor the caller multiplies the GEMV output by -- where
 * tern.rs returns 127/amax.  Applied to each of T rows independently. */
TBO_API void tbo_quantize_act_wasm(const float *x, int64_t T, int64_t K,
                                   int8_t *act, int32_t *xsum, float *asc_out)
{
    for (int64_t t = 0; t < T; t++) {
        const float *xr = x + t * K;
        float amax = 0.0f;
        for (int64_t i = 0; i < K; i++) { float a = fabsf(xr[i]); amax = a > amax ? a : amax; }
        const float asc = amax > 0.0f ? amax / 127.0f : 1e-9f;
        const float inv = 1.0f / asc;
        for (int64_t i = 0; i < K; i++) {
            float v = rintf(xr[i] * inv);          /* round to nearest, ties to even */
            v = v < -127.0f ? -127.0f : (v > 127.0f ? 127.0f : v);
            act[t * K + i] = (int8_t)v;
        }
        for (int64_t b = 0; b < K / 64; b++) {
            int32_t s = 0;
            for (int i = 0; i < 64; i++) s += act[t * K + b * 64 + i];
            xsum[t * (K / 64) + b] = s;
        }
        asc_out[t] = asc;
    }
}

/* tern.rs:79-119 (gemv_tern_scalar), the portable reference every backend is
 * validated against: per row, acc += s*dot and sxs += s*xsum in block order
 * (f32, separately rounded multiply and add), out = acc - sxs.
 * Batched form = the same order per column (cpu/kernel/src/lib.rs:299-307). */
TBO_API void tbo_gemv_tern_scalar(float *out, const uint8_t *codes, const float *scales,
                                  const int8_t *act, const int32_t *xsum,
                                  int64_t N, int64_t K, int64_t batch)
{
    const int64_t nb = K / 64;
    for (int64_t t = 0; t < batch; t++) {
        const int8_t *a = act + t * K;
        const int32_t *xs = xsum + t * nb;
        for (int64_t r = 0; r < N; r++) {
            const uint8_t *rc = codes + r * (K / 4);
            const float *rs = scales + r * nb;
            float acc = 0.0f, sxs = 0.0f;   /* -ffp-contract=off keeps each op rounded */
            for (int64_t b = 0; b < nb; b++) {
                int32_t dot = 0;
                for (int j = 0; j < 4; j++)
                    for (int i = 0; i < 16; i++)
                        dot += (int32_t)((rc[b * 16 + i] >> (2 * j)) & 3) * (int32_t)a[b * 64 + j * 16 + i];
                float s = rs[b];
                float p = s * (float)dot;
                acc = acc + p;
                float q = s * (float)xs[b];
                sxs = sxs + q;
            }
            out[t * N + r] = acc - sxs;
        }
    }
}

/* tern.rs:166-189 (gemv_dequant_reference): the independent oracle,
 * w = (code-1)*s in f32, product in f32, accumulated in f64. */
TBO_API void tbo_gemv_tern_dequant(float *out, const uint8_t *codes, const float *scales,
                                   const int8_t *act, int64_t N, int64_t K, int64_t batch)
{
    const int64_t nb = K / 64;
    for (int64_t t = 0; t < batch; t++)
        for (int64_t r = 0; r < N; r++) {
            double acc = 0.0;
            for (int64_t k = 0; k < K; k++) {
                int64_t b = k / 64, c = k % 64;
                uint8_t raw = codes[r * (K / 4) + b * 16 + (c % 16)];
                int code = (raw >> (2 * (c / 16))) & 3;
                float wv = (float)(code - 1) * scales[r * nb + b];
                acc += (double)(wv * (float)act[t * K + k]);
            }
            out[t * N + r] = (float)acc;
        }
}

/* ------------------------------------------------------------------------ */
/* int8 KV cache and split-KV decode attention                               */
/* ------------------------------------------------------------------------ */

/* WGSL pack4x8snorm component: floor(0.5 + 127*clamp(v,-1,1)). */
static inline int8_t snorm8(float v)
{
    float c = v < -1.0f ? -1.0f : (v > 1.0f ? 1.0f : v);
    return (int8_t)floorf(0.5f + 127.0f * c);
}

/* KVQW qwen3.js:2180-2210 / attnPrep qwen3.js:2277-2295: per 32-element group,
 * m = max(1e-12, max|x|), q = snorm8(x/m), scale = m.  x [n] with n % 32 == 0. */
TBO_API void tbo_kv_quant_q8(const float *x, int64_t n, int8_t *q, float *scale)
{
    for (int64_t g = 0; g < n / 32; g++) {
        float m = 1e-12f;
        for (int j = 0; j < 32; j++) m = fmaxf(m, fabsf(x[g * 32 + j]));
        for (int j = 0; j < 32; j++) q[g * 32 + j] = snorm8(x[g * 32 + j] / m);
        scale[g] = m;
    }
}

/* Per-head RMSNorm + RoPE split-half, attnPrepWgsl qwen3.js:2257-2275 and
 * ROPEQK qwen3.js:1722-1761 (T=1 at position pos).  In place on x[nH*hd].
 * Computed in double (the WGSL pow/cos/sin are not bit-specified). */
TBO_API void tbo_head_norm_rope(double *x, const uint16_t *w16, int64_t nH, int64_t hd,
                                int64_t pos, double theta, double eps)
{
    double *rk = (double *)malloc(sizeof(double) * (size_t)hd);
    const int64_t half = hd / 2;
    for (int64_t h = 0; h < nH; h++) {
        double *v = x + h * hd;
        double ss = 0.0;
        for (int64_t j = 0; j < hd; j++) ss += v[j] * v[j];
        double inv = 1.0 / sqrt(ss / (double)hd + eps);
        for (int64_t j = 0; j < hd; j++) rk[j] = v[j] * inv * tbo_f16_to_f64(w16[j]);
        for (int64_t j = 0; j < hd; j++) {
            int64_t fi = j < half ? j : j - half;
            double ang = (double)pos * pow(theta, -2.0 * (double)fi / (double)hd);
            double partner = j < half ? rk[j + half] : rk[j - half];
            double rot = j < half ? -partner : partner;
            v[j] = rk[j] * cos(ang) + rot * sin(ang);
        }
    }
    free(rk);
}

/* Split-KV streaming decode attention over the int8 KV cache,
 * attnDecStreamQ8Wgsl qwen3.js:2077-2164 + ATTN_DEC_COMBINE qwen3.js:2048-2069.
 * The split/online-softmax structure is exact math, so the oracle is a plain
 * softmax over all S keys in double:
 *   score_t = sum_g (sum_{j in g} q_j * unpack(K_tj)) * Ks_tg / sqrt(hd)
 *   out     = sum_t softmax(score)_t * Vs_tg * unpack(V_tj)
 * with unpack(c) = max(c/127, -1) (WGSL unpack4x8snorm).  GQA: query head hq
 * reads kv head hq / (nHq/nKv).  Layout: Kq int8 [S][nKv*hd], Ks f32
 * [S][nKv*hd/32]; q f32 [nHq*hd]; out double [nHq*hd]. */
TBO_API void tbo_attn_decode_q8(const float *q, const int8_t *Kq, const float *Ks,
                                const int8_t *Vq, const float *Vs, int64_t S,
                                int64_t nHq, int64_t nKv, int64_t hd, double *out)
{
    const int64_t grp = nHq / nKv, row = nKv * hd, rowg = row / 32;
    double *sc = (double *)malloc(sizeof(double) * (size_t)(S > 0 ? S : 1));
    const double scale = 1.0 / sqrt((double)hd);
    for (int64_t hq = 0; hq < nHq; hq++) {
        int64_t hk = hq / grp;
        double mx = -INFINITY;
        for (int64_t t = 0; t < S; t++) {
            double s = 0.0;
            for (int64_t g = 0; g < hd / 32; g++) {
                double p = 0.0;
                for (int j = 0; j < 32; j++) {
                    int64_t d = g * 32 + j;
                    double kv = fmax((double)Kq[t * row + hk * hd + d] / 127.0, -1.0);
                    p += (double)q[hq * hd + d] * kv;
                }
                s += p * (double)Ks[t * rowg + hk * (hd / 32) + g];
            }
            sc[t] = s * scale;
            if (sc[t] > mx) mx = sc[t];
        }
        double l = 0.0;
        for (int64_t t = 0; t < S; t++) { sc[t] = exp(sc[t] - mx); l += sc[t]; }
        for (int64_t d = 0; d < hd; d++) {
            double o = 0.0;
            for (int64_t t = 0; t < S; t++) {
                double vv = fmax((double)Vq[t * row + hk * hd + d] / 127.0, -1.0);
                o += sc[t] * (double)Vs[t * rowg + hk * (hd / 32) + d / 32] * vv;
            }
            out[hq * hd + d] = S > 0 ? o / l : 0.0;
        }
    }
    free(sc);
}

/* The same decode attention at the operand precision of the reference's f16
 * prefill kernel (attnF16Wgsl via _q8PrefillWgsl, qwen3.js:2396-2532, 2540-2560:
 * q, the dequantized K and V (max(c/127,-1) * scale, formed in f32) and the
 * softmax weights p are f16 values), summed exactly here; l = sum of the
 * unrounded p as in its f32 lsh. */
TBO_API void tbo_attn_decode_q8_f16ops(const float *q, const int8_t *Kq, const float *Ks,
                                       const int8_t *Vq, const float *Vs, int64_t S,
                                       int64_t nHq, int64_t nKv, int64_t hd, double *out)
{
    const int64_t grp = nHq / nKv, row = nKv * hd, rowg = row / 32;
    double *sc = (double *)malloc(sizeof(double) * (size_t)(S > 0 ? S : 1));
    const double scale = 1.0 / sqrt((double)hd);
    for (int64_t hq = 0; hq < nHq; hq++) {
        int64_t hk = hq / grp;
        double mx = -INFINITY;
        for (int64_t t = 0; t < S; t++) {
            double s = 0.0;
            for (int64_t d = 0; d < hd; d++) {
                float kf = fmaxf((float)Kq[t * row + hk * hd + d] / 127.0f, -1.0f) * Ks[t * rowg + hk * (hd / 32) + d / 32];
                s += (double)(_Float16)q[hq * hd + d] * (double)(_Float16)kf;
            }
            sc[t] = s * scale;
            if (sc[t] > mx) mx = sc[t];
        }
        double l = 0.0;
        for (int64_t t = 0; t < S; t++) { sc[t] = exp(sc[t] - mx); l += sc[t]; }
        for (int64_t d = 0; d < hd; d++) {
            double o = 0.0;
            for (int64_t t = 0; t < S; t++) {
                float vf = fmaxf((float)Vq[t * row + hk * hd + d] / 127.0f, -1.0f) * Vs[t * rowg + hk * (hd / 32) + d / 32];
                o += (double)(_Float16)(float)sc[t] * (double)(_Float16)vf;
            }
            out[hq * hd + d] = S > 0 ? o / l : 0.0;
        }
    }
    free(sc);
}

/* int8-KV prefill attention, attentionQ8 with T > 1 (qwen3.js:2534-2577: the
 * flash kernels ATTN_WGSL / attnF16Wgsl with int8 tile loads): query i of T sits
 * at position S - T + i and sees keys 0 .. S - T + i (the causal mask
 * gk <= gqpos); per query this is the decode attention above over S - T + i + 1
 * keys.  q [T][nHq*hd], out [T][nHq*hd] in double. */
TBO_API void tbo_attn_prefill_q8(const float *q, const int8_t *Kq, const float *Ks,
                                 const int8_t *Vq, const float *Vs, int64_t T, int64_t S,
                                 int64_t nHq, int64_t nKv, int64_t hd, double *out)
{
    for (int64_t i = 0; i < T; i++)
        tbo_attn_decode_q8(q + i * nHq * hd, Kq, Ks, Vq, Vs, S - T + i + 1, nHq, nKv, hd, out + i * nHq * hd);
}

/* GUMBEL_WGSL (qwen3.js:2719-2730): noise of flat index i under seed is
 * temp * -log(-log(u)), u = (f32(pcg(i ^ seed*2654435761) >> 8) + 0.5) / 2^24;
 * pcg = the PCG output permutation of the WGSL.  u is formed in f32 as the
 * shader forms it: for h >> 8 >= 2^23 the + 0.5 rounds (to even), and at
 * h >> 8 = 2^24 - 1 it gives u = 1 exactly and an infinite noise -- the shader's
 * comment says u is never 1, its f32 arithmetic says otherwise.  The logs are
 * taken in double. */
static uint32_t pcg_hash(uint32_t v0)
{
    uint32_t v = v0 * 747796405u + 2891336453u;
    uint32_t w = ((v >> ((v >> 28u) + 4u)) ^ v) * 277803737u;
    return (w >> 22u) ^ w;
}

TBO_API void tbo_gumbel_noise(int64_t total, uint32_t seed, double temp, double *out)
{
    for (int64_t i = 0; i < total; i++) {
        uint32_t h = pcg_hash((uint32_t)i ^ (seed * 2654435761u));
        volatile float uf = (float)(h >> 8);
        uf = uf + 0.5f;
        double u = (double)(uf / 16777216.0f);
        out[i] = temp * (-log(-log(u)));
    }
}

/* Split count rule, _decNsplit qwen3.js:2354 (DEC_TK = 128, max 16 splits). */
TBO_API int tbo_dec_nsplit(int64_t S)
{
    int64_t a = (S + 127) / 128, b = (S + 447) / 448;
    if (b < 4) b = 4;
    int64_t n = a < b ? a : b;
    if (n > 16) n = 16;
    return n < 1 ? 1 : (int)n;
}

/* Argmax over x[n]: index of the maximum, lowest index on ties (the WGSL
 * kernels at qwen3.js:2625-2690 tie-break by thread order; the result on
 * distinct maxima is the same). */
TBO_API int64_t tbo_argmax(const float *x, int64_t n)
{
    int64_t bi = 0;
    float bv = -INFINITY;
    for (int64_t i = 0; i < n; i++) if (x[i] > bv) { bv = x[i]; bi = i; }
    return bi;
}


/* ------------------------------------------------------------------------ */
/* int3 MoE of LFM2.5 (models/lfm25.js)                                       */
/* ------------------------------------------------------------------------ */

/* engine/webgpu-engine.js:217-236 f32ToF16: half-up on mantissa bit 12, the
 * rounded mantissa ORed into the exponent field (a carry survives only when the
 * exponent's low bit is clear). */
TBO_API uint16_t tbo_engine_f32_to_f16(float v)
{
    uint32_t x;
    memcpy(&x, &v, 4);
    uint32_t sign = (x >> 16) & 0x8000u, mant = x & 0x007fffffu;
    int ex = (int)((x >> 23) & 0xffu);
    if (ex == 255) return (uint16_t)(sign | (mant ? 0x7e00u : 0x7c00u));
    int e = ex - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant = (mant | 0x00800000u) >> (1 - e);
        return (uint16_t)(sign | ((mant + 0x00001000u) >> 13));
    }
    return (uint16_t)(sign | ((uint32_t)e << 10) | ((mant + 0x00001000u) >> 13));
}

/* bf16 -> int3 of the LFM2.5 benchmark configuration (group 32 or 128; no
 * reference counterpart): per (row, group) scale = f16(max|w|/4) by the
 * engine's f32ToF16, q = clamp(round-to-nearest-even(w / scale), -4, 3) in f32,
 * stored q + 4 in the _requant43 bitplanes; max|w| = 0 -> scale 0, q = 0. */
TBO_API void tbo_quant_int3(const uint16_t *w, int64_t rows, int64_t K, int64_t group, uint32_t *p3, uint16_t *s3)
{
    const int64_t ng = rows * (K / group), gp = group / 32;
    for (int64_t gi = 0; gi < ng; gi++) {
        const uint16_t *src = w + gi * group;
        float m = 0.0f;
        for (int64_t i = 0; i < group; i++) {
            float a = fabsf(bits_f32((uint32_t)src[i] << 16));
            m = a > m ? a : m;
        }
        const uint16_t sh = tbo_engine_f32_to_f16(m / 4.0f);
        const float sc = (float)tbo_f16_to_f64(sh);
        for (int64_t j = 0; j < gp; j++) {
            uint32_t b0 = 0, b1 = 0, b2 = 0;
            for (int i = 0; i < 32; i++) {
                const float v = bits_f32((uint32_t)src[j * 32 + i] << 16);
                int q = 0;
                if (sc > 0.0f) {
                    q = (int)rintf(v / sc);
                    q = q > 3 ? 3 : (q < -4 ? -4 : q);
                }
                const uint32_t st = (uint32_t)(q + 4);
                b0 |= (st & 1u) << i;
                b1 |= ((st >> 1) & 1u) << i;
                b2 |= ((st >> 2) & 1u) << i;
            }
            p3[(gi * gp + j) * 3] = b0; p3[(gi * gp + j) * 3 + 1] = b1; p3[(gi * gp + j) * 3 + 2] = b2;
        }
        s3[gi] = sh;
    }
}

/* _requant43, lfm25.js:833-855: int4 group (nibble q+8) -> int3 bitplanes of
 * stored value q3+4 with q3 = clamp(Math.round(q4 * (4/m)), -4, 3), m = max|q4|;
 * scale = f32(f16(s4) * m / 4) through the engine's f32ToF16; m = 0 -> scale 0
 * and planes {0, 0, ~0}.  JS doubles. */
TBO_API void tbo_requant43(const uint32_t *pack4, const uint16_t *s4, int64_t rows, int64_t K, uint32_t *p3,
                           uint16_t *s3)
{
    const int64_t ng = rows * (K / 32);
    for (int64_t gi = 0; gi < ng; gi++) {
        int q4[32], m = 0;
        for (int i = 0; i < 32; i++) {
            q4[i] = (int)((pack4[gi * 4 + (i >> 3)] >> (4 * (i & 7))) & 15u) - 8;
            int a = q4[i] < 0 ? -q4[i] : q4[i];
            if (a > m) m = a;
        }
        if (m == 0) {
            p3[gi * 3] = 0; p3[gi * 3 + 1] = 0; p3[gi * 3 + 2] = 0xFFFFFFFFu;
            s3[gi] = tbo_engine_f32_to_f16(0.0f);
            continue;
        }
        const double ratio = 4.0 / (double)m;
        const float s3f = (float)(tbo_f16_to_f64(s4[gi]) * (double)m / 4.0);
        uint32_t b0 = 0, b1 = 0, b2 = 0;
        for (int i = 0; i < 32; i++) {
            double v = (double)q4[i] * ratio;
            double f = floor(v);
            int q = (int)((v - f) >= 0.5 ? f + 1.0 : f);   /* Math.round: ties toward +inf */
            if (q > 3) q = 3; else if (q < -4) q = -4;
            uint32_t st = (uint32_t)(q + 4);
            b0 |= (st & 1u) << i;
            b1 |= ((st >> 1) & 1u) << i;
            b2 |= ((st >> 2) & 1u) << i;
        }
        p3[gi * 3] = b0; p3[gi * 3 + 1] = b1; p3[gi * 3 + 2] = b2;
        s3[gi] = tbo_engine_f32_to_f16(s3f);
    }
}

/* ROUTER_WGSL, lfm25.js:111-141: sigmoid scores, K first-maximum passes over
 * score + bias (strict >: lower expert on ties), weights score / (sum + 1e-6).
 * f32 arithmetic as the shader (exp in double, rounded to f32). */
TBO_API void tbo_moe_router(const float *logits, const float *bias, int64_t T, int64_t nE, int64_t K, uint32_t *idx,
                            float *wt)
{
    for (int64_t t = 0; t < T; t++) {
        float sc[256], sel[256];
        for (int64_t e = 0; e < nE; e++) {
            float ex = (float)exp(-(double)logits[t * nE + e]);
            sc[e] = 1.0f / (1.0f + ex);
            sel[e] = sc[e] + bias[e];
        }
        float sum = 0.0f;
        for (int64_t k = 0; k < K; k++) {
            int64_t best = 0;
            float bv = -1.0e30f;
            for (int64_t j = 0; j < nE; j++)
                if (sel[j] > bv) { bv = sel[j]; best = j; }
            sel[best] = -2.0e30f;
            idx[t * K + k] = (uint32_t)best;
            wt[t * K + k] = sc[best];
            sum += sc[best];
        }
        for (int64_t k = 0; k < K; k++) wt[t * K + k] = wt[t * K + k] / (sum + 1e-6f);
    }
}

/* idxGemv3 (lfm25.js:1924-1973) for one pair: y[n] = sum_g s[row,g] * sum_i (q_i - 4) x[32g+i],
 * row = e*N + n; f64. */
static void moe_gemv3_row_g(const uint32_t *p3, const uint16_t *s3, int64_t e, int64_t N, int64_t Kc, const double *x,
                            double *y, int64_t sg)
{
    const int64_t G = Kc / 32;
    for (int64_t n = 0; n < N; n++) {
        const int64_t row = e * N + n;
        double acc = 0.0;
        for (int64_t g = 0; g < G; g++) {
            const uint32_t *w = p3 + (row * G + g) * 3;
            double sum = 0.0;
            for (int i = 0; i < 32; i++) {
                int st = (int)(((w[0] >> i) & 1u) | (((w[1] >> i) & 1u) << 1) | (((w[2] >> i) & 1u) << 2));
                sum += (double)(st - 4) * x[g * 32 + i];
            }
            acc += tbo_f16_to_f64(s3[row * (G / sg) + g / sg]) * sum;
        }
        y[n] = acc;
    }
}

/* MoE FFN (w1/w3 gate+up with SiLU, w2 down, MOECOMBINE lfm25.js:1982-2000):
 * x_out[t] = x_in_res[t] + sum_k wt[t,k] * W2_e(silu(W1_e a_t) * W3_e a_t). */
TBO_API void tbo_moe_ffn_int3_g(const float *a, const uint32_t *idx, const float *wt, const uint32_t *w1p,
                                const uint16_t *w1s, const uint32_t *w3p, const uint16_t *w3s, const uint32_t *w2p,
                                const uint16_t *w2s, int64_t T, int64_t K, int64_t H, int64_t I, int64_t group,
                                double *out)
{
    const int64_t sg = group / 32;
    double *xa = (double *)malloc(sizeof(double) * (size_t)H);
    double *g = (double *)malloc(sizeof(double) * (size_t)I);
    double *u = (double *)malloc(sizeof(double) * (size_t)I);
    double *o = (double *)malloc(sizeof(double) * (size_t)H);
    for (int64_t t = 0; t < T; t++) {
        for (int64_t h = 0; h < H; h++) { xa[h] = a[t * H + h]; out[t * H + h] = 0.0; }
        for (int64_t k = 0; k < K; k++) {
            const int64_t e = idx[t * K + k];
            moe_gemv3_row_g(w1p, w1s, e, I, H, xa, g, sg);
            moe_gemv3_row_g(w3p, w3s, e, I, H, xa, u, sg);
            for (int64_t i = 0; i < I; i++) g[i] = g[i] / (1.0 + exp(-g[i])) * u[i];
            moe_gemv3_row_g(w2p, w2s, e, H, I, g, o, sg);
            for (int64_t h = 0; h < H; h++) out[t * H + h] += (double)wt[t * K + k] * o[h];
        }
    }
    free(xa); free(g); free(u); free(o);
}

TBO_API void tbo_moe_ffn_int3(const float *a, const uint32_t *idx, const float *wt, const uint32_t *w1p,
                              const uint16_t *w1s, const uint32_t *w3p, const uint16_t *w3s, const uint32_t *w2p,
                              const uint16_t *w2s, int64_t T, int64_t K, int64_t H, int64_t I, double *out)
{
    tbo_moe_ffn_int3_g(a, idx, wt, w1p, w1s, w3p, w3s, w2p, w2s, T, K, H, I, 32, out);
}
