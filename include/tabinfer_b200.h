/*
 * tabinfer_b200.h -- C ABI of the B200 backend for TabInfer's quantized-GEMV
 * hot path (int4 G=32 decode GEMV / prefill GEMM, int8-KV split-KV decode
 * attention, ternary Q2_0_g64 GEMV).
 *
 * Conventions
 *   - every pointer argument named as a tensor is a DEVICE pointer to a
 *     caller-owned buffer (cudaMalloc / torch / cuMemAlloc), dense row-major;
 *   - every call is enqueued on the context's stream and returns without
 *     synchronising; results are valid once that stream reaches the call;
 *   - the return value is a status (TB_OK = 0); on error, tb_last_error(ctx)
 *     holds a message and nothing was enqueued;
 *   - one context per host thread; a context is bound to one CUDA device.
 * The reference interface each entry point replaces is cited beside it
 * (paths inside the TabInfer checkout).
 */
#ifndef TABINFER_B200_H
#define TABINFER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TB_API __attribute__((visibility("default")))

enum {
    TB_OK = 0,
    TB_ERR_INVALID = 1,     /* bad shape, alignment or argument (reference: JS throw / Rust assert) */
    TB_ERR_CUDA = 2,        /* a CUDA runtime call failed */
    TB_ERR_UNSUPPORTED = 3, /* valid request this build does not implement */
    TB_ERR_TIMEOUT = 4,     /* a bounded device-side wait gave up (see tb_ctx_device_error) */
    TB_ERR_NOMEM = 5
};

/* Numerics mode of the int4 GEMV, the two decode routes of linearQ
 * (models/qwen3.js:1597-1602). */
enum {
    TB_ACT_F32 = 0,  /* gemvQ: f32 activations, f32 dequant math (qwen3.js:276-321) */
    TB_ACT_Q8 = 1    /* gemvDP4A: per-32 int8 activations, int32 dot (qwen3.js:332-400) */
};

typedef struct tb_ctx tb_ctx;

/* ---- context --------------------------------------------------------------
 * Replaces the engine object of engine/webgpu-engine.js:72 (init) and the
 * module-level scratch of models/qwen3.js (ensureDp4 :402, ensureDecSplit :2339). */
TB_API int tb_version(void);
TB_API int tb_ctx_create(int device, tb_ctx **out);
TB_API int tb_ctx_destroy(tb_ctx *ctx);
/* Order all later calls on this stream (a cudaStream_t); NULL = the context's own
 * (non-blocking) stream.  To use the legacy default stream pass cudaStreamLegacy. */
TB_API int tb_ctx_set_stream(tb_ctx *ctx, void *cuda_stream);
TB_API void *tb_ctx_get_stream(tb_ctx *ctx);
/* 1 = launch kernels with programmatic dependent launch (default), 0 = plain. */
TB_API int tb_ctx_set_pdl(tb_ctx *ctx, int enable);
TB_API const char *tb_last_error(tb_ctx *ctx);
TB_API int tb_ctx_synchronize(tb_ctx *ctx);
/* Synchronise and read (and clear) the device error word that bounded waits set. */
TB_API int tb_ctx_device_error(tb_ctx *ctx, int *code);

/* ---- recorded batches (single-submit decode) ------------------------------
 * Replaces beginBatch / endBatch of engine/webgpu-engine.js:372-386, which the
 * forward uses to submit a whole decode step as ONE command buffer
 * (models/qwen3.js:3958).  Here the calls between tb_batch_begin and
 * tb_batch_end are recorded (CUDA stream capture into a graph) instead of
 * executed, and tb_batch_submit replays them with one launch.  Recording needs
 * the context's own stream (tb_ctx_set_stream(ctx, NULL)); the combined calls
 * that use context scratch must have run once beforehand at the same sizes. */
typedef struct tb_batch tb_batch;
TB_API int tb_batch_begin(tb_ctx *ctx);
TB_API int tb_batch_end(tb_ctx *ctx, tb_batch **out);
TB_API int tb_batch_submit(tb_ctx *ctx, tb_batch *batch);
TB_API int tb_batch_destroy(tb_batch *batch);
/* Stream-ordered copies between host memory and device buffers (pinned host
 * memory makes them asynchronous), queue.writeBuffer / mapAsync readback of
 * the reference (qwen3.js:4083). */
TB_API int tb_copy_h2d(tb_ctx *ctx, void *dst_dev, const void *src_host, size_t bytes);
TB_API int tb_copy_d2h(tb_ctx *ctx, void *dst_host, const void *src_dev, size_t bytes);

/* ---- int4 G=32 weight path ------------------------------------------------ */

/* Quant-on-arrival: bf16 [N,K] -> pack u32 [N,K/8] (k=8w+i at bits 4i, nibble
 * q+8), scales f16 bits [N,K/32].  Bit-exact with quantizeInt4Bf16,
 * models/qwen3.js:3405-3426 (JS double math, f32ToF16 :3357-3374).  K%32==0. */
TB_API int tb_quant_int4_g32(tb_ctx *ctx, const uint16_t *w_bf16, uint32_t *pack,
                             uint16_t *scales, int64_t N, int64_t K);

/* Per-32 int8 activation quantization of T rows: xq int8 [T,K], xs f32
 * [T,K/32], xsum16 i32 [T,K/16] (may be NULL).  QUANTQ8 qwen3.js:332-358 and
 * QUANTQ8T qwen3.js:1210-1231 (quantQ8 :414-420). */
TB_API int tb_quant_q8(tb_ctx *ctx, const float *x, int8_t *xq, float *xs, int32_t *xsum16,
                       int64_t T, int64_t K);

/* Fused RMSNorm -> per-32 int8: rmsnormQ, models/qwen3.js:569-621.  w16 = f16
 * norm weight [H].  Outputs as tb_quant_q8.  H%32==0. */
TB_API int tb_rmsnorm_q8(tb_ctx *ctx, const float *x, const uint16_t *w16, float eps,
                         int8_t *xq, float *xs, int32_t *xsum16, int64_t T, int64_t H);

/* int8-activation int4 GEMV for `batch` activation rows (1..8):
 * y[b,n] (+)= sum_g f32(s16[n,g])*xs[b,g] * sum_{k in g} (nib-8)*xq[b,k].
 * gemvDP4_only, models/qwen3.js:422-427 (GEMVDP4 :359-400).  acc=1 adds to y
 * (the fused residual).  K%32==0. */
TB_API int tb_gemv_int4_q8(tb_ctx *ctx, float *y, const int8_t *xq, const float *xs,
                           const uint32_t *pack, const uint16_t *scales,
                           int64_t N, int64_t K, int batch, int acc);

/* f32-activation int4 GEMV: y[b,n] (+)= sum_k x[b,k]*(nib-8)*f32(s16).
 * gemvQ, models/qwen3.js:314-321 (GEMVQ :276-311).  batch 1..8. */
TB_API int tb_gemv_int4_f32(tb_ctx *ctx, float *y, const float *x, const uint32_t *pack,
                            const uint16_t *scales, int64_t N, int64_t K, int batch, int acc);

/* The linearQ router for one int4 matrix, models/qwen3.js:1588-1608:
 * T==1 and N<16384 -> quantQ8 + gemvDP4; T==1 and N>=16384 -> gemvQ;
 * 2<=T<=16 with K%256==0 and N%8==0 -> QUANTQ8T into context scratch + the
 * gemmDP4A group-sum math on the tensor cores, one weight read (tb_gemv_int4_mma);
 * other 1<T<=8 -> per-token int8 (QUANTQ8T) x int4 math of gemmDP4A (:1397-1407);
 * T>16 -> QUANTQ8T into context scratch + gemmDP4A with exact group sums
 * (tb_gemm_dp4, the reference's default; its __noDp4Gemm f16 route is
 * tb_gemm_int4_g32) when T, N and K are multiples of 128, else
 * TB_ERR_UNSUPPORTED. */
TB_API int tb_linear_int4(tb_ctx *ctx, float *y, const float *x, const uint32_t *pack,
                          const uint16_t *scales, int64_t T, int64_t N, int64_t K, int acc);

/* Fused gate+up+SiLU on int8 activations: swi[b,i] = silu(g)*u,
 * gateUpSiluDP4_only, models/qwen3.js:861-877 (gateupDP4Wgsl :679-728).
 * gate/up are int4 [I,H]; batch 1..8. */
TB_API int tb_gateup_silu_int4_q8(tb_ctx *ctx, float *swi, const int8_t *xq, const float *xs,
                                  const uint32_t *gpack, const uint16_t *gscales,
                                  const uint32_t *upack, const uint16_t *uscales,
                                  int64_t I, int64_t H, int batch);

/* Several int4 matrices that read the SAME int8 activation, in one launch
 * (the q/k/v projGemv triple of forward(), models/qwen3.js:3981-3984).
 * ys/packs/scales/Ns are arrays of `count` (<= 4) entries. */
TB_API int tb_gemv_int4_q8_multi(tb_ctx *ctx, int count, float *const *ys,
                                 const uint32_t *const *packs, const uint16_t *const *scales,
                                 const int64_t *Ns, const int8_t *xq, const float *xs,
                                 int64_t K, int batch, int acc);

/* ---- fused activation-prep + GEMV (one launch each) ------------------------
 * The int8 activation is made inside the GEMV from the f32 rows x [batch,K]:
 * with norm_w16 == NULL it is QUANTQ8 of x, otherwise RMSNORMQ of x (eps),
 * bit-identical to tb_quant_q8 / tb_rmsnorm_q8 followed by the _q8 GEMV.
 *   tb_gemv_int4_dp4a        = gemvDP4A (models/qwen3.js:428-431), or
 *                              rmsnormQ + gemvDP4_only (forward, :3981-3984)
 *   tb_gemv_int4_dp4a_multi  = rmsnormQ + the q/k/v projGemv triple
 *   tb_gateup_silu_int4_dp4a = rmsnormQ + gateUpSiluDP4_only (:4023-4024)
 *   tb_gemv_int4_f32_norm    = rmsnorm + gemvQ for the lm_head (:4037-4049) */
TB_API int tb_gemv_int4_dp4a(tb_ctx *ctx, float *y, const float *x, const uint16_t *norm_w16, float eps,
                             const uint32_t *pack, const uint16_t *scales, int64_t N, int64_t K,
                             int batch, int acc);
TB_API int tb_gemv_int4_dp4a_multi(tb_ctx *ctx, int count, float *const *ys,
                                   const uint32_t *const *packs, const uint16_t *const *scales,
                                   const int64_t *Ns, const float *x, const uint16_t *norm_w16,
                                   float eps, int64_t K, int batch, int acc);
TB_API int tb_gateup_silu_int4_dp4a(tb_ctx *ctx, float *swi, const float *x, const uint16_t *norm_w16,
                                    float eps, const uint32_t *gpack, const uint16_t *gscales,
                                    const uint32_t *upack, const uint16_t *uscales,
                                    int64_t I, int64_t H, int batch);
TB_API int tb_gemv_int4_f32_norm(tb_ctx *ctx, float *y, const float *x, const uint16_t *norm_w16,
                                 float eps, const uint32_t *pack, const uint16_t *scales,
                                 int64_t N, int64_t K, int batch, int acc);

/* linearQ's T > 1 route, the DP4A GEMM math (models/qwen3.js:1600-1607,
 * gemmdp4Wgsl :1321-1407, gemmTern :1410-1420), at T = 2..16 rows with every
 * weight read once: QUANTQ8T of x (RMSNORMQ first when norm_w16 is non-null)
 * into context scratch, then per 32-group the exact int32 sum of int8 x times
 * (nib - 8) (or the ternary WebGPU code - 1) on the tensor cores, scaled by
 * xs * s in f32.  K % 256 == 0, N % 8 == 0; x, weights 16-byte aligned.
 *   tb_gemv_int4_mma / tb_gemv_tern_wgsl_mma: y [T,N] (+= with acc)
 *   tb_gemv_int4_mma_multi: the q/k/v triple (count <= 3) from one quantization
 *   tb_gateup_silu_*_mma: swi [T,I] = silu(W_g . a) * (W_u . a) (gateUpSiluDP4) */
TB_API int tb_gemv_int4_mma(tb_ctx *ctx, float *y, const float *x, const uint16_t *norm_w16, float eps,
                            const uint32_t *pack, const uint16_t *scales, int64_t N, int64_t K, int T,
                            int acc);
TB_API int tb_gemv_int4_mma_multi(tb_ctx *ctx, int count, float *const *ys, const uint32_t *const *packs,
                                  const uint16_t *const *scales, const int64_t *Ns, const float *x,
                                  const uint16_t *norm_w16, float eps, int64_t K, int T, int acc);
TB_API int tb_gateup_silu_int4_mma(tb_ctx *ctx, float *swi, const float *x, const uint16_t *norm_w16,
                                   float eps, const uint32_t *gpack, const uint16_t *gscales,
                                   const uint32_t *upack, const uint16_t *uscales, int64_t I, int64_t K,
                                   int T);
TB_API int tb_gemv_tern_wgsl_mma(tb_ctx *ctx, float *y, const float *x, const uint16_t *norm_w16, float eps,
                                 const uint32_t *pack, const uint16_t *scales, int64_t N, int64_t K, int T,
                                 int acc);
TB_API int tb_gateup_silu_tern_wgsl_mma(tb_ctx *ctx, float *swi, const float *x, const uint16_t *norm_w16,
                                        float eps, const uint32_t *gpack, const uint16_t *gscales,
                                        const uint32_t *upack, const uint16_t *uscales, int64_t I,
                                        int64_t K, int T);

/* ---- ternary Q2_0_g64 path (native/crates/n2-kernels) -------------------- */

/* f32 ternary [N,K] -> codes u8 [N,K/4] + f32 scales [N,K/64], bit-exact with
 * pack_ternary, native/crates/n2-kernels/src/tern.rs:131-160 and
 * native/tools/pack_bin.py:19-29.  K%64==0. */
TB_API int tb_pack_tern_q2g64(tb_ctx *ctx, const float *w, uint8_t *codes, float *scales,
                              int64_t N, int64_t K);

/* Per-vector activation quantization of T rows: act i8 [T,K], xsum i32
 * [T,K/64], scale f32 [T] (=127/amax, 1 when amax==0).  quantize_act_into,
 * tern.rs:206-222.  K%64==0. */
TB_API int tb_quant_act_q8(tb_ctx *ctx, const float *x, int8_t *act, int32_t *xsum,
                           float *scale, int64_t T, int64_t K);

/* The browser CPU engine's activation quantizer, in its argument order: the
 * WASM export quantize(dst, xsum, x, k) -> asc, cpu/kernel/src/lib.rs:566-606,
 * which JS workers call before gemv_tern / gemm_tern_b4
 * (cpu/cpukern-fwd-worker.js:326-357).  Per row of `rows`: asc = amax/127
 * (1e-9 when amax == 0), dst = nearest-even(x * (1/asc)) clamped to +-127,
 * xsum i32 per 64; asc f32 [rows] receives what the export returns (the
 * factor the GEMV output is multiplied by).  Bit-exact.  k%64==0. */
TB_API int tb_quantize_wasm(tb_ctx *ctx, int8_t *dst, int32_t *xsum, const float *x, int64_t k,
                            float *asc, int64_t rows);

/* Ternary GEMV for `batch` activation rows (1..8): out[b,n] =
 * sum_blk s*dot - sum_blk s*xsum, accumulated in block order exactly as
 * gemv_tern_scalar, tern.rs:79-119 (bit-exact).  Replaces tern::gemv_tern
 * (tern.rs:56-71), the WASM export gemv_tern (cpu/kernel/src/lib.rs:436-441)
 * and gemm_tern_b4 (lib.rs:331). */
TB_API int tb_gemv_tern_q2g64(tb_ctx *ctx, float *out, const uint8_t *codes, const float *scales,
                              const int8_t *act, const int32_t *xsum, int64_t N, int64_t K, int batch);

/* Model::linear, native/crates/n2-core/src/model.rs:316-339: quantize_act ->
 * gemv_tern -> out *= 1/scale, for T (1..8) rows.  Context-owned scratch. */
TB_API int tb_linear_tern(tb_ctx *ctx, float *y, const float *x, const uint8_t *codes,
                          const float *scales, int64_t T, int64_t N, int64_t K);

/* ---- ternary, WebGPU layout (models/qwen3.js) ------------------------------
 * The layout of the reference's browser engine for Bonsai/BitNet-style weights:
 * pack u32 [N][K/16], 16 codes w+1 in {0,1,2} per word, weight k = 16w+4s+b at
 * bits 8b+2s of word w; f16 scales [N][K/32] (the int4 scale layout).  The
 * GEMVs take the per-32 int8 activation of tb_quant_q8 (QUANTQ8) and compute,
 * per 32-group, f32(scale) * xs * sum((c-1) * xq) with an exact int32 sum. */

/* Lossless ternary detection + pack, quantizeTernaryBf16 (qwen3.js:3435-3469):
 * bf16 [N,K] -> pack + scales as above.  *nonternary (a DEVICE int) is set to
 * nonzero when the matrix is not ternary (some nonzero magnitude more than 2
 * bf16 ulps below its 32-group's maximum, or K % 64 != 0) -- the reference's
 * null return, after which the caller quantizes to int4 instead. */
TB_API int tb_quant_tern_wgsl_bf16(tb_ctx *ctx, const uint16_t *w_bf16, uint32_t *pack,
                                   uint16_t *scales, int64_t N, int64_t K, int *nonternary);

/* gemvTern_only (qwen3.js:548-556; shader gemvTern2Wgsl :449-503) against a
 * pre-quantized QUANTQ8 activation of `batch` rows (1..8); y [batch][N]
 * (+= y when acc).  K % 64 == 0; pack, scales, xq 16-byte aligned. */
TB_API int tb_gemv_tern_wgsl_q8(tb_ctx *ctx, float *y, const int8_t *xq, const float *xs,
                                const uint32_t *pack, const uint16_t *scales, int64_t N, int64_t K,
                                int batch, int acc);

/* quantQ8 (or the fused RMSNorm of RMSNORMQ when norm_w16 != NULL) followed by
 * gemvTern_only for 1..4 matrices sharing the activation (projGemv at the
 * q/k/v call sites, qwen3.js:558-561, 3982-3984), in one launch. */
TB_API int tb_gemv_tern_wgsl_dp4a_multi(tb_ctx *ctx, int count, float *const *ys,
                                        const uint32_t *const *packs, const uint16_t *const *scales,
                                        const int64_t *Ns, const float *x, const uint16_t *norm_w16,
                                        float eps, int64_t K, int batch, int acc);

/* Fused ternary gate+up+SiLU, gateupTern2Wgsl (qwen3.js:747-810) as routed by
 * gateUpSiluDP4_only / gateUpSiluQ (:730, :861-870): swi [batch][I] =
 * silu(g) * u.  _q8 takes the QUANTQ8 activation, _dp4a the f32 row (and the
 * optional RMSNorm weight). */
TB_API int tb_gateup_silu_tern_wgsl_q8(tb_ctx *ctx, float *swi, const int8_t *xq, const float *xs,
                                       const uint32_t *gpack, const uint16_t *gscales,
                                       const uint32_t *upack, const uint16_t *uscales,
                                       int64_t I, int64_t H, int batch);
TB_API int tb_gateup_silu_tern_wgsl_dp4a(tb_ctx *ctx, float *swi, const float *x,
                                         const uint16_t *norm_w16, float eps,
                                         const uint32_t *gpack, const uint16_t *gscales,
                                         const uint32_t *upack, const uint16_t *uscales,
                                         int64_t I, int64_t H, int batch);

/* Prefill GEMM of ternary weights (gemmTern, qwen3.js:1410-1420) on tcgen05:
 * y[M,N] (+)= f16(xs * xq) . f16((c-1) * s)^T with f32 accumulation, from the
 * QUANTQ8T rows xq int8 [M,K] / xs f32 [M,K/32].  M % 128 == 0, N % 256 == 0,
 * K % 64 == 0; xq, pack, y 16-byte aligned, xs and scales 4-byte aligned. */
TB_API int tb_gemm_tern_wgsl(tb_ctx *ctx, float *y, const int8_t *xq, const float *xs,
                             const uint32_t *pack, const uint16_t *scales, int64_t M, int64_t N,
                             int64_t K, int acc);

/* linearQ for a ternary weight record (qwen3.js:1594-1598): 2 <= T <= 16 rows
 * with K % 256 == 0 and N % 8 == 0 run the tensor-core GEMV (tb_gemv_tern_wgsl_mma),
 * other T <= 8 the ternary GEMV (quantQ8 fused), T > 16 quantize (QUANTQ8T) into
 * context scratch and run tb_gemm_tern_wgsl (T % 128 == 0, N % 256 == 0). */
TB_API int tb_linear_tern_wgsl(tb_ctx *ctx, float *y, const float *x, const uint32_t *pack,
                               const uint16_t *scales, int64_t T, int64_t N, int64_t K, int acc);

/* int8-KV prefill attention: attentionQ8 with T > 1 (qwen3.js:2534-2577; the
 * flash kernels ATTN_WGSL / attnF16Wgsl with dequantizing tile loads).  Query i
 * of T (q f32 [T][nHq*hd], after q_norm + RoPE) sits at position S - T + i and
 * attends causally to keys 0 .. S - T + i of the int8 cache (layout of
 * tb_attn_prep_q8: Kq/Vq int8 [S][nKv*hd], Ks/Vs f32 [S][nKv*hd/32]); out f32
 * [T][nHq*hd].  1 <= T <= S, hd 64 or 128, nHq/nKv in {1,2,4,8}.  Tensor-core
 * math with f16 operands and f32 sums (within ~1e-3 of the exact result). */
TB_API int tb_attn_prefill_q8(tb_ctx *ctx, float *out, const float *q, const int8_t *Kq,
                              const float *Ks, const int8_t *Vq, const float *Vs, int64_t T,
                              int64_t S, int64_t nHq, int64_t nKv, int64_t hd);

/* ---- sampling transforms before argmax (qwen3.js:2692-2737) ------------------
 * logits are `rows` rows of n.  The mask is one bit per token, rows of
 * ceil(n/32) u32 words (bit i%32 of word i/32); the Gumbel noise of element
 * (row, i) is that of the flat index row*n + i. */
/* LOGITMASK_WGSL: every token whose bit is clear gets -3e38 (grammar-constrained decoding). */
TB_API int tb_logit_mask(tb_ctx *ctx, float *logits, const uint32_t *mask, int64_t n, int64_t rows);
/* GUMBEL_WGSL: logits += temp * -log(-log(u)), u = (pcg(i ^ seed*2654435761) >> 8 + 0.5) / 2^24,
 * so argmax afterwards is an exact sample of softmax(logits / temp).  The host
 * advances the seed per step (gumbelNoise: seed = seed*1664525 + 1013904223). */
TB_API int tb_gumbel_noise(tb_ctx *ctx, float *logits, int64_t n, int64_t rows, uint32_t seed, float temp);
/* mask (optional) + Gumbel noise (temp > 0) + argmax in one pass, logits left
 * unmodified: the same ids as tb_logit_mask, tb_gumbel_noise and tb_argmax in
 * sequence.  temp == 0 and mask == NULL is greedy argmax. */
TB_API int tb_sample_argmax(tb_ctx *ctx, const float *logits, int64_t n, int64_t rows, const uint32_t *mask,
                            uint32_t seed, float temp, uint32_t *out_idx);

/* ---- `.cpu.bin` ternary model container (native/docs/FORMAT.md) ----------
 * The native Bonsai engine's on-disk format: u32 le header length, a JSON header
 * {"G": 64, "tensors": {...}}, then a blob of 16-byte-aligned entries: `tern`
 * (Q2_0_g64 codes u8 [N][K/4] + f32 scales [N][K/64], ready for
 * tb_gemv_tern_q2g64), `embed_f16` (f16 bits) and `f32` (norm weights). */
typedef struct tb_bin tb_bin;
enum { TB_BIN_TERN = 0, TB_BIN_EMBED_F16 = 1, TB_BIN_F32 = 2 };
typedef struct {
    const char *name;       /* valid while the container is open */
    int kind;               /* TB_BIN_* */
    int64_t N, K;           /* tern: rows, columns */
    int ndim;
    int64_t shape[4];
    const void *data;       /* device: codes (tern) or the tensor's bytes */
    int64_t bytes;
    const void *scales;     /* device: f32 scales (tern), else NULL */
    int64_t scales_bytes;
    int64_t blob_offset;    /* data's offset in the blob */
} tb_bin_tensor;

/* Validate a container's header exactly as the reference reader does
 * (Container::open / assemble / validate, native/crates/n2-core/src/binfmt.rs:
 * 104-257) without touching a GPU: G == 64 (absent means 64), known kinds,
 * K % G == 0, codesLen == N*K/4, scalesLen == N*(K/G)*4, every range inside the
 * blob.  TB_OK, or TB_ERR_INVALID with the reason in err (the reference's wording). */
TB_API int tb_bin_check(const char *path, char *err, size_t err_len);

/* Container::open onto the device: validates as tb_bin_check, then streams the
 * whole blob into one device allocation (pinned double-buffered copies on the
 * context's stream); returns when the blob is resident.  Tensors are pointers
 * into it, in the reference's layout. */
TB_API int tb_bin_open(tb_ctx *ctx, const char *path, tb_bin **out);
TB_API int tb_bin_close(tb_bin *bin);
TB_API int64_t tb_bin_blob_bytes(const tb_bin *bin);
/* tensors in name order (the reference's BTreeMap order) */
TB_API int tb_bin_count(const tb_bin *bin);
TB_API int tb_bin_info(const tb_bin *bin, int index, tb_bin_tensor *info);
/* by name (Container::get / ternary / f32s, binfmt.rs:267-321) */
TB_API int tb_bin_find(const tb_bin *bin, const char *name, tb_bin_tensor *info);

/* ---- int8 KV cache + split-KV GQA decode attention ----------------------- */

/* Fused decode attention prep at position `pos` (T=1):
 * q heads: per-head RMSNorm(qw16) + RoPE -> qr f32 [nHq*hd];
 * k heads: RMSNorm(kw16) + RoPE -> snorm int8 per-32 into Kq/Ks at row pos;
 * v heads: raw -> snorm int8 per-32 into Vq/Vs at row pos.
 * attnPrepQ8, models/qwen3.js:2297-2308 (attnPrepWgsl :2228-2296).
 * KV layout: Kq/Vq int8 [S_max][nKv*hd], Ks/Vs f32 [S_max][nKv*hd/32].
 * hd%32==0, hd<=256. */
TB_API int tb_attn_prep_q8(tb_ctx *ctx, const float *q, const float *k, const float *v,
                           const uint16_t *qw16, const uint16_t *kw16, float *qr,
                           int8_t *Kq, float *Ks, int8_t *Vq, float *Vs,
                           int64_t nHq, int64_t nKv, int64_t hd, int64_t pos,
                           float theta, float eps);

/* K/V-only quantize-write of T rows at posBase (prefill): KVQW,
 * models/qwen3.js:2180-2216.  kr/v f32 [T][nKv*hd]. */
TB_API int tb_kv_quant_write(tb_ctx *ctx, const float *kr, const float *v,
                             int8_t *Kq, float *Ks, int8_t *Vq, float *Vs,
                             int64_t T, int64_t nKv, int64_t hd, int64_t posBase);

/* Split-KV streaming decode attention over S cached positions:
 * attnDecodeStreamQ8 + combine, models/qwen3.js:2165-2173 (kernels :2077-2164,
 * :2048-2069).  nsplit = 0 picks the reference rule _decNsplit (:2354) scaled
 * to fill the GPU.  out f32 [nHq*hd].  Context-owned scratch for partials. */
TB_API int tb_attn_decode_q8(tb_ctx *ctx, float *out, const float *qr,
                             const int8_t *Kq, const float *Ks, const int8_t *Vq, const float *Vs,
                             int64_t S, int64_t nHq, int64_t nKv, int64_t hd, int nsplit);

/* Allocation-free form of tb_attn_decode_q8, for callers that cannot let the
 * library call cudaMalloc (a process that gives its whole device budget to its
 * own pool at start-up, or a loop that must not let an allocation synchronize
 * the device mid-step).  No counterpart in the reference.  The split partials
 * live in a fixed 1 MiB device array inside the library instead of context
 * scratch: an explicit nsplit with nHq*nsplit*(hd+2) > 262144 floats is
 * rejected with TB_ERR_INVALID; nsplit = 0 picks the automatic split count
 * capped at what fits.  The first call on a device looks up the array's address
 * (make it before any stream capture); calls share the array, so calls that
 * overlap on the GPU race and must be ordered by the caller. */
TB_API int tb_attn_decode_q8_noalloc(tb_ctx *ctx, float *out, const float *qr,
                                     const int8_t *Kq, const float *Ks, const int8_t *Vq,
                                     const float *Vs, int64_t S, int64_t nHq, int64_t nKv,
                                     int64_t hd, int nsplit);

/* Batched, graph-replayable forms (the decode step records them once and
 * replays them every token).  `batch` sequences; sequence b's cache holds
 * cache_rows rows and starts cache_rows rows after sequence b-1's; q/k/v/qr/out
 * rows are [batch][heads*hd].  Positions live on the device: dpos[b] is the row
 * written by the prep and the context is S_b = dpos[b] + 1 rows.  A position
 * outside [0, cache_rows) sets the context's device error word
 * (tb_ctx_device_error) and leaves that sequence's cache and output row
 * unwritten / zero.  S_max (<= cache_rows) fixes the split count (nsplit = 0:
 * automatic).  Same math as tb_attn_prep_q8 / tb_attn_decode_q8. */
TB_API int tb_attn_prep_q8_batch(tb_ctx *ctx, const float *q, const float *k, const float *v,
                                 const uint16_t *qw16, const uint16_t *kw16, float *qr,
                                 int8_t *Kq, float *Ks, int8_t *Vq, float *Vs,
                                 int64_t nHq, int64_t nKv, int64_t hd, int64_t batch,
                                 int64_t cache_rows, const int32_t *dpos, float theta, float eps);
TB_API int tb_attn_decode_q8_batch(tb_ctx *ctx, float *out, const float *qr,
                                   const int8_t *Kq, const float *Ks, const int8_t *Vq,
                                   const float *Vs, int64_t batch, int64_t cache_rows,
                                   const int32_t *dpos, int64_t S_max, int64_t nHq, int64_t nKv,
                                   int64_t hd, int nsplit);

/* ---- decode-step glue ------------------------------------------------------ */

/* Argmax over `rows` rows of n logits -> out_idx[row*stride + offset]
 * (u32).  argmaxKernel, models/qwen3.js:2681-2690 (one and two-stage).
 * Lowest index wins on ties. */
TB_API int tb_argmax(tb_ctx *ctx, const float *x, int64_t n, int64_t rows, uint32_t *out_idx,
                     int64_t out_offset);

/* y[T,H] = x * rsqrt(mean(x^2)+eps) * f16 w.  rmsnorm, qwen3.js:81-88. */
TB_API int tb_rmsnorm(tb_ctx *ctx, const float *x, const uint16_t *w16, float *y,
                      int64_t T, int64_t H, float eps);

/* y[t,:] = f32(embed_f16[ids[idoff+t], :]).  embedGather, qwen3.js:1663-1675. */
TB_API int tb_embed_gather(tb_ctx *ctx, const uint32_t *ids, int64_t idoff,
                           const uint16_t *embed_f16, float *y, int64_t T, int64_t H);

/* ---- prefill GEMM (tcgen05 / TMEM) -------------------------------------------
 * Y[M,N] (+)= f16(X[M,K]) . f16(deq(W[N,K]))^T with f32 accumulation: the
 * reference's f16 prefill GEMM gemmQ (models/qwen3.js:964-1026, gemmqWgsl), the
 * weights in the int4 G=32 layout of tb_quant_int4_g32.  X is f32 (x_bf16 = 0,
 * as linearQ's buffers) or bf16 (x_bf16 = 1).  M % 128 == 0, N % 256 == 0,
 * K % 64 == 0; x, pack, y 16-byte aligned, scales 4-byte aligned.  X is rounded
 * to f16 into context scratch first (M rounded up to 256, x K, x 2 bytes), as are
 * the inputs of tb_gemm_int4_q8 and tb_gemm_tern_wgsl; when the output tiles leave
 * SMs idle the K range is split and the splits' f32 partials (up to 8 x M x N x 4
 * bytes) also live in that scratch, which grows on demand. */
TB_API int tb_gemm_int4_g32(tb_ctx *ctx, float *y, const void *x, int x_bf16, const uint32_t *pack,
                            const uint16_t *scales, int64_t M, int64_t N, int64_t K, int acc);

/* The reference's integer prefill GEMMs, gemmDP4A (int4) and gemmTern (ternary
 * WebGPU layout), qwen3.js:1321-1420, with their exact arithmetic: per 32-group
 * the int8 activation (QUANTQ8T xq int8 [M][K], xs f32 [M][K/32]) times the int8
 * weight (nib - 8 or code - 1) summed exactly in int32 on the tensor cores
 * (tcgen05.mma kind::i8, one MMA a group into TMEM), then
 * y (epilogue)= sum_g (f32(s) * xs) * sum in f32, groups in k order.  tern selects
 * the weight layout.  epilogue: 0 y =, 1 y +=, 2 y = silu(y) * (fused swiglu).
 * M, N, K % 128 == 0; xq, xs, pack, y 16-byte, scales 8-byte aligned. */
TB_API int tb_gemm_dp4(tb_ctx *ctx, float *y, const int8_t *xq, const float *xs, const uint32_t *pack,
                       const uint16_t *scales, int64_t M, int64_t N, int64_t K, int epilogue, int tern);

/* The same GEMM on the warp-level MMA (mma.sync m16n8k32 .s8), the same values in
 * the same order (outputs bit-equal to tb_gemm_dp4): a second implementation for
 * cross-checks and comparison.  Same arguments and rules, y 8-byte aligned. */
TB_API int tb_gemm_dp4_warp(tb_ctx *ctx, float *y, const int8_t *xq, const float *xs, const uint32_t *pack,
                            const uint16_t *scales, int64_t M, int64_t N, int64_t K, int epilogue, int tern);

/* gemmDP4A's data flow on tcgen05 with f16 operands (a faster, rounded form of
 * tb_gemm_dp4 -- linearQ routes to the exact one, qwen3.js:1605-1607): X as QUANTQ8T rows xq int8 [M][K] + xs f32 [M][K/32]
 * (tb_quant_q8), W int4 G32; y = f16(xs*q) . f16((nib-8)*s)^T summed in f32
 * (the reference sums each group's int8 products exactly; the f16 rounding of
 * xs*q is the only difference, ~2^-11).  epilogue: 0 y =, 1 y +=, 2 y =
 * silu(y) * (the forward's swiglu fused: y holds the gate projection).
 * M % 128, N % 256, K % 64 == 0. */
TB_API int tb_gemm_int4_q8(tb_ctx *ctx, float *y, const int8_t *xq, const float *xs, const uint32_t *pack,
                           const uint16_t *scales, int64_t M, int64_t N, int64_t K, int epilogue);

/* ---- int3 mixture of experts (LFM2.5, models/lfm25.js) ---------------------
 * int3 layout as the reference: per (row, 32-group) three u32 bitplanes of the
 * stored value q3 + 4 (bit i of plane p = bit p of weight i) and an f16 scale;
 * expert e's rows are e*N .. e*N+N-1. */
/* _requant43 (lfm25.js:833-855): int4 G32 pack/scales -> p3 u32 [rows][K/32][3],
 * s3 f16 [rows][K/32]; bit-exact with the reference (JS doubles, the engine's
 * f32ToF16). */
TB_API int tb_requant_int4_int3(tb_ctx *ctx, uint32_t *p3, uint16_t *s3, const uint32_t *pack4,
                                const uint16_t *s4, int64_t rows, int64_t K);
/* ROUTER_WGSL (lfm25.js:111-141): idx u32 [T][K], wt f32 [T][K] from logits
 * f32 [T][nE] and expert_bias f32 [nE] (nE <= 64). */
TB_API int tb_moe_router(tb_ctx *ctx, uint32_t *idx, float *wt, const float *logits, const float *bias,
                         int64_t T, int64_t nE, int64_t K);
/* The MoE FFN of T tokens (idxGemv3 w1, w3, SiLU, idxGemv3 w2, MOECOMBINE):
 * x_out[t] += sum_k wt[t,k] * W2_e(silu(W1_e x_in[t]) * W3_e x_in[t]), e = idx[t,k].
 * w1/w3 planes [nE*I][H/32][3] + scales, w2 [nE*H][I/32][3] + scales.  The
 * (token, expert) pairs are grouped by expert so each expert's weights are
 * decoded once per chunk of its pairs.  Context-owned scratch. */
TB_API int tb_moe_ffn_int3(tb_ctx *ctx, float *x_out, const float *x_in, const uint32_t *idx, const float *wt,
                           const uint32_t *w1p, const uint16_t *w1s, const uint32_t *w3p, const uint16_t *w3s,
                           const uint32_t *w2p, const uint16_t *w2s, int64_t T, int64_t K, int64_t nE,
                           int64_t H, int64_t I);
/* The same FFN with one f16 scale per `group` weights (32: the reference's
 * _requant43 layout, tb_moe_ffn_int3; 128: the group-128 int3 of the LFM2.5
 * benchmark configuration): planes stay three u32 per 32 weights, scales are
 * [rows][K/group].  H and I multiples of group. */
TB_API int tb_moe_ffn_int3_g(tb_ctx *ctx, float *x_out, const float *x_in, const uint32_t *idx, const float *wt,
                             const uint32_t *w1p, const uint16_t *w1s, const uint32_t *w3p, const uint16_t *w3s,
                             const uint32_t *w2p, const uint16_t *w2s, int64_t T, int64_t K, int64_t nE,
                             int64_t H, int64_t I, int group);
/* bf16 [rows][K] -> int3 planes [rows][K/32][3] (stored q + 4) + f16 scales
 * [rows][K/group], group 32 or 128: scale = f16(max|w| / 4) (the engine's
 * f32ToF16 of _requant43, lfm25.js:833-855), q = clamp(rn(w / scale), -4, 3).
 * No reference counterpart: the reference reaches int3 only from int4 at
 * group 32 (tb_requant_int4_int3); the benchmark's LFM2.5 configuration names
 * group-128 int3 from bf16 weights. */
TB_API int tb_quant_int3_bf16(tb_ctx *ctx, const uint16_t *w_bf16, uint32_t *p3, uint16_t *s3, int64_t rows,
                              int64_t K, int group);

/* Expert parallelism (no reference counterpart: the reference keeps every
 * expert on one device, lfm25.js:824-830): the MoE FFN of tb_moe_ffn_int3 over
 * P ranks (one process and GPU each), experts [r*nE/P, (r+1)*nE/P) on rank r.
 * Each rank routes its own tokens; a forward sends every token row once to each
 * rank that owns one of its experts (stores into that rank's IPC-mapped arena
 * over NVLink), the owner runs the grouped int3 GEMVs on what it received and
 * writes each (token, expert) output straight back into the origin's arena, and
 * the origin combines in top-k order: the result is bit-identical to
 * tb_moe_ffn_int3 on one device with all experts.  Every rank calls
 * tb_moe_ep_forward the same number of times (T may differ per rank); waits
 * for peers are bounded (about a second) and record a device error.
 * Lifecycle: create (every rank) -> handle -> exchange the P handles (any
 * host channel) -> connect (P > 1) -> set_experts -> forward ... -> destroy. */
typedef struct tb_moe_ep tb_moe_ep;
/* nE % P == 0, nE/P <= 256, K <= 8, H and I multiples of 32 up to 2048, up to
 * Tmax <= 1024 tokens per rank and call.  Allocates the arena and buffers. */
TB_API int tb_moe_ep_create(tb_ctx *ctx, int P, int rank, int64_t nE, int64_t K, int64_t H, int64_t I,
                            int64_t Tmax, tb_moe_ep **out);
TB_API void tb_moe_ep_destroy(tb_moe_ep *m);
/* 64-byte CUDA IPC handle of this rank's arena */
TB_API int tb_moe_ep_handle(tb_moe_ep *m, void *out64);
/* handles: P x 64 bytes, rank order */
TB_API int tb_moe_ep_connect(tb_moe_ep *m, const void *handles);
/* this rank's experts, layout as tb_moe_ffn_int3 with nE/P experts (referenced,
 * not copied: keep them alive) */
TB_API int tb_moe_ep_set_experts(tb_moe_ep *m, const uint32_t *w1p, const uint16_t *w1s, const uint32_t *w3p,
                                 const uint16_t *w3s, const uint32_t *w2p, const uint16_t *w2s);
/* x_out [T][H] += MoE FFN of x_in [T][H] routed by idx/wt [T][K] (global
 * expert ids, as tb_moe_router); x rows 16-byte aligned. */
TB_API int tb_moe_ep_forward(tb_moe_ep *m, float *x_out, const float *x_in, const uint32_t *idx, const float *wt,
                             int64_t T);

/* bf16 -> f16 bits, rounded half-up as the loader's bf16ToF16bits
 * (models/qwen3.js:3357-3390): the f16 copies of the embedding table and the
 * norm weights. */
TB_API int tb_convert_bf16_f16(tb_ctx *ctx, const uint16_t *in_bf16, uint16_t *out_f16, int64_t n);

/* ---- Qwen3 decode step (models/qwen3.js forward, :3938-4069) ---------------
 * A model object owns its weights (quantized on arrival), its int8 KV cache,
 * its activations and the recorded step.  One step decodes one token for each
 * of `batch` sequences: ids[b] (device, u32) is read by the embedding gather
 * and overwritten with the argmax token; pos[b] (device, i32) is the cache row
 * written this step and is advanced by one, so consecutive steps need no host
 * work (the reference's GPU token history, :4055-4060).  The first
 * tb_qwen3_decode_step records the step as a CUDA graph; later calls replay it
 * on the context's stream.  At batch 1 on one GPU the step is, by default, one
 * persistent kernel for embed and all layers plus the lm_head and argmax
 * (tb_qwen3_set_step_mode); elsewhere one kernel per operation.
 *
 * Tensor parallelism (tp_size > 1, one context and process per GPU): each
 * rank keeps q/k/v and gate/up row blocks, o and down column blocks, its
 * n_kv_heads/tp_size kv heads (with their q heads) and vocab/tp_size lm_head
 * rows; partial o and down products are summed by an NCCL allreduce of the
 * batch x hidden residual, and the argmax by an allgather of per-rank keys.
 * Every rank passes the FULL bf16 tensors to tb_qwen3_set_weight and keeps its
 * own slice (tb_qwen3_shard tells which). */
typedef struct tb_qwen3_config {
  int32_t hidden, layers, n_heads, n_kv_heads, head_dim, intermediate, vocab;
  float rope_theta, rms_eps;
  int32_t max_seq;   /* KV cache rows per sequence */
  int32_t batch;     /* sequences per step, 1..16 */
  int32_t tp_size;   /* ranks sharing the model (1 = single GPU) */
  int32_t tp_rank;
  int32_t ternary;   /* 1: tb_qwen3_set_weight tries the lossless ternary (WebGPU layout)
                        record before int4, as the reference loader does
                        (qwen3.js:3508-3523); 0: int4 only (its __noTernary) */
} tb_qwen3_config;

typedef struct tb_qwen3 tb_qwen3;

/* weight kinds (checkpoint names as in the reference's _weights map) */
enum {
  TB_QW_EMBED = 0,       /* model.embed_tokens.weight   [vocab][hidden] -> f16 */
  TB_QW_LM_HEAD = 1,     /* lm_head.weight              [vocab][hidden] -> int4 */
  TB_QW_FINAL_NORM = 2,  /* model.norm.weight           [hidden]        -> f16 */
  TB_QW_Q = 3,           /* layers.l.self_attn.q_proj   [n_heads*hd][hidden] */
  TB_QW_K = 4,           /* k_proj [n_kv*hd][hidden] */
  TB_QW_V = 5,           /* v_proj [n_kv*hd][hidden] */
  TB_QW_O = 6,           /* o_proj [hidden][n_heads*hd] */
  TB_QW_GATE = 7,        /* mlp.gate_proj [inter][hidden] */
  TB_QW_UP = 8,          /* mlp.up_proj   [inter][hidden] */
  TB_QW_DOWN = 9,        /* mlp.down_proj [hidden][inter] */
  TB_QW_LN_ATTN = 10,    /* input_layernorm [hidden] */
  TB_QW_LN_MLP = 11,     /* post_attention_layernorm [hidden] */
  TB_QW_Q_NORM = 12,     /* self_attn.q_norm [hd] */
  TB_QW_K_NORM = 13      /* self_attn.k_norm [hd] */
};

/* How the decode step runs.  TB_QW_STEP_PERSISTENT: embed and every layer in
 * ONE persistent kernel (one CTA per SM, grid barriers between the phases, each
 * CTA requesting the weights of its next phases into shared memory while the
 * current one runs), then lm_head and argmax; batch 1, layer weights all int4
 * or all ternary, one GPU or tensor parallel over peer memory (tp_connect: the
 * o / down rows are exchanged inside the kernel, CTA by CTA, over NVLink).
 * TB_QW_STEP_KERNELS: one kernel per operation (6 per layer + 4).
 * TB_QW_STEP_AUTO (default): persistent wherever it applies (one GPU, or
 * tensor parallel over the peer-memory exchange of tb_qwen3_tp_connect), else
 * the multi-kernel step.  Both compute the same bits.  No reference counterpart (the reference dispatches WebGPU passes). */
#define TB_QW_STEP_AUTO 0
#define TB_QW_STEP_KERNELS 1
#define TB_QW_STEP_PERSISTENT 2
TB_API int tb_qwen3_set_step_mode(tb_qwen3 *m, int mode);
/* the kind the recorded step uses (TB_QW_STEP_KERNELS / _PERSISTENT), 0 before the first step */
TB_API int tb_qwen3_step_kind(tb_qwen3 *m);
/* Launch the persistent kernel alone (embed + every layer; no lm_head, no
 * argmax, ids and pos unchanged) on the context's stream, to time it apart.
 * Needs a recorded persistent step. */
TB_API int tb_qwen3_step_layers(tb_qwen3 *m);
/* Profiling: %globaltimer stamps of the persistent kernel into trace (device,
 * u64 [SM count][1 + 38 * layers]; null turns it off): per CTA the kernel start,
 * then per layer and phase (q/k/v, attention, o, gate/up, down) the moments its
 * weights were ready, its activation row arrived, its activation was staged, it
 * finished, and its grid barrier opened; then per layer 8 stamps of the CTA's
 * first attention unit (start, q prep, k/v prep, tiles done, partial written,
 * arrival counted, end, whether it combined), then per layer and phase the
 * moment its request for the next weights was issued. */
TB_API int tb_qwen3_step_trace(tb_qwen3 *m, void *trace);
/* Host-only: the block of a full [rows][cols] tensor of `kind` that rank
 * cfg->tp_rank keeps (norm vectors count as one row). */
TB_API int tb_qwen3_shard(const tb_qwen3_config *cfg, int kind, int64_t *row0, int64_t *nrows,
                          int64_t *col0, int64_t *ncols);
TB_API int tb_qwen3_create(tb_ctx *ctx, const tb_qwen3_config *cfg, tb_qwen3 **out);
TB_API int tb_qwen3_destroy(tb_qwen3 *m);
/* Full bf16 tensor [rows][cols] on the device (16-byte aligned); quantized /
 * converted into the model's shard, ordered on the context's stream. */
TB_API int tb_qwen3_set_weight(tb_qwen3 *m, int kind, int layer, const uint16_t *bf16,
                               int64_t rows, int64_t cols);
/* Formats of an already-quantized tensor (the quant cache's segment kinds,
 * qwen3.js:3671-3717): int4 G32 pack + f16 scales, ternary WebGPU-layout pack +
 * f16 scales, or the f16 buffer of a non-projection tensor. */
enum { TB_QW_FMT_INT4 = 0, TB_QW_FMT_TERN = 1, TB_QW_FMT_F16 = 2 };
/* Set a weight from its FULL [rows][cols] tensor already in `fmt` (host or
 * device memory): `data` = pack (or the f16 buffer), `scales` = f16 scales
 * (NULL for TB_QW_FMT_F16).  The rank's shard is copied out (32-aligned column
 * slices for int4, 64-aligned for ternary).  What loadQuantCache does with
 * each cached segment; synchronous for pageable host memory. */
TB_API int tb_qwen3_set_weight_q(tb_qwen3 *m, int kind, int layer, int fmt, const void *data,
                                 const void *scales, int64_t rows, int64_t cols);
/* forward(ids, posBase) at T > 1 -- prefill -- for sequence `seq` (qwen3.js:
 * 3938-4069): T token ids (host) at positions pos0 .. pos0+T-1 run through every
 * layer as GEMMs (QUANTQ8T + tb_gemm_dp4: gemmDP4A / gemmTern with exact group
 * sums, residual and SwiGLU fused into their epilogues), the rows' K/V are written to the
 * sequence's cache and the int8-KV prefill attention runs over it; the last
 * row's lm_head + argmax sets ids[seq] and pos[seq] = pos0 + T, so the next
 * tb_qwen3_decode_step continues the sequence.  Returns when done.  Under
 * tensor parallelism (NCCL exchange, tb_qwen3_tp_init) every rank calls it with
 * the same ids: column-split q/k/v/gate/up, row-split o/down with an allreduce
 * of the T rows after each, local heads against the local cache shard, the
 * vocab-split lm_head's argmax merged across ranks.  The rank's sizes
 * (hidden, heads*head_dim, kv_heads*head_dim, intermediate) multiples of 128.
 * Buffers grow on the first call for a larger T (allocation). */
TB_API int tb_qwen3_prefill(tb_qwen3 *m, int seq, const uint32_t *ids, int64_t T, int64_t pos0);
/* The format tb_qwen3_set_weight chose for a weight (TB_QW_FMT_*), or -1 if unset. */
TB_API int tb_qwen3_weight_format(const tb_qwen3 *m, int kind, int layer);
/* This rank's cache of a layer: int8 [batch][max_seq][n_kv/tp*hd] and f32
 * scales [batch][max_seq][n_kv/tp*hd/32] (fill prefixes with tb_kv_quant_write). */
TB_API int tb_qwen3_kv(tb_qwen3 *m, int layer, int8_t **Kq, float **Ks, int8_t **Vq, float **Vs);
/* Device buffers: ids u32 [batch], pos i32 [batch], logits f32 [batch][vocab/tp]. */
TB_API int tb_qwen3_io(tb_qwen3 *m, uint32_t **ids, int32_t **pos, float **logits);
/* 128-byte NCCL unique id (rank 0 makes it, every rank passes it to tp_init). */
TB_API int tb_nccl_unique_id(void *out128);
TB_API int tb_qwen3_tp_init(tb_qwen3 *m, const void *unique_id128);
/* Exchange over NVLink peer memory instead of NCCL: every rank gets its
 * 64-byte CUDA IPC handle, the handles of all ranks are shared (rank order,
 * P x 64 bytes) and passed to tb_qwen3_tp_connect.  The step then sums the
 * o/down partials and merges the argmax with this library's own exchange
 * kernels (peer loads + system-scope flags, bounded waits that set the
 * device error word); the result is identical on every rank. */
TB_API int tb_qwen3_tp_handle(tb_qwen3 *m, void *out64);
TB_API int tb_qwen3_tp_connect(tb_qwen3 *m, const void *handles);
/* After a device-side exchange wait gave up under tensor parallelism (the
 * device error word reads 0x5103 / 0x7a01, tb_ctx_device_error returns
 * TB_ERR_TIMEOUT), the ranks' exchange epochs may disagree, so the rank
 * poisons itself: every later step on it does nothing and reports 0x5104
 * (persistent step) or 0x7a02 (exchange kernels) until this reset.  It clears
 * this rank's exchange arena, step control words and attention counters and
 * synchronizes.  Call it on every rank, with every rank's stream idle and
 * behind a host barrier, and step again only after every rank returned from it.
 * No reference counterpart (the reference has no tensor parallelism). */
TB_API int tb_qwen3_tp_reset(tb_qwen3 *m);
TB_API int tb_qwen3_decode_step(tb_qwen3 *m);
/* Kernels of this library in one recorded step, and NCCL collectives. */
TB_API int tb_qwen3_launches_per_step(tb_qwen3 *m, int *kernels, int *collectives);

#ifdef __cplusplus
}
#endif
#endif /* TABINFER_B200_H */
