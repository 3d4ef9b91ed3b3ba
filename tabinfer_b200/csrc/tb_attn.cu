// tb_attn.cu -- int8 KV cache and split-KV GQA decode attention.
//
// KV layout (models/qwen3.js:3835-3846 with bytes instead of packed words, the
// same memory): Kq/Vq int8 [S_max][nKv*hd], one f32 scale per 32 elements in
// Ks/Vs [S_max][nKv*hd/32].  Values are snorm int8: q = floor(0.5 + 127*clamp(x/m)),
// m = max(1e-12, max|x| over the group) (WGSL pack4x8snorm, qwen3.js:2180-2210),
// dequant = max(q/127, -1) * m.
//
// Decode (B200 design): one CTA per (kv head, split) serves all q heads of the
// GQA group, so every KV byte is read once per layer rather than once per q
// head.  Scores use one lane per key (its 128-byte K row in eight 16-byte
// loads); P.V uses one lane per 4 dims (coalesced 4-byte V loads).  Each warp
// keeps its own online-softmax state; the CTA merges warps and writes one
// (m, l, o) partial per q head; a combine kernel merges the splits
// (ATTN_DEC_COMBINE, qwen3.js:2048-2069).
#include "tb_internal.h"
#include "tb_attn_dev.cuh"

namespace {

// ---- fused prep: q rope, k rope + quant-write, v quant-write ---------------
// grid = (nHq + 2*nKv, B) CTAs, block = hd threads (hd % 32 == 0, hd <= 256).
// Sequence b reads q/k/v row b, writes qr row b and cache row pos_b of its own
// cache (cache_rows rows per sequence, caches seq_stride rows apart: seq_stride =
// cache_rows for a batch of sequences, 0 for the T tokens of one sequence's
// prefill); pos_b = dpos[b] when dpos is given (graph-replayable decode), else `pos`.
__global__ void __launch_bounds__(256) k_attn_prep(const float* __restrict__ q, const float* __restrict__ k,
                                                   const float* __restrict__ v, const uint16_t* __restrict__ qw,
                                                   const uint16_t* __restrict__ kw, float* __restrict__ qr,
                                                   int8_t* __restrict__ Kq, float* __restrict__ Ks,
                                                   int8_t* __restrict__ Vq, float* __restrict__ Vs,
                                                   int nHq, int nKv, int hd, long long pos, float theta, float eps,
                                                   const int* __restrict__ dpos, long long cache_rows,
                                                   long long seq_stride, int* err)
{
    __shared__ float rk[256];
    __shared__ float red[8];
    tb_pdl_wait();
    tb_pdl_trigger();
    const int j = threadIdx.x, lane = j & 31, wid = j >> 5, nw = hd >> 5;
    const int role = blockIdx.x, b = blockIdx.y;
    if (dpos) {
        pos = dpos[b];
        if (pos < 0 || pos >= cache_rows) {
            if (j == 0) atomicExch(err, ERR_ATTN_POS);
            return;
        }
    }
    const long long cache_off = (long long)b * seq_stride * nKv * hd;
    Kq += cache_off; Vq += cache_off; Ks += cache_off / 32; Vs += cache_off / 32;
    q += (long long)b * nHq * hd; qr += (long long)b * nHq * hd;
    k += (long long)b * nKv * hd; v += (long long)b * nKv * hd;
    const bool isQ = role < nHq, isK = !isQ && role < nHq + nKv;
    const int head = isQ ? role : (isK ? role - nHq : role - nHq - nKv);
    const float* src = isQ ? q : (isK ? k : v);
    float x = src[(long long)head * hd + j];
    if (isQ || isK) {
        float c, sn;
        rope_cs(j, hd, pos, theta, &c, &sn);
        x = norm_rope(x, isQ ? qw : kw, hd, eps, c, sn, rk, red);
        if (isQ) { qr[(long long)head * hd + j] = x; return; }
    }
    // quantize one 32-group per warp straight into the cache row `pos`
    const long long row = pos * nKv * hd + (long long)head * hd;
    quant_row(x, hd, (isK ? Kq : Vq) + row, (isK ? Ks : Vs) + row / 32);
    (void)lane; (void)wid; (void)nw;
}

// ---- prep of the T rows of one sequence's prefill ----------------------------
// One CTA per token row: its threads first form the row's rotary (cos, sin) pairs
// once (rope_cs, the double-precision angles), then each warp takes whole heads
// (q, k, then v): lane l holds elements l + 32 i, so the split-half rotary
// partner of every element (i +- hd/64) is in the same lane and no block barrier
// is needed.  Every value is the one k_attn_prep forms: the same per-32 warp sums
// added in the same order, the same norm, rotary and quantization arithmetic.
// HD = 64, 128 or 256.
template <int HD>
__global__ void __launch_bounds__(256) k_attn_prep_rows(const float* __restrict__ q, const float* __restrict__ k,
                                                        const float* __restrict__ v, const uint16_t* __restrict__ qw,
                                                        const uint16_t* __restrict__ kw, float* __restrict__ qr,
                                                        int8_t* __restrict__ Kq, float* __restrict__ Ks,
                                                        int8_t* __restrict__ Vq, float* __restrict__ Vs, int nHq,
                                                        int nKv, float theta, float eps,
                                                        const int* __restrict__ dpos, long long cache_rows, int* err)
{
    __shared__ float cs_c[128], cs_s[128];
    tb_pdl_wait();
    tb_pdl_trigger();
    const int t = blockIdx.x, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const long long pos = dpos[t];
    if (pos < 0 || pos >= cache_rows) {
        if (threadIdx.x == 0) atomicExch(err, ERR_ATTN_POS);
        return;
    }
    constexpr int hd = HD, half = HD / 2, nw = HD / 32;
    for (int f = threadIdx.x; f < half; f += blockDim.x) rope_cs(f, hd, pos, theta, &cs_c[f], &cs_s[f]);
    __syncthreads();
    q += (long long)t * nHq * hd;
    qr += (long long)t * nHq * hd;
    k += (long long)t * nKv * hd;
    v += (long long)t * nKv * hd;
    const int nroles = nHq + 2 * nKv;
    for (int role = wid; role < nroles; role += (int)(blockDim.x >> 5)) {
        const bool isQ = role < nHq, isK = !isQ && role < nHq + nKv;
        const int head = isQ ? role : (isK ? role - nHq : role - nHq - nKv);
        const float* src = (isQ ? q : (isK ? k : v)) + (long long)head * hd;
        float x[8];
#pragma unroll
        for (int i = 0; i < 8; i++) x[i] = i < nw ? src[32 * i + lane] : 0.0f;
        if (isQ || isK) {
            const uint16_t* w16 = isQ ? qw : kw;
            float tot = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; i++)
                if (i < nw) tot += warp_sum(x[i] * x[i]);
            const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)hd), eps)));
            float rk[8];
#pragma unroll
            for (int i = 0; i < 8; i++) rk[i] = i < nw ? __fmul_rn(__fmul_rn(x[i], inv), tb_h2f(w16[32 * i + lane])) : 0.0f;
            constexpr int hw = nw / 2;   // the rotary partner is hw registers away
#pragma unroll
            for (int i = 0; i < 8; i++) {
                if (i >= nw) break;
                const int j = 32 * i + lane, fi = j < half ? j : j - half;
                const float partner = i < hw ? rk[i + hw] : rk[i - hw];
                const float rot = j < half ? -partner : partner;
                x[i] = fmaf(rk[i], cs_c[fi], rot * cs_s[fi]);
            }
            if (isQ) {
#pragma unroll
                for (int i = 0; i < 8; i++)
                    if (i < nw) qr[(long long)head * hd + 32 * i + lane] = x[i];
                continue;
            }
        }
        // snorm int8 of each 32-group (quant_row) into the cache row `pos`
        const long long row = pos * nKv * hd + (long long)head * hd;
        int8_t* dq = (isK ? Kq : Vq) + row;
        float* ds = (isK ? Ks : Vs) + row / 32;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            if (i >= nw) break;
            const float m = fmaxf(1e-12f, warp_max(fabsf(x[i])));
            dq[32 * i + lane] = snorm8(__fdiv_rn(x[i], m));
            if (lane == 0) ds[i] = m;
        }
    }
}

// ---- prefill quant-write of T rows (KVQW) -----------------------------------
__global__ void __launch_bounds__(256) k_kv_quant_write(const float* __restrict__ kr, const float* __restrict__ v,
                                                        int8_t* __restrict__ Kq, float* __restrict__ Ks,
                                                        int8_t* __restrict__ Vq, float* __restrict__ Vs,
                                                        long long ngroups, long long base_elems)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    const int lane = threadIdx.x & 31;
    for (long long g = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; g < 2 * ngroups;
         g += ((long long)gridDim.x * blockDim.x) >> 5) {
        const bool isV = g >= ngroups;
        const long long gg = isV ? g - ngroups : g;
        const float x = (isV ? v : kr)[gg * 32 + lane];
        const float m = fmaxf(1e-12f, warp_max(fabsf(x)));
        (isV ? Vq : Kq)[base_elems + gg * 32 + lane] = snorm8(__fdiv_rn(x, m));
        if (lane == 0) (isV ? Vs : Ks)[base_elems / 32 + gg] = m;
    }
}

// hd fixed at compile time (64 or 128); GRP = q heads per kv head.  One CTA
// (W warps) per (kv head, split); the split's work is DecUnit (tb_attn_dev.cuh).
// 4-warp single-stage units of up to 2 q heads run five CTAs an SM (shared memory
// allows five): registers are held to that (wider groups would spill).
template <int HD, int GRP, bool EARLY, int W, int NST>
__global__ void __launch_bounds__(32 * W, (W == 4 && NST == 1 && GRP <= 2) ? 5 : 1) k_attn_decode(const AttnArgs a)
{
    extern __shared__ __align__(128) uint8_t smem[];
    if constexpr (EARLY) {
        // the position and every cache row below S-1 come from earlier steps: a
        // warp's first tile is fetched before griddepcontrol.wait unless it holds
        // row S-1, which the preceding prep kernel writes
        DecUnit<HD, GRP, NST, W> u(a, smem, blockIdx.x, blockIdx.y, blockIdx.z, threadIdx.x, 0);
        u.prefetch(true);
        tb_pdl_wait();
        tb_pdl_trigger();
        u.run(true);
    } else {
        tb_pdl_wait();
        tb_pdl_trigger();
        DecUnit<HD, GRP, NST, W> u(a, smem, blockIdx.x, blockIdx.y, blockIdx.z, threadIdx.x, 0);
        u.prefetch(false);
        u.run(false);
    }
}

template <int HD, int GRP, bool EARLY, int W, int NST>
int launch_decode_w(tb_ctx* ctx, const AttnArgs& a)
{
    constexpr int bytes = DecLayout<HD, GRP, NST, W>::BYTES;
    auto kern = k_attn_decode<HD, GRP, EARLY, W, NST>;
    static bool attr_set[64] = {};   // per device and instantiation; setting it twice is harmless
    if (ctx->device >= 64 || !attr_set[ctx->device]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "attn_decode attribute: %s", cudaGetErrorString(e));
        if (ctx->device < 64) attr_set[ctx->device] = true;
    }
    cudaError_t e = tb_launch(ctx, kern, dim3(a.nKv, a.nsplit, a.grid_z), dim3(32 * W), bytes, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "attn_decode launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

// one sequence (the decode step at batch 1, ~one split per SM): 8-warp splits,
// as the persistent decode step runs them; several sequences: 4-warp splits.
// A grid of at most one CTA an SM keeps two tile stages a warp (a tile in
// flight while one is scored); a larger grid takes one stage, which halves the
// shared memory so several CTAs share an SM (4-warp units: 41 KB, five an SM)
// and their warps hide each other's copies.
template <int HD, int GRP, bool EARLY>
int launch_decode(tb_ctx* ctx, const AttnArgs& a)
{
    const long long ctas = (long long)a.nKv * a.nsplit * a.grid_z;
    const bool one_stage = ctas > ctx->num_sms;
    if (a.grid_z == 1)
        return one_stage ? launch_decode_w<HD, GRP, EARLY, 8, 1>(ctx, a) : launch_decode_w<HD, GRP, EARLY, 8, 2>(ctx, a);
    return one_stage ? launch_decode_w<HD, GRP, EARLY, 4, 1>(ctx, a) : launch_decode_w<HD, GRP, EARLY, 4, 2>(ctx, a);
}

template <bool EARLY>
int decode_dispatch(tb_ctx* ctx, const AttnArgs& a, int64_t hd, int grp)
{
    if (hd == 128) {
        switch (grp) {
        case 1: return launch_decode<128, 1, EARLY>(ctx, a);
        case 2: return launch_decode<128, 2, EARLY>(ctx, a);
        case 4: return launch_decode<128, 4, EARLY>(ctx, a);
        case 8: return launch_decode<128, 8, EARLY>(ctx, a);
        default: return tb_fail(ctx, TB_ERR_UNSUPPORTED, "nHq/nKv = %d not built (1, 2, 4, 8)", grp);
        }
    } else if (hd == 64) {
        switch (grp) {
        case 1: return launch_decode<64, 1, EARLY>(ctx, a);
        case 2: return launch_decode<64, 2, EARLY>(ctx, a);
        case 4: return launch_decode<64, 4, EARLY>(ctx, a);
        case 8: return launch_decode<64, 8, EARLY>(ctx, a);
        default: return tb_fail(ctx, TB_ERR_UNSUPPORTED, "nHq/nKv = %d not built (1, 2, 4, 8)", grp);
        }
    }
    return tb_fail(ctx, TB_ERR_UNSUPPORTED, "head_dim %lld not built (64, 128)", (long long)hd);
}

}  // namespace

// Split count used when the caller passes nsplit = 0: at least 128 keys per
// CTA, and at long context as many (kv head, split) CTAs as fit in one wave of
// single-stage 4-warp units (five an SM), rounded down so no second, partial
// wave follows; a unit's combine weighs at most 256 splits.
int tb_attn_auto_nsplit(tb_ctx* ctx, int64_t S, int64_t nKv)
{
    long long by_keys = (S + 127) / 128;
    long long by_fill = std::max(1LL, 5LL * ctx->num_sms / nKv);
    long long n = std::min(by_keys, by_fill);
    return (int)std::max(1LL, std::min(n, 256LL));
}

// batch sequences (grid.z); sequence b's cache starts cache_rows rows after
// sequence b-1's; with dpos, S_b = dpos[b] + 1 is read on the device.
int tb_attn_decode_impl(tb_ctx* ctx, float* out, const float* qr, const int8_t* Kq, const float* Ks,
                        const int8_t* Vq, const float* Vs, int64_t S, int64_t nHq, int64_t nKv, int64_t hd,
                        int nsplit, float* PO, float* PML, unsigned* counters, int64_t batch,
                        int64_t cache_rows, const int32_t* dpos, bool early, unsigned char* mxa, uint2* mxk,
                        int mts, bool mtern)
{
    AttnArgs a{qr, Kq, Ks, Vq, Vs, PO, PML, out, counters, (const int*)dpos, ctx->dev_error,
               (long long)(cache_rows > 0 ? cache_rows : S), (int)S, (int)nHq, (int)nKv, nsplit};
    a.grid_z = (int)batch;
    if (mxa) {
        TB_REQUIRE(ctx, mxk && batch <= mts && ((nHq / nKv) * hd) % 128 == 0,
                   "attention: a fragment-order output needs its row slots and whole warps of groups");
        a.mxa = mxa;
        a.mxk = mxk;
        a.mts = mts;
        a.mtern = mtern ? 1 : 0;
    }
    return early ? decode_dispatch<true>(ctx, a, hd, (int)(nHq / nKv))
                 : decode_dispatch<false>(ctx, a, hd, (int)(nHq / nKv));
}

int tb_attn_check(tb_ctx* ctx, const float* qr, const int8_t* Kq, const float* Ks, const int8_t* Vq, const float* Vs,
                  int64_t S, int64_t nHq, int64_t nKv, int64_t hd, int nsplit)
{
    TB_REQUIRE(ctx, qr && Kq && Ks && Vq && Vs, "null pointer");
    TB_REQUIRE(ctx, S >= 0 && S < (1LL << 31), "bad S");
    TB_REQUIRE(ctx, nKv > 0 && nKv <= TB_ATTN_MAX_KV && nHq > 0 && nHq % nKv == 0 && nHq / nKv <= ATT_MAXG,
               "bad head counts nHq=%lld nKv=%lld", (long long)nHq, (long long)nKv);
    TB_REQUIRE(ctx, hd == 64 || hd == 128, "head_dim must be 64 or 128 (got %lld)", (long long)hd);
    TB_REQUIRE(ctx, TB_ALIGNED(Kq, 16) && TB_ALIGNED(Vq, 16) && TB_ALIGNED(Ks, 16) && TB_ALIGNED(Vs, 16),
               "KV cache must be 16-byte aligned");
    TB_REQUIRE(ctx, nsplit >= 0 && nsplit <= ATT_MAXSPLIT, "nsplit must be 0..%d", ATT_MAXSPLIT);
    return TB_OK;
}

// the prep of T tokens of ONE sequence (prefill): row t reads q/k/v row t,
// writes qr row t and cache row dpos[t] < cache_rows of the same cache
int tb_attn_prep_rows_impl(tb_ctx* ctx, const float* q, const float* k, const float* v, const uint16_t* qw16,
                           const uint16_t* kw16, float* qr, int8_t* Kq, float* Ks, int8_t* Vq, float* Vs, int64_t nHq,
                           int64_t nKv, int64_t hd, int64_t T, int64_t cache_rows, const int32_t* dpos, float theta,
                           float eps)
{
    TB_REQUIRE(ctx, hd % 32 == 0 && hd >= 32 && hd <= 256 && T > 0 && T <= 65535, "attn prep rows: bad shape");
    if ((hd == 64 || hd == 128 || hd == 256) && dpos) {
        auto kern = hd == 64 ? k_attn_prep_rows<64> : (hd == 128 ? k_attn_prep_rows<128> : k_attn_prep_rows<256>);
        cudaError_t e = tb_launch(ctx, kern, dim3((unsigned)T), dim3(256), 0, q, k, v, qw16, kw16, qr, Kq, Ks, Vq, Vs,
                                  (int)nHq, (int)nKv, theta, eps, (const int*)dpos, (long long)cache_rows,
                                  ctx->dev_error);
        if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "attn_prep_rows launch: %s", cudaGetErrorString(e));
        return TB_OK;
    }
    cudaError_t e = tb_launch(ctx, k_attn_prep, dim3((unsigned)(nHq + 2 * nKv), (unsigned)T), dim3((unsigned)hd), 0,
                              q, k, v, qw16, kw16, qr, Kq, Ks, Vq, Vs, (int)nHq, (int)nKv, (int)hd, 0LL, theta, eps,
                              (const int*)dpos, (long long)cache_rows, 0LL, ctx->dev_error);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "attn_prep launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

extern "C" {

TB_API int tb_attn_prep_q8(tb_ctx* ctx, const float* q, const float* k, const float* v, const uint16_t* qw16,
                           const uint16_t* kw16, float* qr, int8_t* Kq, float* Ks, int8_t* Vq, float* Vs,
                           int64_t nHq, int64_t nKv, int64_t hd, int64_t pos, float theta, float eps)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, q && k && v && qw16 && kw16 && qr && Kq && Ks && Vq && Vs, "null pointer");
    TB_REQUIRE(ctx, hd % 32 == 0 && hd >= 32 && hd <= 256, "head_dim must be a multiple of 32 in [32, 256]");
    TB_REQUIRE(ctx, nHq > 0 && nKv > 0 && pos >= 0, "bad head counts or position");
    cudaError_t e = tb_launch(ctx, k_attn_prep, dim3((unsigned)(nHq + 2 * nKv)), dim3((unsigned)hd), 0, q, k, v, qw16,
                              kw16, qr, Kq, Ks, Vq, Vs, (int)nHq, (int)nKv, (int)hd, (long long)pos, theta, eps,
                              (const int*)nullptr, (long long)(pos + 1), 0LL, ctx->dev_error);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "attn_prep launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_attn_prep_q8_batch(tb_ctx* ctx, const float* q, const float* k, const float* v, const uint16_t* qw16,
                                 const uint16_t* kw16, float* qr, int8_t* Kq, float* Ks, int8_t* Vq, float* Vs,
                                 int64_t nHq, int64_t nKv, int64_t hd, int64_t batch, int64_t cache_rows,
                                 const int32_t* dpos, float theta, float eps)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, q && k && v && qw16 && kw16 && qr && Kq && Ks && Vq && Vs && dpos, "null pointer");
    TB_REQUIRE(ctx, hd % 32 == 0 && hd >= 32 && hd <= 256, "head_dim must be a multiple of 32 in [32, 256]");
    TB_REQUIRE(ctx, nHq > 0 && nKv > 0 && batch > 0 && batch <= 65535 && cache_rows > 0, "bad head counts, batch or cache rows");
    cudaError_t e = tb_launch(ctx, k_attn_prep, dim3((unsigned)(nHq + 2 * nKv), (unsigned)batch), dim3((unsigned)hd), 0,
                              q, k, v, qw16, kw16, qr, Kq, Ks, Vq, Vs, (int)nHq, (int)nKv, (int)hd, 0LL, theta, eps,
                              (const int*)dpos, (long long)cache_rows, (long long)cache_rows, ctx->dev_error);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "attn_prep launch: %s", cudaGetErrorString(e));
    return TB_OK;
}



TB_API int tb_kv_quant_write(tb_ctx* ctx, const float* kr, const float* v, int8_t* Kq, float* Ks, int8_t* Vq,
                             float* Vs, int64_t T, int64_t nKv, int64_t hd, int64_t posBase)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, kr && v && Kq && Ks && Vq && Vs, "null pointer");
    TB_REQUIRE(ctx, T > 0 && nKv > 0 && hd % 32 == 0 && posBase >= 0, "bad shape");
    long long ng = T * nKv * hd / 32;
    int grid = (int)std::min<long long>((2 * ng * 32 + 255) / 256, (long long)ctx->num_sms * 8);
    cudaError_t e = tb_launch(ctx, k_kv_quant_write, dim3(grid), dim3(256), 0, kr, v, Kq, Ks, Vq, Vs, ng,
                              (long long)(posBase * nKv * hd));
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "kv_quant_write launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_attn_decode_q8(tb_ctx* ctx, float* out, const float* qr, const int8_t* Kq, const float* Ks,
                             const int8_t* Vq, const float* Vs, int64_t S, int64_t nHq, int64_t nKv, int64_t hd,
                             int nsplit)
{
    if (!ctx) return TB_ERR_INVALID;
    int rc = tb_attn_check(ctx, qr, Kq, Ks, Vq, Vs, S, nHq, nKv, hd, nsplit);
    if (rc) return rc;
    TB_REQUIRE(ctx, out != nullptr && TB_ALIGNED(out, 16), "output must be non-null and 16-byte aligned");
    if (nsplit == 0) nsplit = tb_attn_auto_nsplit(ctx, S, nKv);
    size_t po = (size_t)nHq * nsplit * hd * sizeof(float), pml = (size_t)nHq * nsplit * 2 * sizeof(float);
    float* scr = static_cast<float*>(tb_ctx_scratch(ctx, po + pml));
    if (!scr) return TB_ERR_NOMEM;
    return tb_attn_decode_impl(ctx, out, qr, Kq, Ks, Vq, Vs, S, nHq, nKv, hd, nsplit, scr, scr + po / sizeof(float),
                               ctx->attn_counters);
}

TB_API int tb_attn_decode_q8_batch(tb_ctx* ctx, float* out, const float* qr, const int8_t* Kq, const float* Ks,
                                   const int8_t* Vq, const float* Vs, int64_t batch, int64_t cache_rows,
                                   const int32_t* dpos, int64_t S_max, int64_t nHq, int64_t nKv, int64_t hd, int nsplit)
{
    if (!ctx) return TB_ERR_INVALID;
    int rc = tb_attn_check(ctx, qr, Kq, Ks, Vq, Vs, S_max, nHq, nKv, hd, nsplit);
    if (rc) return rc;
    TB_REQUIRE(ctx, out != nullptr && TB_ALIGNED(out, 16), "output must be non-null and 16-byte aligned");
    TB_REQUIRE(ctx, dpos != nullptr, "null positions");
    TB_REQUIRE(ctx, batch > 0 && batch <= 65535 && batch * nKv <= TB_ATTN_MAX_KV, "batch * nKv must be <= %d",
               TB_ATTN_MAX_KV);
    TB_REQUIRE(ctx, cache_rows >= S_max && S_max >= 1, "S_max must be in [1, cache_rows]");
    if (nsplit == 0) nsplit = tb_attn_auto_nsplit(ctx, S_max, nKv * batch);
    size_t po = (size_t)batch * nHq * nsplit * hd * sizeof(float), pml = (size_t)batch * nHq * nsplit * 2 * sizeof(float);
    float* scr = static_cast<float*>(tb_ctx_scratch(ctx, po + pml));
    if (!scr) return TB_ERR_NOMEM;
    return tb_attn_decode_impl(ctx, out, qr, Kq, Ks, Vq, Vs, S_max, nHq, nKv, hd, nsplit, scr,
                               scr + po / sizeof(float), ctx->attn_counters, batch, cache_rows, dpos);
}

}  // extern "C"

// ---- allocation-free split-KV decode ----------------------------------------------
// No counterpart in the reference.  tb_attn_decode_q8 keeps its split partials in
// context scratch, which it allocates with cudaMalloc the first time a size is
// needed.  Some callers cannot allow that: a serving process that hands its whole
// device memory budget to its own pool at start-up and forbids later driver
// allocations, or a host loop that must not let cudaMalloc/cudaFree synchronize
// the device in the middle of a decode step.  This variant allocates nothing: its
// partials live in the file-scope array below, sized at NOALLOC_SCRATCH_FLOATS
// floats (1 MiB), which every GPU that loads this library holds until exit.
//  * Limit: nHq * nsplit * (hd + 2) <= NOALLOC_SCRATCH_FLOATS (Qwen3-1.7B, 16 q
//    heads x hd 128, fits up to 126 splits); an explicit split count beyond it is
//    rejected with TB_ERR_INVALID before anything is enqueued.  With nsplit = 0
//    the automatic split count is capped at what fits, so wide models (64 q heads
//    at long context) still run, with fewer splits.
//  * The device address of the array is looked up once per device, on the first
//    call made on that device (cudaGetSymbolAddress with the device current); make
//    that first call before any stream capture.
//  * Every call shares the one array and it keeps the last call's contents.
//    Nothing needs clearing (each split writes its partial before the combine
//    reads it; the split-arrival counters beside it start at zero and each call
//    leaves them at zero), but calls that overlap on the GPU (other streams,
//    other contexts on the same device) race on them: order them.
constexpr size_t NOALLOC_SCRATCH_FLOATS = size_t(1) << 18;
static __device__ __align__(256) float g_attn_noalloc_scratch[NOALLOC_SCRATCH_FLOATS];
static __device__ unsigned g_attn_noalloc_counters[TB_ATTN_MAX_KV];

#include <mutex>

namespace {
constexpr int NOALLOC_MAX_DEVICES = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[NOALLOC_MAX_DEVICES] = {};
unsigned* g_noalloc_cnt[NOALLOC_MAX_DEVICES] = {};

// Device addresses of the arrays on ctx's device (host code may not use the
// symbols themselves as addresses).
int noalloc_scratch(tb_ctx* ctx, float** out, unsigned** counters)
{
    TB_REQUIRE(ctx, ctx->device >= 0 && ctx->device < NOALLOC_MAX_DEVICES, "device index out of range");
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[ctx->device]) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaError_t e = cudaSetDevice(ctx->device);
        void* p = nullptr;
        void* c = nullptr;
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&c, g_attn_noalloc_counters);
        cudaSetDevice(prev);
        if (e != cudaSuccess || !p || !c)
            return tb_fail(ctx, TB_ERR_CUDA, "cudaGetSymbolAddress(attention scratch): %s", cudaGetErrorString(e));
        g_noalloc_cnt[ctx->device] = static_cast<unsigned*>(c);
        g_noalloc_ptr[ctx->device] = static_cast<float*>(p);
    }
    *out = g_noalloc_ptr[ctx->device];
    *counters = g_noalloc_cnt[ctx->device];
    return TB_OK;
}
}  // namespace

extern "C" TB_API int tb_attn_decode_q8_noalloc(tb_ctx* ctx, float* out, const float* qr, const int8_t* Kq,
                                                const float* Ks, const int8_t* Vq, const float* Vs, int64_t S,
                                                int64_t nHq, int64_t nKv, int64_t hd, int nsplit)
{
    if (!ctx) return TB_ERR_INVALID;
    int rc = tb_attn_check(ctx, qr, Kq, Ks, Vq, Vs, S, nHq, nKv, hd, nsplit);
    if (rc) return rc;
    TB_REQUIRE(ctx, out != nullptr && TB_ALIGNED(out, 16), "output must be non-null and 16-byte aligned");
    if (nsplit == 0) {
        const int64_t fit = (int64_t)(NOALLOC_SCRATCH_FLOATS / (size_t)(nHq * (hd + 2)));
        nsplit = (int)std::max<int64_t>(1, std::min<int64_t>(tb_attn_auto_nsplit(ctx, S, nKv), fit));
    }
    const size_t need = (size_t)nHq * nsplit * (hd + 2);
    if (need > NOALLOC_SCRATCH_FLOATS)
        return tb_fail(ctx, TB_ERR_INVALID,
                       "attn_decode_q8_noalloc: nHq*nsplit*(hd+2) = %zu floats exceeds the fixed scratch of %zu floats "
                       "(use fewer splits or tb_attn_decode_q8)", need, NOALLOC_SCRATCH_FLOATS);
    float* scr = nullptr;
    unsigned* cnt = nullptr;
    rc = noalloc_scratch(ctx, &scr, &cnt);
    if (rc) return rc;
    return tb_attn_decode_impl(ctx, out, qr, Kq, Ks, Vq, Vs, S, nHq, nKv, hd, nsplit, scr,
                               scr + (size_t)nHq * nsplit * hd, cnt);
}
