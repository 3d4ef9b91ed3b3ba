// tb_moe.cu -- int3 mixture-of-experts FFN of LFM2.5 (models/lfm25.js):
//   _requant43 (:833-855)   int4 G=32 entries -> int3 bitplanes + f16 scales
//   ROUTER_WGSL (:111-141)  sigmoid scores, top-k of score + bias, normalised weights
//   idxGemv3 (:1924-1980)   pair-indexed expert GEMV on int3 bitplanes
//   MOECOMBINE (:1982-2000) x += sum_k wt_k * o_k
//
// int3 layout (identical to the reference, so its packed experts load as is):
// per (row, 32-group) three u32 bitplanes b0, b1, b2 -- bit i of plane p is bit
// p of the stored value q3 + 4 of weight i -- at words (row*G + g)*3 + p, and an
// f16 scale at row*G + g.  Expert e's rows are rows e*N .. e*N + N-1.
//
// The expert GEMV here is grouped: the (token, k) pairs are sorted by expert
// (k_moe_group), one CTA takes an expert's row block and every pair routed to
// that expert (in chunks of up to MB), decoding each 32-weight group once and
// applying it to all the chunk's activation rows staged in shared memory.
#include "tb_internal.h"

namespace {

constexpr int MB = 8;          // pairs per chunk
constexpr int MOE_THREADS = 256;
// rows per warp (and per CTA): gate/up decodes two matrices, so one row a warp
template <int KIND> constexpr int moe_rpw() { return KIND == 0 ? 1 : 2; }
template <int KIND> constexpr int moe_rb() { return moe_rpw<KIND>() * MOE_THREADS / 32; }
constexpr int MOE_GPL = 2;     // 32-groups per lane and row (K <= 2048)
constexpr int MOE_BPC = 4;     // row blocks per CTA (weights of the next one in flight) with many pairs
constexpr int XS_PAD = 36;     // floats per staged 32-group (4 of padding: conflict-free 16-byte reads)

// ---- _requant43 -------------------------------------------------------------
// The engine's f32ToF16 (engine/webgpu-engine.js:217-236): mantissa rounded
// half-up on bit 12, and the rounded mantissa ORed (not added) into the
// exponent field, so a carry out of the mantissa is kept only when the
// exponent's low bit is clear.  Reproduced as is.
__device__ __forceinline__ uint32_t engine_f32_to_f16(float v)
{
    const uint32_t x = __float_as_uint(v);
    const uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t mant = x & 0x007fffffu;
    const int ex = (int)((x >> 23) & 0xffu);
    if (ex == 255) return sign | (mant ? 0x7e00u : 0x7c00u);
    const int e = ex - 127 + 15;
    if (e >= 31) return sign | 0x7c00u;
    if (e <= 0) {
        if (e < -10) return sign;
        mant = (mant | 0x00800000u) >> (1 - e);
        return sign | ((mant + 0x00001000u) >> 13);
    }
    return sign | ((uint32_t)e << 10) | ((mant + 0x00001000u) >> 13);
}

// JavaScript Math.round (ties toward +inf)
__device__ __forceinline__ double js_round_d(double v)
{
    const double f = floor(v);
    return __dsub_rn(v, f) >= 0.5 ? __dadd_rn(f, 1.0) : f;
}

__device__ __forceinline__ double f16_to_f64(uint32_t h)
{
    return (double)__half2float(__ushort_as_half((unsigned short)h));
}

// one thread per (row, 32-group)
__global__ void __launch_bounds__(256) k_requant43(const uint32_t* __restrict__ pack4, const uint16_t* __restrict__ s4,
                                                   uint32_t* __restrict__ p3, uint16_t* __restrict__ s3, long long ngroups)
{
    tb_pdl_wait();
    for (long long gi = blockIdx.x * (long long)blockDim.x + threadIdx.x; gi < ngroups;
         gi += (long long)gridDim.x * blockDim.x) {
        const uint4 w = reinterpret_cast<const uint4*>(pack4)[gi];
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        int m = 0;
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const int q = (int)((ws[i >> 3] >> (4 * (i & 7))) & 15u) - 8;
            m = max(m, q < 0 ? -q : q);
        }
        if (m == 0) {
            p3[gi * 3] = 0u; p3[gi * 3 + 1] = 0u; p3[gi * 3 + 2] = 0xFFFFFFFFu;
            s3[gi] = 0;
            continue;
        }
        const double ratio = __ddiv_rn(4.0, (double)m);
        // f16 scale * m / 4 in double (exact), stored as f32, then the engine's f32ToF16
        const float s3f = (float)__ddiv_rn(__dmul_rn(f16_to_f64(s4[gi]), (double)m), 4.0);
        uint32_t b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const int q4 = (int)((ws[i >> 3] >> (4 * (i & 7))) & 15u) - 8;
            int q = (int)js_round_d(__dmul_rn((double)q4, ratio));
            q = q > 3 ? 3 : (q < -4 ? -4 : q);
            const uint32_t st = (uint32_t)(q + 4);
            b0 |= (st & 1u) << i;
            b1 |= ((st >> 1) & 1u) << i;
            b2 |= ((st >> 2) & 1u) << i;
        }
        p3[gi * 3] = b0; p3[gi * 3 + 1] = b1; p3[gi * 3 + 2] = b2;
        s3[gi] = (uint16_t)engine_f32_to_f16(s3f);
    }
}

// ---- router ---------------------------------------------------------------------
// one CTA per token: scores = sigmoid(logits); K passes of a first-maximum search
// over score + bias (strict >, so the lower expert wins ties); weights =
// score / (sum of the selected scores + 1e-6), summed in selection order
__global__ void __launch_bounds__(64) k_moe_router(const float* __restrict__ logits, const float* __restrict__ bias,
                                                   uint32_t* __restrict__ idx, float* __restrict__ wt, int nE, int K)
{
    __shared__ float sc[64], sel[64];
    tb_pdl_wait();
    tb_pdl_trigger();
    const int t = blockIdx.x, e = threadIdx.x;
    if (e < nE) {
        const float s = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-logits[(long long)t * nE + e])));
        sc[e] = s;
        sel[e] = __fadd_rn(s, bias[e]);
    }
    __syncthreads();
    if (e == 0) {
        float sum = 0.0f;
        for (int k = 0; k < K; k++) {
            int best = 0;
            float bv = -1.0e30f;
            for (int j = 0; j < nE; j++)
                if (sel[j] > bv) { bv = sel[j]; best = j; }
            sel[best] = -2.0e30f;
            idx[(long long)t * K + k] = (uint32_t)best;
            wt[(long long)t * K + k] = sc[best];
            sum = __fadd_rn(sum, sc[best]);
        }
        const float den = __fadd_rn(sum, 1e-6f);
        for (int k = 0; k < K; k++) wt[(long long)t * K + k] = __fdiv_rn(wt[(long long)t * K + k], den);
    }
}

// ---- grouping: the pairs (t, k) = t*K + k sorted by expert, stable ------------
// one CTA: offsets[e] = first position of expert e in `order`, offsets[nE] = P;
// active[0 .. *nactive) = the experts with pairs, in order (the GEMVs launch
// one expert slot per pair at most and read their expert from this list)
__global__ void __launch_bounds__(256) k_moe_group(const uint32_t* __restrict__ idx, int P, int nE,
                                                   int* __restrict__ order, int* __restrict__ offsets,
                                                   int* __restrict__ active, int* __restrict__ nactive, int* err)
{
    __shared__ int cnt[257];
    tb_pdl_wait();
    tb_pdl_trigger();
    for (int e = threadIdx.x; e <= nE; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < P; p += blockDim.x) {
        const uint32_t e = idx[p];
        if (e < (uint32_t)nE) atomicAdd(&cnt[e + 1], 1);
        else atomicExch(err, 0x6c01);   // an expert id out of range: the pair is dropped
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int na = 0;
        for (int e = 0; e < nE; e++) {
            if (cnt[e + 1] > 0) active[na++] = e;
            cnt[e + 1] += cnt[e];
        }
        *nactive = na;
        for (int e = 0; e <= nE; e++) offsets[e] = cnt[e];
        // stable placement in pair order
        for (int p = 0; p < P; p++) {
            const uint32_t e = idx[p];
            if (e < (uint32_t)nE) order[cnt[e]++] = p;
        }
    }
}

// ---- bf16 -> int3 at group 32 or 128 (config 5's format; not in the reference) ----
// One warp per (row, group): scale = f16(max|w| / 4) through the engine's
// f32ToF16 (the conversion _requant43 uses for its scales), q = clamp(rn(w /
// scale), -4, 3) in f32, stored q + 4 in the three bitplanes of every 32-group
// of the group (the same planes as _requant43's); max|w| == 0 gives scale 0 and
// q = 0.  GP = 32-groups per scale group.
__global__ void __launch_bounds__(256) k_quant_int3(const uint16_t* __restrict__ w, uint32_t* __restrict__ p3,
                                                    uint16_t* __restrict__ s3, long long ngroups, int GP)
{
    // weights are inputs only; a dependent GEMV may start once they are all written
    tb_pdl_wait();
    const int lane = threadIdx.x & 31;
    for (long long gi = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; gi < ngroups;
         gi += ((long long)gridDim.x * blockDim.x) >> 5) {
        const uint16_t* src = w + gi * 32 * GP;
        float m = 0.0f;
        for (int j = 0; j < GP; j++) m = fmaxf(m, fabsf(__uint_as_float((uint32_t)src[j * 32 + lane] << 16)));
        m = warp_max(m);
        const uint32_t sh = engine_f32_to_f16(__fdiv_rn(m, 4.0f));
        const float sc = __half2float(__ushort_as_half((unsigned short)sh));
        for (int j = 0; j < GP; j++) {
            const float v = __uint_as_float((uint32_t)src[j * 32 + lane] << 16);
            const int q = sc > 0.0f ? max(-4, min(3, __float2int_rn(__fdiv_rn(v, sc)))) : 0;
            const uint32_t st = (uint32_t)(q + 4);
            const uint32_t b0 = __ballot_sync(0xffffffffu, st & 1u), b1 = __ballot_sync(0xffffffffu, (st >> 1) & 1u),
                           b2 = __ballot_sync(0xffffffffu, (st >> 2) & 1u);
            if (lane == 0) {
                uint32_t* d = p3 + (gi * GP + j) * 3;
                d[0] = b0; d[1] = b1; d[2] = b2;
            }
        }
        if (lane == 0) s3[gi] = (uint16_t)sh;
    }
}

// ---- grouped int3 expert GEMV ---------------------------------------------------
enum { MOE_GATEUP = 0, MOE_DOWN = 1 };

constexpr int EP_MAX = 8;       // expert-parallel ranks

struct MoeArgs {
    const float* x;              // activation rows
    long long x_stride;          // floats between activation rows
    int xdiv;                    // pair p reads activation row p / xdiv (K for gate/up, 1 for down)
    const uint32_t* p3[2];       // [E*N][G][3]
    const uint16_t* s3[2];       // [E*N][G]
    float* y;                    // [P][N]: swi (gate/up) or expert outputs (down)
    const int* order;            // position -> pair; null: the identity
    const int* offsets;
    int N, Kc, G;
    int sg = 1;                  // 32-groups per scale: 1 (group 32, the reference's) or 4 (group 128)
    const int* xrow = nullptr;   // when set, pair p reads activation row xrow[p]
    int bpc = MOE_BPC;           // row blocks per CTA
    int mb = MB;                 // pairs per chunk (<= MB): the staged activations' rows
    // when set, expert slot blockIdx.y runs expert active[blockIdx.y] (slots past
    // *nactive return); else slot = expert
    const int* active = nullptr;
    const int* nactive = nullptr;
    // when set (expert parallel), pair p's output row goes to another rank's
    // memory: c = ydst[p], row (c & 0xffffff) of ypeer[c >> 24]
    const uint32_t* ydst = nullptr;
    float* ypeer[EP_MAX] = {};
};

// weights 4j .. 4j+3 (q3 + 4 in three bitplanes) of one 32-group as floats q - 4
__device__ __forceinline__ void decode4(uint32_t b0, uint32_t b1, uint32_t b2, int j, float* q)
{
    // spread the 4 bits of each plane's nibble j into the low bit of 4 bytes
    const uint32_t n0 = ((b0 >> (4 * j)) & 15u) * 0x00204081u & 0x01010101u;
    const uint32_t n1 = ((b1 >> (4 * j)) & 15u) * 0x00204081u & 0x01010101u;
    const uint32_t n2 = ((b2 >> (4 * j)) & 15u) * 0x00204081u & 0x01010101u;
    const uint32_t v = n0 | (n1 << 1) | (n2 << 2);   // 4 bytes, each q3 + 4 in 0..7
#pragma unroll
    for (int k = 0; k < 4; k++)
        q[k] = __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7540 + k)) - 8388612.0f;   // 2^23 + 4
}

template <int KIND>
__global__ void __launch_bounds__(MOE_THREADS) k_moe_gemv3(const MoeArgs a)
{
    constexpr int NM = KIND == MOE_GATEUP ? 2 : 1;
    constexpr int RPW = moe_rpw<KIND>();
    extern __shared__ __align__(16) float xs[];   // [MB][G][XS_PAD]: xs[b][g][i] = x_b[32 g + i]
    tb_pdl_wait();
    tb_pdl_trigger();
    int e = blockIdx.y;
    if (a.active) {
        if ((int)blockIdx.y >= *a.nactive) return;
        e = a.active[blockIdx.y];
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int G = a.G;
    const int p0 = a.offsets[e], np = a.offsets[e + 1] - p0;
    if (np == 0) return;
    // planes and scales of one row block of this warp, requested before use
    struct W {
        uint32_t w[RPW][MOE_GPL][NM][3];
        float s[RPW][MOE_GPL][NM];
    };
    auto fetch = [&](int blk, W& d) {
        const int rw0 = (blockIdx.x * a.bpc + blk) * moe_rb<KIND>() + wid * RPW;
#pragma unroll
        for (int j = 0; j < RPW; j++)
#pragma unroll
            for (int t = 0; t < MOE_GPL; t++)
#pragma unroll
                for (int m = 0; m < NM; m++) {
                    const int r = rw0 + j, g = lane + 32 * t;
                    const bool ok = r < a.N && g < G;
                    const long long row = (long long)e * a.N + (ok ? r : 0);
                    const uint32_t* w = a.p3[m] + (row * G + (ok ? g : 0)) * 3;
                    d.w[j][t][m][0] = ok ? __ldg(w) : 0u;
                    d.w[j][t][m][1] = ok ? __ldg(w + 1) : 0u;
                    d.w[j][t][m][2] = ok ? __ldg(w + 2) : 0u;
                    d.s[j][t][m] = ok ? tb_h2f(__ldg(a.s3[m] + row * (G / a.sg) + (ok ? g : 0) / a.sg)) : 0.0f;
                }
    };
    for (int c0 = 0; c0 < np; c0 += a.mb) {
        const int nb = min(a.mb, np - c0);
        W cur, nxt;
        fetch(0, cur);                       // in flight while the activations are staged
        __syncthreads();                     // the previous chunk's reads are done
        for (int b = 0; b < nb; b++) {
            const int p = a.order ? a.order[p0 + c0 + b] : p0 + c0 + b;
            const float* src = a.x + (long long)(a.xrow ? a.xrow[p] : p / a.xdiv) * a.x_stride;
            for (int k = threadIdx.x; k < a.Kc; k += MOE_THREADS)
                xs[(b * G + (k >> 5)) * XS_PAD + (k & 31)] = src[k];
        }
        __syncthreads();
        for (int blk = 0; blk < a.bpc; blk++) {
            if (blk + 1 < a.bpc) fetch(blk + 1, nxt);
            const int rw0 = (blockIdx.x * a.bpc + blk) * moe_rb<KIND>() + wid * RPW;
            float acc[NM][RPW][MB];
#pragma unroll
            for (int m = 0; m < NM; m++)
#pragma unroll
                for (int j = 0; j < RPW; j++)
#pragma unroll
                    for (int b = 0; b < MB; b++) acc[m][j][b] = 0.0f;
#pragma unroll
            for (int t = 0; t < MOE_GPL; t++) {
                const int g = lane + 32 * t;
                if (g < G) {
                    // the group nibble by nibble: weights 4 i4 .. 4 i4 + 3 of every (row,
                    // matrix) of the warp, then each staged activation float4 read from
                    // shared memory ONCE for all of them (not once per row and matrix);
                    // every sum still runs over the group's k in order, then one fmaf
                    // with the group scale, so the results are the same bits
                    float sum[RPW][NM][MB];
#pragma unroll
                    for (int j = 0; j < RPW; j++)
#pragma unroll
                        for (int m = 0; m < NM; m++)
#pragma unroll
                            for (int b = 0; b < MB; b++) sum[j][m][b] = 0.0f;
#pragma unroll
                    for (int i4 = 0; i4 < 8; i4++) {
                        float q[RPW][NM][4];
#pragma unroll
                        for (int j = 0; j < RPW; j++)
#pragma unroll
                            for (int m = 0; m < NM; m++)
                                decode4(cur.w[j][t][m][0], cur.w[j][t][m][1], cur.w[j][t][m][2], i4, q[j][m]);
#pragma unroll
                        for (int b = 0; b < MB; b++) {
                            if (b >= nb) break;      // one failed test per pass, not MB - nb
                            const float4 xv = reinterpret_cast<const float4*>(xs + (b * G + g) * XS_PAD)[i4];
#pragma unroll
                            for (int j = 0; j < RPW; j++)
#pragma unroll
                                for (int m = 0; m < NM; m++) {
                                    float v = sum[j][m][b];
                                    v = fmaf(q[j][m][0], xv.x, v);
                                    v = fmaf(q[j][m][1], xv.y, v);
                                    v = fmaf(q[j][m][2], xv.z, v);
                                    v = fmaf(q[j][m][3], xv.w, v);
                                    sum[j][m][b] = v;
                                }
                        }
                    }
#pragma unroll
                    for (int j = 0; j < RPW; j++)
#pragma unroll
                        for (int m = 0; m < NM; m++)
#pragma unroll
                            for (int b = 0; b < MB; b++) {
                                if (b >= nb) break;
                                acc[m][j][b] = fmaf(cur.s[j][t][m], sum[j][m][b], acc[m][j][b]);
                            }
                }
            }
#pragma unroll
            for (int m = 0; m < NM; m++)
#pragma unroll
                for (int j = 0; j < RPW; j++)
#pragma unroll
                    for (int b = 0; b < MB; b++) acc[m][j][b] = warp_sum(acc[m][j][b]);
            if (lane == 0) {
#pragma unroll
                for (int j = 0; j < RPW; j++) {
                    const int r = rw0 + j;
                    if (r >= a.N) continue;
                    for (int b = 0; b < nb; b++) {
                        const int p = a.order ? a.order[p0 + c0 + b] : p0 + c0 + b;
                        float v;
                        if (KIND == MOE_GATEUP) {
                            const float gg = acc[0][j][b], u = acc[NM - 1][j][b];
                            v = __fdiv_rn(gg, 1.0f + expf(-gg)) * u;      // silu(gate) * up
                        } else {
                            v = acc[0][j][b];
                        }
                        if (a.ydst) {
                            const uint32_t c = a.ydst[p];
                            a.ypeer[c >> 24][(long long)(c & 0xffffffu) * a.N + r] = v;
                        } else {
                            a.y[(long long)p * a.N + r] = v;
                        }
                    }
                }
            }
            cur = nxt;
        }
    }
}

// x[t, h] += sum_k wt[t, k] * o[t*K + k, h]  (k in order)
__global__ void __launch_bounds__(256) k_moe_combine(float* __restrict__ x, const float* __restrict__ o,
                                                     const float* __restrict__ wt, int H, int K, long long total)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
        const long long t = i / H, h = i - t * H;
        float s = 0.0f;
        for (int k = 0; k < K; k++) s = fmaf(wt[t * K + k], o[(t * K + k) * H + h], s);
        x[i] += s;
    }
}

size_t moe_smem(int Kc, int mb) { return (size_t)mb * (Kc / 32) * XS_PAD * sizeof(float); }

// nslots: expert slots of the grid (nE, or at most the pair count with a.active)
template <int KIND>
int launch_moe(tb_ctx* ctx, const MoeArgs& a, int nslots)
{
    const size_t smem = moe_smem(a.Kc, a.mb);
    TB_REQUIRE(ctx, a.G <= 32 * MOE_GPL, "moe: K = %d above %d", a.Kc, 32 * 32 * MOE_GPL);
    TB_REQUIRE(ctx, smem <= 200 * 1024, "moe: K = %d too large for the staged activations", a.Kc);
    cudaError_t e = cudaFuncSetAttribute(k_moe_gemv3<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
        e = tb_launch(ctx, k_moe_gemv3<KIND>, dim3((unsigned)tb_cdiv(a.N, moe_rb<KIND>() * a.bpc), (unsigned)nslots),
                      dim3(MOE_THREADS),
                      smem, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "moe gemv launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

}  // namespace

extern "C" {

TB_API int tb_requant_int4_int3(tb_ctx* ctx, uint32_t* p3, uint16_t* s3, const uint32_t* pack4, const uint16_t* s4,
                                int64_t rows, int64_t K)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, p3 && s3 && pack4 && s4, "null pointer");
    TB_REQUIRE(ctx, rows > 0 && K > 0 && K % 32 == 0, "bad shape (K %% 32 must be 0)");
    TB_REQUIRE(ctx, TB_ALIGNED(pack4, 16), "int4 pack must be 16-byte aligned");
    const long long ng = rows * (K / 32);
    const int grid = (int)std::min<long long>((ng + 255) / 256, (long long)ctx->num_sms * 16);
    cudaError_t e = tb_launch(ctx, k_requant43, dim3(grid), dim3(256), 0, pack4, s4, p3, s3, ng);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "requant43 launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_moe_router(tb_ctx* ctx, uint32_t* idx, float* wt, const float* logits, const float* bias, int64_t T,
                         int64_t nE, int64_t K)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, idx && wt && logits && bias, "null pointer");
    TB_REQUIRE(ctx, T > 0 && T <= 65535 && nE > 0 && nE <= 64 && K > 0 && K <= nE, "bad router shape (nE <= 64)");
    cudaError_t e = tb_launch(ctx, k_moe_router, dim3((unsigned)T), dim3(64), 0, logits, bias, idx, wt, (int)nE, (int)K);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "router launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

// The MoE FFN of T tokens: x_out[t] += sum_k wt[t,k] * W2_e (silu(W1_e a_t) * (W3_e a_t)),
// e = idx[t,k], a_t = x_in row t.  w1/w3: [nE*I][H/32][3] planes + [nE*I][H/32]
// scales; w2: [nE*H][I/32][3] + [nE*H][I/32].  Scratch: context-owned.
TB_API int tb_moe_ffn_int3_g(tb_ctx* ctx, float* x_out, const float* x_in, const uint32_t* idx, const float* wt,
                             const uint32_t* w1p, const uint16_t* w1s, const uint32_t* w3p, const uint16_t* w3s,
                             const uint32_t* w2p, const uint16_t* w2s, int64_t T, int64_t K, int64_t nE, int64_t H,
                             int64_t I, int group)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, x_out && x_in && idx && wt && w1p && w1s && w3p && w3s && w2p && w2s, "null pointer");
    TB_REQUIRE(ctx, group == 32 || group == 128, "int3 scale group must be 32 or 128 (got %d)", group);
    TB_REQUIRE(ctx, H % group == 0 && I % group == 0, "H and I must be multiples of the scale group");
    TB_REQUIRE(ctx, T > 0 && K > 0 && nE > 0 && nE <= 256 && H % 32 == 0 && I % 32 == 0 && H > 0 && I > 0 &&
                        H <= 2048 && I <= 2048,
               "bad MoE shape (H, I multiples of 32 up to 2048, nE <= 256)");
    const int64_t P = T * K;
    TB_REQUIRE(ctx, P <= (1 << 20), "too many (token, expert) pairs");
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    const size_t b_order = up(P * 4), b_off = up((nE + 1) * 4), b_act = up((nE + 1) * 4), b_swi = up(P * I * 4),
                 b_o = up(P * H * 4);
    char* scr = static_cast<char*>(tb_ctx_scratch(ctx, b_order + b_off + b_act + b_swi + b_o));
    if (!scr) return TB_ERR_NOMEM;
    int* order = reinterpret_cast<int*>(scr);
    int* offsets = reinterpret_cast<int*>(scr + b_order);
    int* active = reinterpret_cast<int*>(scr + b_order + b_off);     // [nE] then the count
    float* swi = reinterpret_cast<float*>(scr + b_order + b_off + b_act);
    float* o = reinterpret_cast<float*>(scr + b_order + b_off + b_act + b_swi);
    cudaError_t e = tb_launch(ctx, k_moe_group, dim3(1), dim3(256), 0, idx, (int)P, (int)nE, order, offsets, active,
                              active + nE, ctx->dev_error);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "moe group launch: %s", cudaGetErrorString(e));
    MoeArgs g{x_in, H, (int)K, {w1p, w3p}, {w1s, w3s}, swi, order, offsets, (int)I, (int)H, (int)(H / 32)};
    g.sg = group / 32;
    // fewer pairs than experts (decode): each routed expert's rows spread over
    // more CTAs, one row block each, for more weight bytes in flight
    g.bpc = P < nE ? 1 : MOE_BPC;
    // only the routed experts get CTAs (at most one slot per pair), and an expert
    // has at most T pairs (a token's top-k experts are distinct), which sizes the
    // staged activations
    g.active = active;
    g.nactive = active + nE;
    g.mb = (int)std::min<int64_t>(MB, T);
    const int nslots = (int)std::min<int64_t>(nE, P);
    int rc = launch_moe<MOE_GATEUP>(ctx, g, nslots);
    if (rc) return rc;
    MoeArgs d{swi, I, 1, {w2p, w2p}, {w2s, w2s}, o, order, offsets, (int)H, (int)I, (int)(I / 32)};
    d.sg = g.sg;
    d.bpc = g.bpc;
    d.active = g.active;
    d.nactive = g.nactive;
    d.mb = g.mb;
    rc = launch_moe<MOE_DOWN>(ctx, d, nslots);
    if (rc) return rc;
    const long long total = T * H;
    const int grid = (int)std::min<long long>((total + 255) / 256, (long long)ctx->num_sms * 8);
    e = tb_launch(ctx, k_moe_combine, dim3(grid), dim3(256), 0, x_out, (const float*)o, wt, (int)H, (int)K, total);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "moe combine launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_moe_ffn_int3(tb_ctx* ctx, float* x_out, const float* x_in, const uint32_t* idx, const float* wt,
                           const uint32_t* w1p, const uint16_t* w1s, const uint32_t* w3p, const uint16_t* w3s,
                           const uint32_t* w2p, const uint16_t* w2s, int64_t T, int64_t K, int64_t nE, int64_t H,
                           int64_t I)
{
    return tb_moe_ffn_int3_g(ctx, x_out, x_in, idx, wt, w1p, w1s, w3p, w3s, w2p, w2s, T, K, nE, H, I, 32);
}

TB_API int tb_quant_int3_bf16(tb_ctx* ctx, const uint16_t* w_bf16, uint32_t* p3, uint16_t* s3, int64_t rows,
                              int64_t K, int group)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, w_bf16 && p3 && s3, "null pointer");
    TB_REQUIRE(ctx, group == 32 || group == 128, "int3 scale group must be 32 or 128 (got %d)", group);
    TB_REQUIRE(ctx, rows > 0 && K > 0 && K % group == 0, "bad shape (K %% group must be 0)");
    const long long ng = rows * (K / group);
    const int grid = (int)std::min<long long>((ng * 32 + 255) / 256, (long long)ctx->num_sms * 16);
    cudaError_t e = tb_launch(ctx, k_quant_int3, dim3(grid), dim3(256), 0, w_bf16, p3, s3, ng, group / 32);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "quant_int3 launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

}  // extern "C"

// ============================================================================
// Expert parallelism: the MoE FFN over P ranks (one process and GPU each), nE/P
// experts per rank.  The reference keeps every expert on its one device
// (lfm25.js:824-830); the exchange below is this library's own.
//
// Each rank owns an exchange arena in its HBM, mapped into every other rank
// with CUDA IPC:
//   rows[P][Tmax][H]  f32   token rows sent here, region s written by rank s
//   meta[P][Tmax][K]  u32   per row and top-k slot: (local expert << 24) | origin
//                           pair t*K + k, or ~0 when that slot's expert is elsewhere
//   cnt[8], dflag[8], rflag[8]   u32 rows sent by / dispatch epoch of / return
//                           epoch of each rank; then cfg[6] (P, nE, K, H, I,
//                           Tmax), compared across ranks at connect
//   ret[Tmax*K][H]    f32   the expert outputs of this rank's own pairs, each
//                           written straight into its slot by the owner
// A forward (epoch e): dispatch stores every local token row once per rank
// that owns one of its experts (plain stores over NVLink), the last CTA per
// destination releases cnt + dflag there; the owner's plan kernel acquires all
// P dispatch flags and groups the received pairs by local expert; the grouped
// int3 GEMVs run (the down GEMV's epilogue writes each pair's output row into
// its origin's ret slot); a signal kernel releases rflag on every rank; the
// combine waits for all P owners and adds sum_k wt * o_k in k order -- the
// single-device arithmetic, so the result is bit-identical to tb_moe_ffn_int3.
// Buffers are reused without double buffering: rank s dispatches epoch e+1
// only after its combine of e saw every owner's return flag, which an owner
// releases after it finished reading epoch e's rows; an owner writes epoch
// e+1's outputs into s's ret only after s's dispatch of e+1, issued after s's
// combine of e.  Every wait is bounded (~1 s) and records an error on timeout.
namespace {

constexpr int EP_TMAX = 1024;
constexpr long long EP_WAIT_LIMIT = 1LL << 22;
constexpr int ERR_EP_WAIT = 0x6c10;
constexpr int ERR_EP_EXPERT = 0x6c11;
constexpr int EP_CFG_OFF = 3 * EP_MAX * 4;    // bytes into the flags block
constexpr int EP_CFG_WORDS = 6;

size_t ep_up(size_t v) { return (v + 255) & ~size_t(255); }

struct EpLayout {
    size_t rows, meta, flags, ret, total;
};
EpLayout ep_layout(int P, int64_t Tmax, int64_t K, int64_t H)
{
    EpLayout L{};
    L.rows = 0;
    L.meta = L.rows + ep_up((size_t)P * Tmax * H * 4);
    L.flags = L.meta + ep_up((size_t)P * Tmax * K * 4);
    L.ret = L.flags + ep_up(3 * EP_MAX * 4);
    L.total = L.ret + ep_up((size_t)Tmax * K * H * 4);
    return L;
}

__device__ __forceinline__ void ep_wait(const unsigned* flag, unsigned e, int* err)
{
    long long it = 0;
    while ((int)(ld_acquire_sys(flag) - e) < 0) {
        if (++it > EP_WAIT_LIMIT) {
            atomicExch(err, ERR_EP_WAIT);
            break;
        }
        if (it > 4096) __nanosleep(64);
    }
}

__device__ __forceinline__ unsigned ld_volatile_u32(const unsigned* p)
{
    unsigned v;
    asm volatile("ld.volatile.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct EpDispatchArgs {
    const float* x;                 // [T][H] this rank's token rows
    const uint32_t* idx;            // [T][K] routed experts (global ids)
    float* rows[EP_MAX];            // destination d: its rows region of this rank
    uint32_t* meta[EP_MAX];         // destination d: its meta region of this rank
    unsigned* cnt[EP_MAX];          // destination d: &cnt[this rank]
    unsigned* flag[EP_MAX];         // destination d: &dflag[this rank]
    unsigned* ctr;                  // [EP_MAX] CTA arrival counters (local, zero between calls)
    int T, K, H, El, nE;
    unsigned e;
    int* err;
};

// grid (P, NB): CTA (d, b) lists the tokens routed to rank d (one slot per
// token, in token order), copies the rows of slots b*8+w, b*8+w + 8*NB, ...
// (warp w) with their meta, and the last CTA of d publishes the count
__global__ void __launch_bounds__(256) k_ep_dispatch(const EpDispatchArgs a)
{
    __shared__ int slot_tok[EP_TMAX];
    __shared__ int wtot[8];
    tb_pdl_wait();
    tb_pdl_trigger();
    const int d = blockIdx.x, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int t0 = threadIdx.x * 4;
    unsigned m = 0;
    int c = 0;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int t = t0 + i;
        if (t >= a.T) break;
        bool in = false;
        for (int k = 0; k < a.K; k++) {
            const uint32_t ex = a.idx[(long long)t * a.K + k];
            if (ex >= (uint32_t)a.nE) {
                if (d == 0 && blockIdx.y == 0) atomicExch(a.err, ERR_EP_EXPERT);
            } else if ((int)(ex / (uint32_t)a.El) == d) {
                in = true;
            }
        }
        if (in) { m |= 1u << i; c++; }
    }
    // block exclusive scan of c
    int incl = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    if (lane == 31) wtot[w] = incl;
    __syncthreads();
    int before = 0, total = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        before += i < w ? wtot[i] : 0;
        total += wtot[i];
    }
    int j = before + incl - c;
#pragma unroll
    for (int i = 0; i < 4; i++)
        if (m & (1u << i)) slot_tok[j++] = t0 + i;
    __syncthreads();
    float* rows = a.rows[d];
    uint32_t* meta = a.meta[d];
    const int H4 = a.H >> 2;
    for (int s = blockIdx.y * 8 + w; s < total; s += gridDim.y * 8) {
        const int t = slot_tok[s];
        const float4* src = reinterpret_cast<const float4*>(a.x + (long long)t * a.H);
        float4* dst = reinterpret_cast<float4*>(rows + (long long)s * a.H);
        for (int i = lane; i < H4; i += 32) dst[i] = src[i];
        if (lane < a.K) {
            const uint32_t ex = a.idx[(long long)t * a.K + lane];
            const bool here = ex < (uint32_t)a.nE && (int)(ex / (uint32_t)a.El) == d;
            meta[(long long)s * a.K + lane] =
                here ? ((ex % (uint32_t)a.El) << 24) | (uint32_t)(t * a.K + lane) : 0xffffffffu;
        }
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned old = atomicAdd(a.ctr + d, 1u);
        if (old == gridDim.y - 1) {          // every CTA of d has fenced its stores
            a.ctr[d] = 0u;
            __threadfence_system();
            *reinterpret_cast<volatile unsigned*>(a.cnt[d]) = (unsigned)total;
            st_release_sys(a.flag[d], a.e);
        }
    }
}

struct EpPlanArgs {
    const uint32_t* meta;           // this rank's meta [P][Tmax][K]
    const unsigned* cnt;            // this rank's cnt[P]
    const unsigned* dflag;          // this rank's dflag[P]
    int* xrow;                      // [pairs] received row s*Tmax + j
    uint32_t* ydst;                 // [pairs] (origin rank << 24) | origin pair
    int* offsets;                   // [El + 1]
    int P, Tmax, K, El;
    unsigned e;
    int* err;
};

// one CTA: wait for every rank's dispatch, then place the received pairs
// grouped by local expert (positions within an expert in arrival order of the
// atomics: a pair's result does not depend on its position)
__global__ void __launch_bounds__(512) k_ep_plan(const EpPlanArgs a)
{
    __shared__ int ecnt[256], ecur[256];
    __shared__ unsigned scnt[EP_MAX];
    tb_pdl_wait();
    tb_pdl_trigger();
    if (threadIdx.x < a.P) {
        ep_wait(a.dflag + threadIdx.x, a.e, a.err);
        const unsigned n = ld_volatile_u32(a.cnt + threadIdx.x);
        scnt[threadIdx.x] = n <= (unsigned)a.Tmax ? n : 0u;
    }
    for (int i = threadIdx.x; i < a.El; i += blockDim.x) ecnt[i] = 0;
    __syncthreads();
    for (int s = 0; s < a.P; s++) {
        const int n = (int)scnt[s] * a.K;
        const uint32_t* ms = a.meta + (long long)s * a.Tmax * a.K;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const uint32_t code = ld_volatile_u32(ms + i);
            if (code != 0xffffffffu && (int)(code >> 24) < a.El) atomicAdd(&ecnt[code >> 24], 1);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int run = 0;
        for (int i = 0; i < a.El; i++) {
            a.offsets[i] = run;
            ecur[i] = run;
            run += ecnt[i];
        }
        a.offsets[a.El] = run;
    }
    __syncthreads();
    for (int s = 0; s < a.P; s++) {
        const int n = (int)scnt[s] * a.K;
        const uint32_t* ms = a.meta + (long long)s * a.Tmax * a.K;
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const uint32_t code = ld_volatile_u32(ms + i);
            if (code == 0xffffffffu || (int)(code >> 24) >= a.El) continue;
            const int pos = atomicAdd(&ecur[code >> 24], 1);
            a.xrow[pos] = s * a.Tmax + i / a.K;
            a.ydst[pos] = ((uint32_t)s << 24) | (code & 0xffffffu);
        }
    }
}

// after the down GEMV (griddepcontrol.wait: its stores are complete), release
// this rank's return flag on every rank
struct EpSignalArgs {
    unsigned* flag[EP_MAX];         // rank s: &rflag[this rank]
    int P;
    unsigned e;
};
__global__ void __launch_bounds__(32) k_ep_signal(const EpSignalArgs a)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    __threadfence_system();
    if ((int)threadIdx.x < a.P) st_release_sys(a.flag[threadIdx.x], a.e);
}

// x[t, :] += sum_k wt[t, k] * ret[t*K + k, :] (k in order, as k_moe_combine),
// after every owner's return flag
__global__ void __launch_bounds__(256) k_ep_combine(float* __restrict__ x, const float* ret, const float* __restrict__ wt,
                                                    const unsigned* rflag, int P, unsigned e, int H, int K, int total4,
                                                    int* err)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    if ((int)threadIdx.x < P) ep_wait(rflag + threadIdx.x, e, err);
    __syncthreads();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total4; i += gridDim.x * blockDim.x) {
        const int t = (4 * i) / H, h = 4 * i - t * H;
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k = 0; k < K; k++) {
            const float wk = wt[t * K + k];
            const float4 o = ld_volatile_f4(ret + (long long)(t * K + k) * H + h);
            s.x = fmaf(wk, o.x, s.x);
            s.y = fmaf(wk, o.y, s.y);
            s.z = fmaf(wk, o.z, s.z);
            s.w = fmaf(wk, o.w, s.w);
        }
        float4 v = reinterpret_cast<float4*>(x)[i];
        v.x += s.x; v.y += s.y; v.z += s.z; v.w += s.w;
        reinterpret_cast<float4*>(x)[i] = v;
    }
}

}  // namespace

struct tb_moe_ep {
    tb_ctx* ctx = nullptr;
    int P = 1, r = 0;
    int64_t nE = 0, El = 0, K = 0, H = 0, I = 0, Tmax = 0;
    EpLayout L{};
    char* arena = nullptr;
    char* peer[EP_MAX] = {};
    bool connected = false;
    float* swi = nullptr;
    int* xrow = nullptr;
    uint32_t* ydst = nullptr;
    int* offsets = nullptr;
    unsigned* ctr = nullptr;
    const uint32_t* wp[3] = {};
    const uint16_t* ws[3] = {};
    unsigned epoch = 0;
};

namespace {

void ep_free(tb_moe_ep* m)
{
    for (int s = 0; s < m->P; s++)
        if (s != m->r && m->peer[s]) cudaIpcCloseMemHandle(m->peer[s]);
    for (void* p : {(void*)m->arena, (void*)m->swi, (void*)m->xrow, (void*)m->ydst, (void*)m->offsets, (void*)m->ctr})
        if (p) cudaFree(p);
}

}  // namespace

extern "C" {

TB_API int tb_moe_ep_create(tb_ctx* ctx, int P, int rank, int64_t nE, int64_t K, int64_t H, int64_t I, int64_t Tmax,
                            tb_moe_ep** out)
{
    if (!ctx || !out) return TB_ERR_INVALID;
    *out = nullptr;
    TB_REQUIRE(ctx, P >= 1 && P <= EP_MAX && rank >= 0 && rank < P, "moe ep: %d ranks (1..%d), rank %d", P, EP_MAX,
               rank);
    TB_REQUIRE(ctx, nE > 0 && nE % P == 0 && nE / P <= 256, "moe ep: %lld experts over %d ranks", (long long)nE, P);
    TB_REQUIRE(ctx, K >= 1 && K <= 8 && K <= nE, "moe ep: top-k %lld (1..8)", (long long)K);
    TB_REQUIRE(ctx, H > 0 && I > 0 && H % 32 == 0 && I % 32 == 0 && H <= 2048 && I <= 2048,
               "moe ep: H, I multiples of 32 up to 2048");
    TB_REQUIRE(ctx, Tmax >= 1 && Tmax <= EP_TMAX, "moe ep: up to %d tokens per rank and call", EP_TMAX);
    tb_moe_ep* m = new tb_moe_ep;
    m->ctx = ctx; m->P = P; m->r = rank; m->nE = nE; m->El = nE / P; m->K = K; m->H = H; m->I = I; m->Tmax = Tmax;
    m->L = ep_layout(P, Tmax, K, H);
    const int64_t pairs = (int64_t)P * Tmax * K;     // at most K codes per received row
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ctx->device);
    cudaError_t e = cudaMalloc(&m->arena, m->L.total);
    if (e == cudaSuccess) e = cudaMemset(m->arena, 0, m->L.total);
    if (e == cudaSuccess) e = cudaMalloc(&m->swi, (size_t)pairs * I * 4);
    if (e == cudaSuccess) e = cudaMalloc(&m->xrow, (size_t)pairs * 4);
    if (e == cudaSuccess) e = cudaMalloc(&m->ydst, (size_t)pairs * 4);
    if (e == cudaSuccess) e = cudaMalloc(&m->offsets, (size_t)(m->El + 1) * 4);
    if (e == cudaSuccess) e = cudaMalloc(&m->ctr, EP_MAX * 4);
    if (e == cudaSuccess) e = cudaMemset(m->ctr, 0, EP_MAX * 4);
    const uint32_t cfg[EP_CFG_WORDS] = {(uint32_t)P, (uint32_t)nE, (uint32_t)K, (uint32_t)H, (uint32_t)I, (uint32_t)Tmax};
    if (e == cudaSuccess)
        e = cudaMemcpy(m->arena + m->L.flags + EP_CFG_OFF, cfg, sizeof cfg, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        ep_free(m);
        delete m;
        return tb_fail(ctx, TB_ERR_NOMEM, "moe ep buffers: %s", cudaGetErrorString(e));
    }
    m->peer[rank] = m->arena;
    m->connected = P == 1;
    *out = m;
    return TB_OK;
}

TB_API void tb_moe_ep_destroy(tb_moe_ep* m)
{
    if (!m) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    ep_free(m);
    cudaSetDevice(prev);
    delete m;
}

TB_API int tb_moe_ep_handle(tb_moe_ep* m, void* out64)
{
    if (!m || !out64) return TB_ERR_INVALID;
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, m->arena);
    if (e != cudaSuccess) return tb_fail(m->ctx, TB_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    memcpy(out64, &h, sizeof h);
    return TB_OK;
}

TB_API int tb_moe_ep_connect(tb_moe_ep* m, const void* handles)
{
    if (!m || !handles) return TB_ERR_INVALID;
    tb_ctx* ctx = m->ctx;
    TB_REQUIRE(ctx, m->P > 1 && !m->connected, "moe ep connect: single rank or already connected");
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ctx->device);
    int rc = TB_OK;
    for (int s = 0; s < m->P && rc == TB_OK; s++) {
        if (s == m->r) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char*>(handles) + 64 * s, sizeof h);
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            rc = tb_fail(ctx, TB_ERR_CUDA, "cudaIpcOpenMemHandle(rank %d): %s", s, cudaGetErrorString(e));
            break;
        }
        m->peer[s] = static_cast<char*>(p);
        // every rank must lay out its arena with the same sizes
        uint32_t mine[EP_CFG_WORDS], theirs[EP_CFG_WORDS];
        e = cudaMemcpy(mine, m->arena + m->L.flags + EP_CFG_OFF, sizeof mine, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(theirs, m->peer[s] + m->L.flags + EP_CFG_OFF, sizeof theirs, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) rc = tb_fail(ctx, TB_ERR_CUDA, "moe ep connect: reading rank %d: %s", s, cudaGetErrorString(e));
        else if (memcmp(mine, theirs, sizeof mine) != 0)
            rc = tb_fail(ctx, TB_ERR_INVALID, "moe ep connect: rank %d was created with other sizes (P, nE, K, H, I, Tmax)", s);
    }
    cudaSetDevice(prev);
    if (rc != TB_OK) {
        for (int s = 0; s < m->P; s++)
            if (s != m->r && m->peer[s]) { cudaIpcCloseMemHandle(m->peer[s]); m->peer[s] = nullptr; }
        return rc;
    }
    m->connected = true;
    return TB_OK;
}

TB_API int tb_moe_ep_set_experts(tb_moe_ep* m, const uint32_t* w1p, const uint16_t* w1s, const uint32_t* w3p,
                                 const uint16_t* w3s, const uint32_t* w2p, const uint16_t* w2s)
{
    if (!m) return TB_ERR_INVALID;
    TB_REQUIRE(m->ctx, w1p && w1s && w3p && w3s && w2p && w2s, "null pointer");
    m->wp[0] = w1p; m->ws[0] = w1s; m->wp[1] = w3p; m->ws[1] = w3s; m->wp[2] = w2p; m->ws[2] = w2s;
    return TB_OK;
}

TB_API int tb_moe_ep_forward(tb_moe_ep* m, float* x_out, const float* x_in, const uint32_t* idx, const float* wt,
                             int64_t T)
{
    if (!m) return TB_ERR_INVALID;
    tb_ctx* ctx = m->ctx;
    TB_REQUIRE(ctx, x_out && x_in && idx && wt, "null pointer");
    TB_REQUIRE(ctx, m->connected, "moe ep: connect the ranks first (tb_moe_ep_connect)");
    TB_REQUIRE(ctx, m->wp[0], "moe ep: experts not set");
    TB_REQUIRE(ctx, T >= 1 && T <= m->Tmax, "moe ep: %lld tokens (1..%lld)", (long long)T, (long long)m->Tmax);
    TB_REQUIRE(ctx, TB_ALIGNED(x_out, 16) && TB_ALIGNED(x_in, 16), "moe ep: x rows must be 16-byte aligned");
    const unsigned e = ++m->epoch;
    const int P = m->P, r = m->r;
    EpDispatchArgs da{};
    for (int d = 0; d < P; d++) {
        char* b = m->peer[d];
        da.rows[d] = reinterpret_cast<float*>(b + m->L.rows) + (size_t)r * m->Tmax * m->H;
        da.meta[d] = reinterpret_cast<uint32_t*>(b + m->L.meta) + (size_t)r * m->Tmax * m->K;
        unsigned* fl = reinterpret_cast<unsigned*>(b + m->L.flags);
        da.cnt[d] = fl + r;
        da.flag[d] = fl + EP_MAX + r;
    }
    da.x = x_in; da.idx = idx; da.ctr = m->ctr; da.T = (int)T; da.K = (int)m->K; da.H = (int)m->H;
    da.El = (int)m->El; da.nE = (int)m->nE; da.e = e; da.err = ctx->dev_error;
    const int NB = std::min(16, tb_cdiv(T, 8));
    cudaError_t ce = tb_launch(ctx, k_ep_dispatch, dim3((unsigned)P, (unsigned)NB), dim3(256), 0, da);
    if (ce != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "moe ep dispatch launch: %s", cudaGetErrorString(ce));
    unsigned* myfl = reinterpret_cast<unsigned*>(m->arena + m->L.flags);
    EpPlanArgs pa{reinterpret_cast<const uint32_t*>(m->arena + m->L.meta), myfl, myfl + EP_MAX, m->xrow, m->ydst,
                  m->offsets, P, (int)m->Tmax, (int)m->K, (int)m->El, e, ctx->dev_error};
    ce = tb_launch(ctx, k_ep_plan, dim3(1), dim3(512), 0, pa);
    if (ce != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "moe ep plan launch: %s", cudaGetErrorString(ce));
    const int H = (int)m->H, I = (int)m->I;
    MoeArgs g{reinterpret_cast<const float*>(m->arena + m->L.rows), H, 1, {m->wp[0], m->wp[1]}, {m->ws[0], m->ws[1]},
              m->swi, nullptr, m->offsets, I, H, H / 32};
    g.xrow = m->xrow;
    g.bpc = T * m->K < m->nE ? 1 : MOE_BPC;
    int rc = launch_moe<MOE_GATEUP>(ctx, g, (int)m->El);
    if (rc) return rc;
    MoeArgs dn{m->swi, I, 1, {m->wp[2], m->wp[2]}, {m->ws[2], m->ws[2]}, nullptr, nullptr, m->offsets, H, I, I / 32};
    dn.ydst = m->ydst;
    dn.bpc = g.bpc;
    for (int s = 0; s < P; s++) dn.ypeer[s] = reinterpret_cast<float*>(m->peer[s] + m->L.ret);
    rc = launch_moe<MOE_DOWN>(ctx, dn, (int)m->El);
    if (rc) return rc;
    EpSignalArgs sa{};
    for (int s = 0; s < P; s++) sa.flag[s] = reinterpret_cast<unsigned*>(m->peer[s] + m->L.flags) + 2 * EP_MAX + r;
    sa.P = P;
    sa.e = e;
    ce = tb_launch(ctx, k_ep_signal, dim3(1), dim3(32), 0, sa);
    if (ce != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "moe ep signal launch: %s", cudaGetErrorString(ce));
    const int total4 = (int)(T * m->H / 4);
    const int grid = std::max(1, std::min(tb_cdiv(total4, 256), ctx->num_sms));
    ce = tb_launch(ctx, k_ep_combine, dim3((unsigned)grid), dim3(256), 0, x_out,
                   (const float*)(m->arena + m->L.ret), wt, (const unsigned*)(myfl + 2 * EP_MAX), P, e, H, (int)m->K,
                   total4, ctx->dev_error);
    if (ce != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "moe ep combine launch: %s", cudaGetErrorString(ce));
    return TB_OK;
}

}  // extern "C"
