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
constexpr int MOE_BPC = 4;     // row blocks per CTA (weights of the next one in flight)
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
// one CTA: offsets[e] = first position of expert e in `order`, offsets[nE] = P
__global__ void __launch_bounds__(256) k_moe_group(const uint32_t* __restrict__ idx, int P, int nE,
                                                   int* __restrict__ order, int* __restrict__ offsets, int* err)
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
        for (int e = 0; e < nE; e++) cnt[e + 1] += cnt[e];
        for (int e = 0; e <= nE; e++) offsets[e] = cnt[e];
        // stable placement in pair order
        for (int p = 0; p < P; p++) {
            const uint32_t e = idx[p];
            if (e < (uint32_t)nE) order[cnt[e]++] = p;
        }
    }
}

// ---- grouped int3 expert GEMV ---------------------------------------------------
enum { MOE_GATEUP = 0, MOE_DOWN = 1 };

struct MoeArgs {
    const float* x;              // activation rows
    long long x_stride;          // floats between activation rows
    int xdiv;                    // pair p reads activation row p / xdiv (K for gate/up, 1 for down)
    const uint32_t* p3[2];       // [E*N][G][3]
    const uint16_t* s3[2];       // [E*N][G]
    float* y;                    // [P][N]: swi (gate/up) or expert outputs (down)
    const int* order;
    const int* offsets;
    int N, Kc, G;
};

// 32 weights (q3 + 4 in three bitplanes) of one group as floats q - 4
__device__ __forceinline__ void decode32(uint32_t b0, uint32_t b1, uint32_t b2, float* q)
{
#pragma unroll
    for (int j = 0; j < 8; j++) {
        // spread the 4 bits of each plane's nibble j into the low bit of 4 bytes
        const uint32_t n0 = ((b0 >> (4 * j)) & 15u) * 0x00204081u & 0x01010101u;
        const uint32_t n1 = ((b1 >> (4 * j)) & 15u) * 0x00204081u & 0x01010101u;
        const uint32_t n2 = ((b2 >> (4 * j)) & 15u) * 0x00204081u & 0x01010101u;
        const uint32_t v = n0 | (n1 << 1) | (n2 << 2);   // 4 bytes, each q3 + 4 in 0..7
#pragma unroll
        for (int k = 0; k < 4; k++)
            q[4 * j + k] = __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7540 + k)) - 8388612.0f;   // 2^23 + 4
    }
}

template <int KIND>
__global__ void __launch_bounds__(MOE_THREADS) k_moe_gemv3(const MoeArgs a)
{
    constexpr int NM = KIND == MOE_GATEUP ? 2 : 1;
    constexpr int RPW = moe_rpw<KIND>();
    extern __shared__ __align__(16) float xs[];   // [MB][G][XS_PAD]: xs[b][g][i] = x_b[32 g + i]
    tb_pdl_wait();
    tb_pdl_trigger();
    const int e = blockIdx.y;
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
        const int rw0 = (blockIdx.x * MOE_BPC + blk) * moe_rb<KIND>() + wid * RPW;
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
                    d.s[j][t][m] = ok ? tb_h2f(__ldg(a.s3[m] + row * G + (ok ? g : 0))) : 0.0f;
                }
    };
    for (int c0 = 0; c0 < np; c0 += MB) {
        const int nb = min(MB, np - c0);
        W cur, nxt;
        fetch(0, cur);                       // in flight while the activations are staged
        __syncthreads();                     // the previous chunk's reads are done
        for (int b = 0; b < nb; b++) {
            const int p = a.order[p0 + c0 + b];
            const float* src = a.x + (long long)(p / a.xdiv) * a.x_stride;
            for (int k = threadIdx.x; k < a.Kc; k += MOE_THREADS)
                xs[(b * G + (k >> 5)) * XS_PAD + (k & 31)] = src[k];
        }
        __syncthreads();
        for (int blk = 0; blk < MOE_BPC; blk++) {
            if (blk + 1 < MOE_BPC) fetch(blk + 1, nxt);
            const int rw0 = (blockIdx.x * MOE_BPC + blk) * moe_rb<KIND>() + wid * RPW;
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
#pragma unroll
                    for (int j = 0; j < RPW; j++)
#pragma unroll
                        for (int m = 0; m < NM; m++) {
                            float q[32];
                            decode32(cur.w[j][t][m][0], cur.w[j][t][m][1], cur.w[j][t][m][2], q);
#pragma unroll
                            for (int b = 0; b < MB; b++) {
                                if (b < nb) {
                                    const float4* xb = reinterpret_cast<const float4*>(xs + (b * G + g) * XS_PAD);
                                    float sum = 0.0f;
#pragma unroll
                                    for (int i4 = 0; i4 < 8; i4++) {
                                        const float4 xv = xb[i4];
                                        sum = fmaf(q[4 * i4], xv.x, sum);
                                        sum = fmaf(q[4 * i4 + 1], xv.y, sum);
                                        sum = fmaf(q[4 * i4 + 2], xv.z, sum);
                                        sum = fmaf(q[4 * i4 + 3], xv.w, sum);
                                    }
                                    acc[m][j][b] = fmaf(cur.s[j][t][m], sum, acc[m][j][b]);
                                }
                            }
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
                        const int p = a.order[p0 + c0 + b];
                        float v;
                        if (KIND == MOE_GATEUP) {
                            const float gg = acc[0][j][b], u = acc[NM - 1][j][b];
                            v = __fdiv_rn(gg, 1.0f + expf(-gg)) * u;      // silu(gate) * up
                        } else {
                            v = acc[0][j][b];
                        }
                        a.y[(long long)p * a.N + r] = v;
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

size_t moe_smem(int Kc) { return (size_t)MB * (Kc / 32) * XS_PAD * sizeof(float); }

template <int KIND>
int launch_moe(tb_ctx* ctx, const MoeArgs& a, int nE)
{
    const size_t smem = moe_smem(a.Kc);
    TB_REQUIRE(ctx, a.G <= 32 * MOE_GPL, "moe: K = %d above %d", a.Kc, 32 * 32 * MOE_GPL);
    TB_REQUIRE(ctx, smem <= 200 * 1024, "moe: K = %d too large for the staged activations", a.Kc);
    cudaError_t e = cudaFuncSetAttribute(k_moe_gemv3<KIND>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
        e = tb_launch(ctx, k_moe_gemv3<KIND>, dim3((unsigned)tb_cdiv(a.N, moe_rb<KIND>() * MOE_BPC), (unsigned)nE),
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
TB_API int tb_moe_ffn_int3(tb_ctx* ctx, float* x_out, const float* x_in, const uint32_t* idx, const float* wt,
                           const uint32_t* w1p, const uint16_t* w1s, const uint32_t* w3p, const uint16_t* w3s,
                           const uint32_t* w2p, const uint16_t* w2s, int64_t T, int64_t K, int64_t nE, int64_t H,
                           int64_t I)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, x_out && x_in && idx && wt && w1p && w1s && w3p && w3s && w2p && w2s, "null pointer");
    TB_REQUIRE(ctx, T > 0 && K > 0 && nE > 0 && nE <= 256 && H % 32 == 0 && I % 32 == 0 && H > 0 && I > 0 &&
                        H <= 2048 && I <= 2048,
               "bad MoE shape (H, I multiples of 32 up to 2048, nE <= 256)");
    const int64_t P = T * K;
    TB_REQUIRE(ctx, P <= (1 << 20), "too many (token, expert) pairs");
    auto up = [](size_t v) { return (v + 255) & ~size_t(255); };
    const size_t b_order = up(P * 4), b_off = up((nE + 1) * 4), b_swi = up(P * I * 4), b_o = up(P * H * 4);
    char* scr = static_cast<char*>(tb_ctx_scratch(ctx, b_order + b_off + b_swi + b_o));
    if (!scr) return TB_ERR_NOMEM;
    int* order = reinterpret_cast<int*>(scr);
    int* offsets = reinterpret_cast<int*>(scr + b_order);
    float* swi = reinterpret_cast<float*>(scr + b_order + b_off);
    float* o = reinterpret_cast<float*>(scr + b_order + b_off + b_swi);
    cudaError_t e = tb_launch(ctx, k_moe_group, dim3(1), dim3(256), 0, idx, (int)P, (int)nE, order, offsets,
                              ctx->dev_error);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "moe group launch: %s", cudaGetErrorString(e));
    MoeArgs g{x_in, H, (int)K, {w1p, w3p}, {w1s, w3s}, swi, order, offsets, (int)I, (int)H, (int)(H / 32)};
    int rc = launch_moe<MOE_GATEUP>(ctx, g, (int)nE);
    if (rc) return rc;
    MoeArgs d{swi, I, 1, {w2p, w2p}, {w2s, w2s}, o, order, offsets, (int)H, (int)I, (int)(I / 32)};
    rc = launch_moe<MOE_DOWN>(ctx, d, (int)nE);
    if (rc) return rc;
    const long long total = T * H;
    const int grid = (int)std::min<long long>((total + 255) / 256, (long long)ctx->num_sms * 8);
    e = tb_launch(ctx, k_moe_combine, dim3(grid), dim3(256), 0, x_out, (const float*)o, wt, (int)H, (int)K, total);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "moe combine launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

}  // extern "C"
