// tb_attn_prefill.cu -- int8-KV prefill attention: T queries (positions
// S-T .. S-1) over S cached keys with the causal mask, GQA.
//
// Reference: attentionQ8 at T > 1 (models/qwen3.js:2534-2577), the flash
// kernels ATTN_WGSL / attnF16Wgsl whose K/V tile loads dequantize the per-32
// snorm int8 cache while staging: v = max(c/127, -1) * group scale; scores
// q.k / sqrt(hd) masked to keys <= the query's position; online softmax; out =
// sum p v / sum p.
//
// B200 design.  One CTA (8 warps) per (query tile, kv head): warp w serves q
// head hk*GRP + w / (8/GRP) and 16 consecutive queries, so every q head of the
// GQA group shares each dequantized K/V tile.  Per 64-key tile the CTA loads
// the int8 rows (16-byte loads, issued before the previous tile's math so they
// overlap it), dequantizes them to f16 in shared memory (rows padded to break
// bank conflicts), and each warp runs S = Q K^T and O += P V on the tensor
// cores (mma.sync m16n8k16, f16 operands, f32 accumulators) with ldmatrix
// fragment loads; P stays in registers between the two products.  Softmax in
// f32 with exp2 (log2 e folded into the score scale).  Tiles wholly above a
// query tile's diagonal are skipped; heavy (late) query tiles are scheduled
// first.  Differences from the reference's f32 kernel: Q, K, V and P rounded
// to f16 (2^-11), sums in f32 -- the reference's f16 kernel also rounds them,
// and sums in f16.
#include "tb_internal.h"

namespace {

constexpr int NW = 8, THREADS = NW * 32, KT = 64;

struct PrefArgs {
    const float* q;      // [T][nHq*HD]
    const int8_t* Kq;    // [S][nKv*HD]
    const float* Ks;     // [S][nKv*HD/32]
    const int8_t* Vq;
    const float* Vs;
    float* out;          // [T][nHq*HD]
    int T, S, nHq, nKv;
    float sl2;           // log2(e) / sqrt(HD)
};

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi)
{
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t* r, const void* p)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t* r, const void* p)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}

// int8 snorm -> float, WGSL unpack4x8snorm: max(c / 127, -1)
__device__ __forceinline__ float snorm(int c) { return fmaxf((float)c * (1.0f / 127.0f), -1.0f); }

// 16 int8 (one uint4) times a group scale -> 16 f16 (two uint4)
__device__ __forceinline__ void dequant16(uint4 v, float s, uint4& o0, uint4& o1)
{
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t h[8];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int b0 = (int)(int8_t)(w[i] & 0xff), b1 = (int)(int8_t)((w[i] >> 8) & 0xff);
        const int b2 = (int)(int8_t)((w[i] >> 16) & 0xff), b3 = (int)(int8_t)(w[i] >> 24);
        h[2 * i] = pack_h2(snorm(b0) * s, snorm(b1) * s);
        h[2 * i + 1] = pack_h2(snorm(b2) * s, snorm(b3) * s);
    }
    o0 = make_uint4(h[0], h[1], h[2], h[3]);
    o1 = make_uint4(h[4], h[5], h[6], h[7]);
}

template <int HD, int GRP>
__global__ void __launch_bounds__(THREADS) k_attn_prefill(const PrefArgs a)
{
    constexpr int WPH = NW / GRP;          // warps per q head
    constexpr int QT = WPH * 16;           // queries per CTA
    constexpr int RS = HD + 8;             // smem row stride (f16): 16-byte aligned, conflict-free ldmatrix
    constexpr int CPR = HD / 16;           // 16-byte int8 chunks per key row
    constexpr int CPT = KT * CPR / THREADS;  // chunks per thread per tile (K and V each)
    static_assert(KT * CPR % THREADS == 0, "tile split");
    __shared__ __align__(16) __half ksm[KT * RS];
    __shared__ __align__(16) __half vsm[KT * RS];

    const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int hk = blockIdx.y;
    const int qtile = gridDim.x - 1 - blockIdx.x;          // late (heavy) tiles first
    const int hq = hk * GRP + w / WPH;
    const int q0 = qtile * QT + (w % WPH) * 16;             // this warp's first query
    const int off = a.S - a.T;                              // position of query 0
    const int kvrow = a.nKv * HD, kvg = kvrow / 32, qrow = a.nHq * HD;

    tb_pdl_wait();
    tb_pdl_trigger();

    // Q fragments (A operand, row-major 16 x HD), f16, kept in registers
    uint32_t qf[HD / 16][4];
    {
        const int r0 = q0 + g, r1 = q0 + g + 8;
        const float* p0 = a.q + (size_t)r0 * qrow + hq * HD;
        const float* p1 = a.q + (size_t)r1 * qrow + hq * HD;
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
            const int c = 16 * kk + 2 * t;
            float2 x00 = make_float2(0.f, 0.f), x10 = x00, x01 = x00, x11 = x00;
            if (r0 < a.T) { x00 = *reinterpret_cast<const float2*>(p0 + c); x01 = *reinterpret_cast<const float2*>(p0 + c + 8); }
            if (r1 < a.T) { x10 = *reinterpret_cast<const float2*>(p1 + c); x11 = *reinterpret_cast<const float2*>(p1 + c + 8); }
            qf[kk][0] = pack_h2(x00.x, x00.y);
            qf[kk][1] = pack_h2(x10.x, x10.y);
            qf[kk][2] = pack_h2(x01.x, x01.y);
            qf[kk][3] = pack_h2(x11.x, x11.y);
        }
    }
    float o[HD / 8][4];
#pragma unroll
    for (int i = 0; i < HD / 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    // keys any query of this CTA can see
    const int qlast = min(qtile * QT + QT, a.T) - 1;
    const int kend = min(a.S, off + qlast + 1);
    const int wq_last = min(q0 + 15, a.T - 1);              // this warp's last real query
    const int wkend = off + wq_last + 1;

    // raw int8 tile in registers: chunk (key, part) of K and of V, plus scales
    uint4 rk[CPT], rv[CPT];
    float sk[CPT], sv[CPT];
    auto fetch = [&](int k0) {
#pragma unroll
        for (int i = 0; i < CPT; i++) {
            const int c = i * THREADS + tid, key = c / CPR, part = c % CPR, gk = k0 + key;
            if (gk < a.S) {
                const size_t ro = (size_t)gk * kvrow + hk * HD + part * 16;
                const size_t so = (size_t)gk * kvg + hk * (HD / 32) + part / 2;
                rk[i] = __ldg(reinterpret_cast<const uint4*>(a.Kq + ro));
                rv[i] = __ldg(reinterpret_cast<const uint4*>(a.Vq + ro));
                sk[i] = __ldg(a.Ks + so);
                sv[i] = __ldg(a.Vs + so);
            } else {
                rk[i] = rv[i] = make_uint4(0, 0, 0, 0);
                sk[i] = sv[i] = 0.f;
            }
        }
    };
    auto stage = [&]() {
#pragma unroll
        for (int i = 0; i < CPT; i++) {
            const int c = i * THREADS + tid, key = c / CPR, part = c % CPR;
            uint4 a0, a1;
            dequant16(rk[i], sk[i], a0, a1);
            *reinterpret_cast<uint4*>(ksm + key * RS + part * 16) = a0;
            *reinterpret_cast<uint4*>(ksm + key * RS + part * 16 + 8) = a1;
            dequant16(rv[i], sv[i], a0, a1);
            *reinterpret_cast<uint4*>(vsm + key * RS + part * 16) = a0;
            *reinterpret_cast<uint4*>(vsm + key * RS + part * 16 + 8) = a1;
        }
    };

    if (kend > 0) fetch(0);
    for (int k0 = 0; k0 < kend; k0 += KT) {
        __syncthreads();          // the previous tile's fragments are consumed
        stage();
        __syncthreads();
        if (k0 + KT < kend) fetch(k0 + KT);   // next tile's loads fly during this tile's math
        if (k0 >= wkend) continue;            // wholly above this warp's diagonal
        // ---- S = Q K^T : 16 queries x 64 keys
        float s[KT / 8][4];
#pragma unroll
        for (int j = 0; j < KT / 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < HD / 16; kk++) {
#pragma unroll
            for (int jp = 0; jp < KT / 16; jp++) {
                // keys 16jp..16jp+15, dims 16kk..16kk+15: B fragments of n-tiles 2jp, 2jp+1
                uint32_t b[4];
                const int key = 16 * jp + (lane & 7) + (lane >> 4) * 8, dim = 16 * kk + ((lane >> 3) & 1) * 8;
                ldsm_x4(b, ksm + key * RS + dim);
                mma16816(s[2 * jp], qf[kk], b[0], b[1]);
                mma16816(s[2 * jp + 1], qf[kk], b[2], b[3]);
            }
        }
        // ---- mask, online softmax (rows g and g+8 of the warp's 16)
        const int p0 = off + q0 + g, p1 = p0 + 8;   // positions of the two rows
        const bool diag = k0 + KT - 1 > off + q0;   // some key of the tile beyond some row's position
        float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
        for (int j = 0; j < KT / 8; j++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int gk = k0 + 8 * j + 2 * t + e;
                float v0 = s[j][e] * a.sl2, v1 = s[j][2 + e] * a.sl2;
                if (diag || gk >= a.S) {
                    if (gk > p0 || gk >= a.S) v0 = -INFINITY;
                    if (gk > p1 || gk >= a.S) v1 = -INFINITY;
                }
                s[j][e] = v0;
                s[j][2 + e] = v1;
                mx0 = fmaxf(mx0, v0);
                mx1 = fmaxf(mx1, v1);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        // a row whose keys so far are all masked keeps max -inf: no correction, p = 0
        const float c0 = mn0 == -INFINITY ? 1.f : exp2f(m0 - mn0), c1 = mn1 == -INFINITY ? 1.f : exp2f(m1 - mn1);
        const float b0 = mn0 == -INFINITY ? 0.f : mn0, b1 = mn1 == -INFINITY ? 0.f : mn1;
        m0 = mn0;
        m1 = mn1;
        l0 *= c0;
        l1 *= c1;
#pragma unroll
        for (int i = 0; i < HD / 8; i++) {
            o[i][0] *= c0; o[i][1] *= c0;
            o[i][2] *= c1; o[i][3] *= c1;
        }
        uint32_t pf[KT / 16][4];   // P as A fragments (keys = k dimension)
#pragma unroll
        for (int j = 0; j < KT / 8; j++) {
            const float e0 = exp2f(s[j][0] - b0), e1 = exp2f(s[j][1] - b0);
            const float e2 = exp2f(s[j][2] - b1), e3 = exp2f(s[j][3] - b1);
            l0 += e0 + e1;
            l1 += e2 + e3;
            pf[j >> 1][(j & 1) * 2 + 0] = pack_h2(e0, e1);
            pf[j >> 1][(j & 1) * 2 + 1] = pack_h2(e2, e3);
        }
        // ---- O += P V : 16 queries x HD dims over 64 keys
#pragma unroll
        for (int kk = 0; kk < KT / 16; kk++) {
#pragma unroll
            for (int np = 0; np < HD / 16; np++) {
                uint32_t b[4];
                const int key = 16 * kk + (lane & 7) + ((lane >> 3) & 1) * 8, dim = 16 * np + (lane >> 4) * 8;
                ldsm_x4_t(b, vsm + key * RS + dim);
                mma16816(o[2 * np], pf[kk], b[0], b[1]);
                mma16816(o[2 * np + 1], pf[kk], b[2], b[3]);
            }
        }
    }
    // ---- normalise and store
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
    const int r0 = q0 + g, r1 = q0 + g + 8;
#pragma unroll
    for (int i = 0; i < HD / 8; i++) {
        const int d = 8 * i + 2 * t;
        if (r0 < a.T)
            *reinterpret_cast<float2*>(a.out + (size_t)r0 * qrow + hq * HD + d) = make_float2(o[i][0] * i0, o[i][1] * i0);
        if (r1 < a.T)
            *reinterpret_cast<float2*>(a.out + (size_t)r1 * qrow + hq * HD + d) = make_float2(o[i][2] * i1, o[i][3] * i1);
    }
}

template <int HD, int GRP>
int launch(tb_ctx* ctx, const PrefArgs& a)
{
    constexpr int QT = (NW / GRP) * 16;
    const dim3 grid((unsigned)tb_cdiv(a.T, QT), (unsigned)a.nKv);
    cudaError_t e = tb_launch(ctx, k_attn_prefill<HD, GRP>, grid, dim3(THREADS), 0, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "attn_prefill launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

template <int HD>
int launch_grp(tb_ctx* ctx, const PrefArgs& a, int grp)
{
    switch (grp) {
    case 1: return launch<HD, 1>(ctx, a);
    case 2: return launch<HD, 2>(ctx, a);
    case 4: return launch<HD, 4>(ctx, a);
    case 8: return launch<HD, 8>(ctx, a);
    }
    return tb_fail(ctx, TB_ERR_UNSUPPORTED, "attn_prefill: n_heads / n_kv_heads must be 1, 2, 4 or 8");
}

}  // namespace

extern "C" TB_API int tb_attn_prefill_q8(tb_ctx* ctx, float* out, const float* q, const int8_t* Kq, const float* Ks,
                                         const int8_t* Vq, const float* Vs, int64_t T, int64_t S, int64_t nHq,
                                         int64_t nKv, int64_t hd)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, out && q && Kq && Ks && Vq && Vs, "null pointer");
    TB_REQUIRE(ctx, T >= 1 && T <= S && S < (1LL << 30), "attn_prefill: need 1 <= T <= S (T=%lld S=%lld)",
               (long long)T, (long long)S);
    TB_REQUIRE(ctx, nKv >= 1 && nHq % nKv == 0 && nKv <= 65535, "attn_prefill: bad head counts");
    TB_REQUIRE(ctx, hd == 64 || hd == 128, "attn_prefill: head_dim must be 64 or 128");
    TB_REQUIRE(ctx, TB_ALIGNED(q, 8) && TB_ALIGNED(out, 8) && TB_ALIGNED(Kq, 16) && TB_ALIGNED(Vq, 16) &&
                        TB_ALIGNED(Ks, 4) && TB_ALIGNED(Vs, 4),
               "attn_prefill: q/out 8-byte, Kq/Vq 16-byte, scales 4-byte aligned");
    PrefArgs a{q, Kq, Ks, Vq, Vs, out, (int)T, (int)S, (int)nHq, (int)nKv, 0.f};
    a.sl2 = 1.4426950408889634f / sqrtf((float)hd);
    const int grp = (int)(nHq / nKv);
    return hd == 64 ? launch_grp<64>(ctx, a, grp) : launch_grp<128>(ctx, a, grp);
}
