// tb_gemm_dp4.cu -- the prefill GEMM with the reference's integer semantics:
// gemmDP4A (int4 weights) and gemmTern (ternary WebGPU layout), models/qwen3.js
// gemmdp4Wgsl :1321-1407 and gemmTern :1410-1420.
//
// y[m][n] (epilogue) sum_g f32(s[n][g]) * xs[m][g] * sum_{k in g} w[n][k] * xq[m][k]
// with the per-32-group integer sum exact -- int8 activations (QUANTQ8T) times
// int8 weights (nib - 8, or code - 1) -- exactly as the reference's dot4I8Packed
// sums, then scaled in f32 once per group.
//
// This file is the warp-level form (tb_gemm_dp4_warp): the integer products run
// on mma.sync m16n8k32 .s8 (one instruction is one 32-group of a 16 x 8 tile,
// int32 accumulators started fresh every group) and each group's int32 tile is
// scaled and folded into f32 accumulators in registers (packed f32x2 ops; the
// int32 -> f32 conversion by the exact magic-number add, |sum| < 2^22), the MMA
// and the scaling sharing the same warps' issue slots.  The product path
// (tb_gemm_dp4) is the tcgen05 form in tb_gemm_i8.cu, which computes the same
// values in the same order (bit-equal outputs); this one stays as the
// cross-check.  CTA tile 128 x 128, 8 warps of 64 x 32, K in stages of 128
// (4 groups): int8 activations arrive by cp.async straight into XOR-swizzled
// shared rows; packed weights are loaded a stage ahead into registers and
// widened to int8 (byte permutes + per-byte subtract) while the previous stage
// computes; fragments via ldmatrix.
#include "tb_internal.h"

namespace {

constexpr int BM = 128, BN = 128, BK = 128, THREADS = 256, NG = BK / 32;
constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK;
constexpr int XS_BYTES = BM * NG * 4, SW_BYTES = BN * NG * 4;
constexpr int STAGE = A_BYTES + B_BYTES + XS_BYTES + SW_BYTES;   // 36 KB
constexpr int NST = 2;
constexpr int SMEM = NST * STAGE + 128;

struct DArgs {
    const int8_t* xq;       // [M][K]
    const float* xs;        // [M][K/32]
    const uint32_t* pack;   // [N][K/8] int4 or [N][K/16] ternary
    const uint16_t* scales; // [N][K/32] f16
    float* y;               // [M][N]
    int M, N, K, epi;
};

__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
// 16-byte chunk c (0..7) of row r of a 128-byte-row tile, XOR-swizzled by row
__device__ __forceinline__ int swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

__device__ __forceinline__ void cp16(void* s, const void* g)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(saddr(s)), "l"(g) : "memory");
}
__device__ __forceinline__ void ldsm4(uint32_t* r, const void* p)
{
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(saddr(p)));
}
__device__ __forceinline__ void mma_s8(int* c, const uint32_t* a, uint32_t b0, uint32_t b1)
{
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 8 packed nibbles (k = 8i..8i+7 at bits 4i) -> 8 int8 (nib - 8) in k order
__device__ __forceinline__ uint2 widen_int4(uint32_t w)
{
    const uint32_t lo = w & 0x0f0f0f0fu, hi = (w >> 4) & 0x0f0f0f0fu;   // n0 n2 n4 n6 / n1 n3 n5 n7
    return make_uint2(__vsub4(__byte_perm(lo, hi, 0x5140), 0x08080808u),
                      __vsub4(__byte_perm(lo, hi, 0x7362), 0x08080808u));
}
// 16 ternary codes (k = 4s+b at bits 8b+2s) -> 16 int8 (code - 1) in k order
__device__ __forceinline__ uint4 widen_tern(uint32_t w)
{
    constexpr uint32_t M = 0x03030303u;
    return make_uint4(__vsub4(w & M, 0x01010101u), __vsub4((w >> 2) & M, 0x01010101u),
                      __vsub4((w >> 4) & M, 0x01010101u), __vsub4((w >> 6) & M, 0x01010101u));
}

template <bool TERN>
__global__ void __launch_bounds__(THREADS) k_gemm_dp4(const DArgs a)
{
    extern __shared__ __align__(128) unsigned char smem_raw[];
    unsigned char* smem = smem_raw + ((128 - (saddr(smem_raw) & 127)) & 127);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int wm = (warp & 1) * 64, wn = (warp >> 1) * 32;   // this warp's 64 x 32 tile
    const int nk = a.K / BK, G = a.K / 32;
    constexpr int WPR = TERN ? BK / 16 : BK / 8;             // packed words per weight row per stage

    tb_pdl_wait();
    tb_pdl_trigger();

    // producer mapping: A 1024 16-byte chunks (4 per thread); W rows (2 threads a
    // row, WPR/2 words each); scales: thread < 128 -> xs row, 128.. -> w row
    const int wr = tid >> 1, wh = tid & 1;
    uint32_t wreg[WPR / 2];
    auto load_w = [&](int ks) {
        const uint32_t* src = a.pack + (size_t)(n0 + wr) * (a.K / (TERN ? 16 : 8)) + ks * WPR + wh * (WPR / 2);
#pragma unroll
        for (int i = 0; i < WPR / 2; i += 4) {
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(src + i));
            wreg[i] = v.x; wreg[i + 1] = v.y; wreg[i + 2] = v.z; wreg[i + 3] = v.w;
        }
    };
    auto issue_a = [&](int ks, unsigned char* st) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int c = i * THREADS + tid, r = c >> 3, ch = c & 7;
            cp16(st + swz(r, ch), a.xq + (size_t)(m0 + r) * a.K + ks * BK + ch * 16);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    auto stage_w = [&](int ks, unsigned char* st) {
        unsigned char* B = st + A_BYTES;
        // widened row: 128 int8 = 8 chunks; this thread writes chunks 4 wh .. 4 wh + 3
        if (TERN) {
#pragma unroll
            for (int i = 0; i < WPR / 2; i++) {     // 4 words = 64 k = 4 chunks
                const uint4 v = widen_tern(wreg[i]);
                *reinterpret_cast<uint4*>(B + swz(wr, 4 * wh + i)) = v;
            }
        } else {
#pragma unroll
            for (int i = 0; i < WPR / 2; i += 2) {  // 8 words = 64 k = 4 chunks
                const uint2 p = widen_int4(wreg[i]), q = widen_int4(wreg[i + 1]);
                *reinterpret_cast<uint4*>(B + swz(wr, 4 * wh + i / 2)) = make_uint4(p.x, p.y, q.x, q.y);
            }
        }
        // scales of the stage's 4 groups, f32
        float* xsm = reinterpret_cast<float*>(st + A_BYTES + B_BYTES);
        float* swm = xsm + BM * NG;
        if (tid < BM) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(a.xs + (size_t)(m0 + tid) * G + ks * NG));
            *reinterpret_cast<float4*>(xsm + tid * NG) = v;
        } else {
            const int r = tid - BM;
            const uint2 v = __ldg(reinterpret_cast<const uint2*>(a.scales + (size_t)(n0 + r) * G + ks * NG));
            swm[r * NG + 0] = tb_h2f((uint16_t)(v.x & 0xffffu));
            swm[r * NG + 1] = tb_h2f((uint16_t)(v.x >> 16));
            swm[r * NG + 2] = tb_h2f((uint16_t)(v.y & 0xffffu));
            swm[r * NG + 3] = tb_h2f((uint16_t)(v.y >> 16));
        }
        (void)ks;
    };

    float acc[4][4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j][0] = acc[i][j][1] = acc[i][j][2] = acc[i][j][3] = 0.f;

    // prologue: stage 0
    load_w(0);
    issue_a(0, smem);
    stage_w(0, smem);
    for (int ks = 0; ks < nk; ks++) {
        unsigned char* st = smem + (ks & 1) * STAGE;
        unsigned char* nx = smem + ((ks + 1) & 1) * STAGE;
        const bool more = ks + 1 < nk;
        if (more) {
            load_w(ks + 1);            // registers, consumed after this stage's math
            issue_a(ks + 1, nx);       // the other buffer was released by the barrier below
        }
        if (more) asm volatile("cp.async.wait_group 1;" ::: "memory");
        else asm volatile("cp.async.wait_group 0;" ::: "memory");
        __syncthreads();               // stage ks (A by cp.async, W and scales by stores) complete
        const unsigned char* A = st;
        const unsigned char* B = st + A_BYTES;
        const float* xsm = reinterpret_cast<const float*>(st + A_BYTES + B_BYTES);
        const float* swm = xsm + BM * NG;
#pragma unroll
        for (int gi = 0; gi < NG; gi++) {
            // A fragments (4 m-tiles) and B fragments (4 n-tiles) of group gi: 32 k = 2 chunks
            uint32_t af[4][4], bf[4][2];
#pragma unroll
            for (int mt = 0; mt < 4; mt++) {
                const int r = wm + mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                ldsm4(af[mt], A + swz(r, 2 * gi + (lane >> 4)));
            }
#pragma unroll
            for (int np = 0; np < 2; np++) {
                uint32_t r4[4];
                const int r = wn + np * 16 + (lane & 7) + (lane >> 4) * 8;
                ldsm4(r4, B + swz(r, 2 * gi + ((lane >> 3) & 1)));
                bf[2 * np][0] = r4[0]; bf[2 * np][1] = r4[1];
                bf[2 * np + 1][0] = r4[2]; bf[2 * np + 1][1] = r4[3];
            }
            float sx[4][2], sw[4][2];
#pragma unroll
            for (int mt = 0; mt < 4; mt++) {
                sx[mt][0] = xsm[(wm + mt * 16 + g) * NG + gi];
                sx[mt][1] = xsm[(wm + mt * 16 + g + 8) * NG + gi];
            }
#pragma unroll
            for (int nt = 0; nt < 4; nt++) {
                sw[nt][0] = swm[(wn + nt * 8 + 2 * t) * NG + gi];
                sw[nt][1] = swm[(wn + nt * 8 + 2 * t + 1) * NG + gi];
            }
#pragma unroll
            for (int mt = 0; mt < 4; mt++) {
#pragma unroll
                for (int nt = 0; nt < 4; nt++) {
                    int c[4] = {0, 0, 0, 0};
                    mma_s8(c, af[mt], bf[nt][0], bf[nt][1]);
                    // exact int -> f32 (|c| < 2^22): 2^23 + 2^22 + c, minus the same
                    const float2 M2 = make_float2(-12582912.f, -12582912.f);
                    const float2 f01 = fadd2(make_float2(__int_as_float(c[0] + 0x4B400000), __int_as_float(c[1] + 0x4B400000)), M2);
                    const float2 f23 = fadd2(make_float2(__int_as_float(c[2] + 0x4B400000), __int_as_float(c[3] + 0x4B400000)), M2);
                    // f32(s) * xs per output (the shader's f32(sc) * xsc), then * the group sum
                    const float2 p01 = make_float2(sw[nt][0] * sx[mt][0], sw[nt][1] * sx[mt][0]);
                    const float2 p23 = make_float2(sw[nt][0] * sx[mt][1], sw[nt][1] * sx[mt][1]);
                    float2 a01 = make_float2(acc[mt][nt][0], acc[mt][nt][1]);
                    float2 a23 = make_float2(acc[mt][nt][2], acc[mt][nt][3]);
                    a01 = ffma2(p01, f01, a01);
                    a23 = ffma2(p23, f23, a23);
                    acc[mt][nt][0] = a01.x; acc[mt][nt][1] = a01.y;
                    acc[mt][nt][2] = a23.x; acc[mt][nt][3] = a23.y;
                }
            }
        }
        __syncthreads();               // stage ks consumed: its buffer may be refilled
        if (more) stage_w(ks + 1, nx);
    }
    // epilogue: rows g, g+8 of each m-tile, columns 2t, 2t+1 of each n-tile
#pragma unroll
    for (int mt = 0; mt < 4; mt++) {
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const int row = m0 + wm + mt * 16 + g + 8 * h;
            float* yr = a.y + (size_t)row * a.N + n0 + wn;
#pragma unroll
            for (int nt = 0; nt < 4; nt++) {
                float2 v = make_float2(acc[mt][nt][2 * h], acc[mt][nt][2 * h + 1]);
                float2* yp = reinterpret_cast<float2*>(yr + nt * 8 + 2 * t);
                if (a.epi == 1) {
                    const float2 o = *yp;
                    v.x += o.x; v.y += o.y;
                } else if (a.epi == 2) {
                    const float2 gt = *yp;
                    v.x = __fdiv_rn(gt.x, 1.0f + expf(-gt.x)) * v.x;
                    v.y = __fdiv_rn(gt.y, 1.0f + expf(-gt.y)) * v.y;
                }
                *yp = v;
            }
        }
    }
}

template <bool TERN>
int launch(tb_ctx* ctx, const DArgs& a)
{
    static bool attr[64] = {};
    if (ctx->device >= 64 || !attr[ctx->device]) {
        cudaError_t e = cudaFuncSetAttribute(k_gemm_dp4<TERN>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
        if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "gemm_dp4 attribute: %s", cudaGetErrorString(e));
        if (ctx->device < 64) attr[ctx->device] = true;
    }
    cudaError_t e = tb_launch(ctx, k_gemm_dp4<TERN>, dim3(a.N / BN, a.M / BM), dim3(THREADS), (size_t)SMEM, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "gemm_dp4 launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

}  // namespace

int tb_gemm_dp4_warp_impl(tb_ctx* ctx, float* y, const int8_t* xq, const float* xs, const uint32_t* pack,
                          const uint16_t* scales, int64_t M, int64_t N, int64_t K, int epilogue, bool tern)
{
    TB_REQUIRE(ctx, y && xq && xs && pack && scales, "null pointer");
    TB_REQUIRE(ctx, M > 0 && M % BM == 0 && N > 0 && N % BN == 0 && K > 0 && K % BK == 0,
               "gemm_dp4: M %% %d, N %% %d and K %% %d must be 0 (got %lld x %lld x %lld)", BM, BN, BK,
               (long long)M, (long long)N, (long long)K);
    TB_REQUIRE(ctx, M / BM <= 65535 && N / BN <= 65535 && K < (1LL << 30), "gemm_dp4: shape too large");
    TB_REQUIRE(ctx, epilogue >= 0 && epilogue <= 2, "gemm_dp4: bad epilogue %d", epilogue);
    TB_REQUIRE(ctx, TB_ALIGNED(xq, 16) && TB_ALIGNED(xs, 16) && TB_ALIGNED(pack, 16) && TB_ALIGNED(scales, 8) &&
                        TB_ALIGNED(y, 8),
               "gemm_dp4: xq, xs, pack 16-byte, scales and y 8-byte aligned");
    DArgs a{xq, xs, pack, scales, y, (int)M, (int)N, (int)K, epilogue};
    return tern ? launch<true>(ctx, a) : launch<false>(ctx, a);
}

extern "C" TB_API int tb_gemm_dp4_warp(tb_ctx* ctx, float* y, const int8_t* xq, const float* xs,
                                       const uint32_t* pack, const uint16_t* scales, int64_t M, int64_t N, int64_t K,
                                       int epilogue, int tern)
{
    if (!ctx) return TB_ERR_INVALID;
    return tb_gemm_dp4_warp_impl(ctx, y, xq, xs, pack, scales, M, N, K, epilogue, tern != 0);
}
