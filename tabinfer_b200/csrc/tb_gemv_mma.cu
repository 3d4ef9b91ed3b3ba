// tb_gemv_mma.cu -- decode GEMVs over 2..16 activation rows that read every
// weight once, with the integer products on the tensor cores.
//
// Semantics: linearQ's T > 1 route, the DP4A GEMM (models/qwen3.js:1600-1607,
// gemmdp4Wgsl :1321-1407; ternary gemmTern :1410-1420): per 32-group the exact
// int32 sum of int8 activations (QUANTQ8T, qwen3.js:332-358, or RMSNORMQ
// :569-612) times the int4 weights (nib - 8), or the ternary WebGPU codes
// (code - 1), then one f32 scaling by xs[t][g] * s[n][g] per group.
//
// B200 design
//  * Tokens are the MMA's M (16, zero rows past the batch) and weight rows its
//    N: one mma.sync m16n8k32 (s8 activations x u8 weights) is one 32-group of
//    an 8-row tile for all tokens.  The weight operand is the raw nibble (or
//    2-bit code) masked in place -- (word >> s) & 0x0f0f0f0f -- with no
//    widening: the bias is folded into the group sum as
//       sum x*(nib - 8) = sum x*nib - 8*sum x,
//    and the -8*sum x (or -sum x) rides on the exact int32 -> f32 conversion,
//    float(v) = as_float(v + 0x4B400000) - 12582912 for |v| < 2^22, through a
//    per-token-group constant kc = 0x4B400000 - 8*sum(x) the quantizer stores.
//  * The quantizer (k_quant_mma) writes the activation once per call, already
//    in fragment order: per group and token 32 bytes holding the MMA k-slots
//    t and 4+t of thread t side by side, so an A fragment is one 8-byte shared
//    load per token half, conflict-free.  For int4 the k-slots follow the
//    nibble lanes of a packed word (slot i = k 8i+{0,2,4,6}, the low nibbles
//    of word i; slot 4+i = k 8i+{1,3,5,7}, its high nibbles), so thread t's B
//    fragment is word t of the group masked twice: one shared load.  For
//    ternary they are natural order (slot s = k 4s..4s+3).
//  * The MMA starts from C = kc, so the bias and the magic constant ride in
//    the tensor core's accumulator: D = kc + sum, float(D) - 12582912.
//  * Each CTA owns a contiguous range of 8-row tiles (an even split of all
//    tiles over the grid), taken in work items of up to 64 rows of one matrix
//    (gate/up: 32 rows of each).  An item streams through a ring of stages of
//    16 groups, each moved by TMA tensor copies (cp.async.bulk.tensor.2d over
//    a tensor map of the packed weights, 64 rows x 128 bytes a box, 128-byte
//    swizzle; one box of the f16 scales) plus two bulk copies of the stage's
//    activation slice: five copies a stage.  The swizzle (16-byte chunk c of
//    row r lands at chunk c ^ (r & 7)) makes the B-fragment loads of the eight
//    rows of a tile hit eight different bank groups.  The weight copies of the
//    first stages are issued before griddepcontrol.wait, so they overlap the
//    previous kernel.
//  * The 16 warps split a stage's 16 groups (warp w: group w); every warp
//    covers all tiles of the item with its group's A fragment in registers.  Tiles sit at fixed places of the
//    stage (gate/up: gate tiles 0-3, up tiles 4-7), so every shared address is
//    the stage base plus a compile-time and a per-thread constant.
//    At the item's end the 16 partial tiles meet in shared memory in warp order
//    (deterministic, independent of the grid) and the epilogue stores, adds
//    the residual, or applies silu(gate) * up.
#include <cuda.h>
#include <cudaTypedefs.h>
#include "tb_gemv_dev.cuh"
#include "tb_internal.h"

namespace {

constexpr int MM_THREADS = 512, MM_WARPS = 16;
constexpr int MM_KS = 16;          // 32-groups per stage
constexpr int MM_MAXT = 8;         // 8-row tiles per work item
constexpr int MM_NST = 4;          // stages in the ring
constexpr uint32_t MM_MAGIC = MMA_KC_MAGIC;   // bits of 12582912.0f = 2^23 + 2^22
constexpr float MM_MAGIC_F = 12582912.0f;
constexpr int ERR_MMA_WAIT = 0x6d03;

// bytes of one 32-group of a packed weight row: 16 (int4) or 8 (ternary)
__host__ __device__ constexpr int mm_wg(bool tern) { return tern ? 8 : 16; }
// 128-byte boxes a stage row spans (16 groups): 2 (int4) or 1 (ternary)
__host__ __device__ constexpr int mm_nbox(bool tern) { return tern ? 1 : 2; }
__host__ __device__ constexpr int mm_w_bytes(bool tern) { return mm_nbox(tern) * 64 * 128; }
constexpr int MM_S_BYTES = 64 * MM_KS * 2;   // f16 scales of the stage's rows
__host__ __device__ constexpr int mm_stage_bytes(bool tern, int ts)
{
    return mm_w_bytes(tern) + MM_S_BYTES
           + MM_KS * ts * 32                // activation slots
           + MM_KS * ts * 8;                // {xs, kc} per token-group
}
// ring (1024-aligned stages for the 128-byte swizzle) + the cross-warp partials
__host__ __device__ constexpr int mm_smem_bytes(bool tern, int ts)
{
    return 1024 + MM_NST * mm_stage_bytes(tern, ts) + MM_WARPS * MM_MAXT * 32 * 4 * 4;
}

struct MmMat {
    float* y;          // [B][N]
    int N;
    int tile_begin;    // first tile of this matrix in the concatenated tile list
};

struct MmArgs {
    CUtensorMap tw[3];     // packed weights: u8 [N][K/2 or K/4], box 128 x (64 or 32) rows, 128-byte swizzle
    CUtensorMap tsc[3];    // f16 scales [N][K/32], box 16 x (64 or 32) rows
    MmMat m[3];
    int count;         // matrices (gate/up: m[0] gate, m[1] up, one unit = a tile of each)
    int units;         // tiles, or tile pairs for gate/up
    int nu;            // units per work item (<= 8 tiles, <= 4 pairs): the boxes are 8 * nu rows
    int ualign;        // a CTA's unit range starts on a multiple of this (4 pairs: one swi group)
    int K, G, B, acc;
    const unsigned char* xa;   // [G][TS][32] activation slots
    const uint2* xk;           // [G][TS] {xs bits, kc}
    // gate/up only: swi written QUANTQ8'd in the same fragment order for the next
    // GEMV ([I/32][TS][32] + [I/32][TS]; items are whole 32-row groups), instead of f32
    unsigned char* oxa;
    uint2* oxk;
    int otern;                 // the next GEMV's weights are ternary (natural k order, kc factor 1)
    int grid;          // CTAs: ceil(units / units per CTA)
    int* err;
};

__device__ __forceinline__ float2 fmul2(float2 a, float2 b)
{
    float2 d;
    asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2,%3};\n mov.b64 rb, {%4,%5};\n"
        " mul.rn.f32x2 rd, ra, rb;\n mov.b64 {%0,%1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// d = a . b + c (c: the token rows' kc, so d is the biased sum; c and d are
// separate register quads, so the seed is built once per group)
__device__ __forceinline__ void mma_s8u8(int* d, const uint32_t* a, uint32_t b0, uint32_t b1, const int* c)
{
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c[0]), "r"(c[1]), "r"(c[2]),
          "r"(c[3]));
}

// QUANTQ8 of one 32-group held one element per lane (the whole warp), stored in
// fragment order at row slot m of group g
__device__ __forceinline__ void mm_store_group(float v, int g, int m, int ts, bool tern, unsigned char* xa,
                                               uint2* xk)
{
    const int lane = threadIdx.x & 31;
    const Q8Group qg = q8_group(v);
    int sum = qg.q;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    xa[((size_t)g * ts + m) * 32 + mma_slot_pos(lane, tern)] = (unsigned char)(qg.q & 0xff);
    if (lane == 0) xk[(size_t)g * ts + m] = make_uint2(__float_as_uint(qg.scale), MM_MAGIC - (tern ? 1u : 8u) * (uint32_t)sum);
}

// One group of one stage for the first NT tiles of the item (gate/up: NT pairs,
// gate tiles at slots 0..NT-1, up tiles at 4..4+NT-1): NT is a compile-time count,
// so every tile's MMA runs unconditionally.
template <bool TERN, bool GU, bool M16, int NT>
__device__ __forceinline__ void mm_group(float2 (&acc)[MM_MAXT][2], const unsigned char* W, const uint16_t* S,
                                         int BR, int wofs, int sh, int g, int t, int gl, const uint32_t* af,
                                         const int* cq, float2 xslo, float2 xshi)
{
    constexpr int NBOX = mm_nbox(TERN);
    constexpr uint32_t mask = TERN ? 0x03030303u : 0x0f0f0f0fu;
    const float2 nmagic = make_float2(-MM_MAGIC_F, -MM_MAGIC_F);
#pragma unroll
    for (int i = 0; i < MM_MAXT; i++) {
        if (GU ? (i & 3) < NT : i < NT) {
            const int sm = GU ? (i >> 2) : 0;              // gate or up
            const int rt = GU ? (i & 3) * 8 : i * 8;       // tile's first row within the box
            const unsigned char* wb = W + sm * NBOX * BR * 128 + (rt + g) * 128 + wofs;
            uint32_t b0, b1;
            if (TERN) {
                const uint2 v = *reinterpret_cast<const uint2*>(wb);
                b0 = (v.x >> sh) & mask;
                b1 = (v.y >> sh) & mask;
            } else {
                const uint32_t w = *reinterpret_cast<const uint32_t*>(wb);
                b0 = w & mask;
                b1 = (w >> 4) & mask;
            }
            // f16 scales of rows rt + 2t, rt + 2t + 1
            const uint16_t* sb = S + sm * BR * MM_KS + (rt + 2 * t) * MM_KS + gl;
            const float2 ws = make_float2(tb_h2f(sb[0]), tb_h2f(sb[MM_KS]));
            int d[4];
            mma_s8u8(d, af, b0, b1, cq);
            const float2 vlo = fadd2(make_float2(__int_as_float(d[0]), __int_as_float(d[1])), nmagic);
            acc[i][0] = ffma2(vlo, fmul2(xslo, ws), acc[i][0]);
            if (M16) {
                const float2 vhi = fadd2(make_float2(__int_as_float(d[2]), __int_as_float(d[3])), nmagic);
                acc[i][1] = ffma2(vhi, fmul2(xshi, ws), acc[i][1]);
            }
        }
    }
}


// ---- activation quantizer ---------------------------------------------------
// One 256-thread CTA per (token slot, group range); token slots >= B are zero
// (q = 0, xs = 0, kc = magic).  Per 32-group: QUANTQ8 of the (optionally
// RMSNorm-ed) values with the shared code of every quantizer here (bit-identical
// int8 and scale), stored in fragment order.
template <bool TERN>
__global__ void __launch_bounds__(256) k_quant_mma(const float* __restrict__ x, const uint16_t* __restrict__ w16,
                                                   float eps, int K, int B, int ts, unsigned char* __restrict__ xa,
                                                   uint2* __restrict__ xk)
{
    __shared__ float red[80];
    tb_pdl_wait();
    tb_pdl_trigger();
    const int b = blockIdx.x, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int G = K >> 5;
    const int g0 = (int)((long long)blockIdx.y * G / gridDim.y), g1 = (int)((long long)(blockIdx.y + 1) * G / gridDim.y);
    if (b >= B) {
        for (int g = g0 + wid; g < g1; g += 8) {
            xa[((size_t)g * ts + b) * 32 + lane] = 0;
            if (lane == 0) xk[(size_t)g * ts + b] = make_uint2(0u, MM_MAGIC);
        }
        return;
    }
    const float* xr = x + (size_t)b * K;
    float inv = 0.0f;
    if (w16) inv = rms_inv(block256_sumsq(xr, K, red), K, eps);
    for (int g = g0 + wid; g < g1; g += 8) {
        const int k = g * 32 + lane;
        float v = xr[k];
        if (w16) v = __fmul_rn(__fmul_rn(v, inv), tb_h2f(w16[k]));
        mm_store_group(v, g, b, ts, TERN, xa, xk);
    }
}

// ---- the GEMV ---------------------------------------------------------------
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(saddr(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(saddr(bar))
                 : "memory");
}

// A work item: up to a.nu consecutive units of one matrix (gate/up: of the pair list)
struct MmItem {
    int ub, n, mi;
};
template <bool GU>
__device__ __forceinline__ MmItem mm_item(const MmArgs& a, int u, int u1)
{
    const int NU = a.nu;
    int mi = 0, end = u1;
    if (!GU) {
#pragma unroll
        for (int i = 1; i < 3; i++) if (i < a.count && u >= a.m[i].tile_begin) mi = i;
        end = min(end, a.m[mi].tile_begin + a.m[mi].N / 8);
    }
    return MmItem{u, min(NU, end - u), mi};
}

template <bool TERN, bool GU, bool M16>
__global__ void __launch_bounds__(MM_THREADS, 1) k_gemv_mma(const __grid_constant__ MmArgs a)
{
    constexpr int TS = M16 ? 16 : 8;
    constexpr int WG = mm_wg(TERN), NBOX = mm_nbox(TERN), NM = GU ? 2 : 1;
    constexpr int SB = mm_stage_bytes(TERN, TS);
    constexpr int W_BYTES = mm_w_bytes(TERN), A_BYTES = MM_KS * TS * 32;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full[MM_NST];
    __shared__ float swq[GU ? 16 * 33 : 1];      // gate/up with a quantized output: one group of swi
    unsigned char* stages = smem_raw + ((1024 - (saddr(smem_raw) & 1023)) & 1023);
    float* red = reinterpret_cast<float*>(stages + MM_NST * SB);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
    const int G = a.G;
    const int nks = (G + MM_KS - 1) / MM_KS;
    const int BR = 8 * a.nu;              // rows of a weight / scale box (one item)
    const int nq = a.units / a.ualign;
    const int u0 = (int)((long long)blockIdx.x * nq / gridDim.x) * a.ualign;
    const int u1 = blockIdx.x + 1 == (int)gridDim.x ? a.units : (int)((long long)(blockIdx.x + 1) * nq / gridDim.x) * a.ualign;
    int nitems = 0;
    for (int u = u0; u < u1; nitems++) u += mm_item<GU>(a, u, u1).n;
    const int total = nitems * nks;

    // producer (thread 0): stage `it` of item `pi` into its ring slot; weights and
    // scales (wpart, with the stage's expect_tx) and / or the activation (apart)
    auto issue = [&](int it, const MmItem& pi, int ks, bool wpart, bool apart) {
        const int slot = it % MM_NST;
        unsigned char* st = stages + slot * SB;
        const int g0 = ks * MM_KS, kg = min(MM_KS, G - g0);
        const int nbox = TERN ? 1 : (kg > 8 ? 2 : 1);   // no box wholly past K
        if (wpart) {
            mbar_expect_tx(&full[slot], (uint32_t)(NM * (nbox * BR * 128 + BR * MM_KS * 2) + kg * TS * 40));
#pragma unroll
            for (int s = 0; s < NM; s++) {
                const int mi = GU ? s : pi.mi;
                const int row0 = (pi.ub - (GU ? 0 : a.m[mi].tile_begin)) * 8;
                for (int b = 0; b < nbox; b++)
                    tma_2d(st + (s * NBOX + b) * BR * 128, &a.tw[mi], g0 * WG + b * 128, row0, &full[slot]);
                tma_2d(st + W_BYTES + s * BR * MM_KS * 2, &a.tsc[mi], g0, row0, &full[slot]);
            }
        }
        if (apart) {
            bulk_g2s(st + W_BYTES + MM_S_BYTES, a.xa + (size_t)g0 * TS * 32, (uint32_t)(kg * TS * 32), &full[slot]);
            bulk_g2s(st + W_BYTES + MM_S_BYTES + A_BYTES, a.xk + (size_t)g0 * TS, (uint32_t)(kg * TS * 8),
                     &full[slot]);
        }
    };

    if (tid == 0) {
        for (int s = 0; s < MM_NST; s++) mbar_init(&full[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();
    const int npro = min(MM_NST, total);
    MmItem pi = mm_item<GU>(a, u0, u1);   // producer's item and stage within it
    int pks = 0;
    if (tid == 0) {
        // weights do not depend on the previous kernel: request them first
        MmItem q = pi;
        int qks = 0;
        for (int it = 0; it < npro; it++) {
            issue(it, q, qks, true, false);
            if (++qks == nks) { qks = 0; q = mm_item<GU>(a, q.ub + q.n, u1); }
        }
    }
    tb_pdl_wait();
    tb_pdl_trigger();
    if (tid == 0) {
        for (int it = 0; it < npro; it++) {
            issue(it, pi, pks, false, true);
            if (++pks == nks) { pks = 0; pi = mm_item<GU>(a, pi.ub + pi.n, u1); }
        }
    }

    // this warp's group of every stage and this thread's byte offset of its weight
    // word(s) within a box row (row & 7 == g: the 128-byte swizzle puts chunk c of
    // the row at c ^ g)
    const int gl = warp;
    const int wofs = TERN ? ((((gl >> 1) ^ g) << 4) + (gl & 1) * 8)
                          : (gl >> 3) * BR * 128 + (((gl & 7) ^ g) << 4) + 4 * t;
    const int sh = TERN ? 2 * t : 0;

    float2 acc[MM_MAXT][2];
    MmItem ci = mm_item<GU>(a, u0, u1);
    int cks = 0;
    for (int it = 0; it < total; it++) {
        const int slot = it % MM_NST;
        const int kg = min(MM_KS, G - cks * MM_KS);
        if (cks == 0) {
#pragma unroll
            for (int i = 0; i < MM_MAXT; i++) acc[i][0] = acc[i][1] = make_float2(0.0f, 0.0f);
        }
        const bool ok = mbar_wait(&full[slot], (uint32_t)((it / MM_NST) & 1));
        if (ok && gl < kg) {
            const unsigned char* W = stages + slot * SB;
            const uint16_t* S = reinterpret_cast<const uint16_t*>(W + W_BYTES);
            const unsigned char* A = W + W_BYTES + MM_S_BYTES;
            const uint2* X = reinterpret_cast<const uint2*>(A + A_BYTES);
            const uint2 alo = *reinterpret_cast<const uint2*>(A + (gl * TS + g) * 32 + 8 * t);
            const uint2 xlo = X[gl * TS + g];
            uint2 ahi = make_uint2(0u, 0u), xhi = make_uint2(0u, MM_MAGIC);
            if (M16) {
                ahi = *reinterpret_cast<const uint2*>(A + (gl * TS + g + 8) * 32 + 8 * t);
                xhi = X[gl * TS + g + 8];
            }
            const uint32_t af[4] = {alo.x, ahi.x, alo.y, ahi.y};
            const int cq[4] = {(int)xlo.y, (int)xlo.y, (int)xhi.y, (int)xhi.y};
            const float2 xslo = make_float2(__uint_as_float(xlo.x), __uint_as_float(xlo.x));
            const float2 xshi = make_float2(__uint_as_float(xhi.x), __uint_as_float(xhi.x));
#define MM_GROUP(N) mm_group<TERN, GU, M16, N>(acc, W, S, BR, wofs, sh, g, t, gl, af, cq, xslo, xshi)
            switch (ci.n) {   // warp-uniform: one branch a group
            case 1: MM_GROUP(1); break;
            case 2: MM_GROUP(2); break;
            case 3: MM_GROUP(3); break;
            case 4: MM_GROUP(4); break;
            case 5: if (!GU) MM_GROUP(5); break;
            case 6: if (!GU) MM_GROUP(6); break;
            case 7: if (!GU) MM_GROUP(7); break;
            default: if (!GU) MM_GROUP(8); break;
            }
#undef MM_GROUP
        }
        const bool last = cks == nks - 1;
        if (last && ok) {
            // the item's partial tiles, warp by warp: red[warp][tile][lane][4]
#pragma unroll
            for (int i = 0; i < MM_MAXT; i++)
                if (GU ? (i & 3) < ci.n : i < ci.n)
                    *reinterpret_cast<float4*>(red + ((warp * MM_MAXT + i) * 32 + lane) * 4) =
                        make_float4(acc[i][0].x, acc[i][0].y, acc[i][1].x, acc[i][1].y);
        }
        if (__syncthreads_or(!ok)) {
            // a stage never arrived: record it, let the copies still in flight land
            // (bounded), and leave
            if (tid == 0 && a.err) atomicExch(a.err, ERR_MMA_WAIT);
            for (int j = it; j < min(total, it + MM_NST); j++) mbar_wait(&full[j % MM_NST], (uint32_t)((j / MM_NST) & 1));
            return;
        }
        // every warp is past stage it: refill its slot with stage it + NST before the
        // item's epilogue, so the stream does not pause at item ends
        if (tid == 0 && it + MM_NST < total) {
            issue(it + MM_NST, pi, pks, true, true);
            if (++pks == nks) { pks = 0; pi = mm_item<GU>(a, pi.ub + pi.n, u1); }
        }
        if (last) {
            const int nout = ci.n * 128;
            for (int q = tid; q < nout; q += MM_THREADS) {
                const int i = q >> 7, l = (q >> 2) & 31, e = q & 3;
                const int m = (l >> 2) + 8 * (e >> 1), col = 2 * (l & 3) + (e & 1);
                if (m >= a.B) continue;
                float v = red[(i * 32 + l) * 4 + e];
#pragma unroll
                for (int w = 1; w < MM_WARPS; w++) v += red[((w * MM_MAXT + i) * 32 + l) * 4 + e];
                if (GU) {
                    float u = red[((i + 4) * 32 + l) * 4 + e];          // up tiles sit at slots 4..7
#pragma unroll
                    for (int w = 1; w < MM_WARPS; w++) u += red[((w * MM_MAXT + i + 4) * 32 + l) * 4 + e];
                    const float sw = __fdiv_rn(v, 1.0f + expf(-v)) * u;
                    if (a.oxa) swq[m * 33 + i * 8 + col] = sw;           // the item is one 32-row group
                    else a.m[0].y[(size_t)m * a.m[0].N + (ci.ub + i) * 8 + col] = sw;
                } else {
                    const MmMat& M = a.m[ci.mi];
                    float* y = M.y + (size_t)m * M.N + (ci.ub - M.tile_begin + i) * 8 + col;
                    *y = a.acc ? *y + v : v;
                }
            }
            __syncthreads();   // red is rewritten by the next item
            if (GU && a.oxa) {
                // swi group ci.ub / 4 of every row, QUANTQ8'd for the down GEMV: warp = row
                if (warp < a.B) mm_store_group(swq[warp * 33 + lane], ci.ub >> 2, warp, TS, a.otern, a.oxa, a.oxk);
                __syncthreads();   // swq is rewritten by the next item
            }
        }
        if (++cks == nks) { cks = 0; ci = mm_item<GU>(a, ci.ub + ci.n, u1); }
    }
}

// ---- host -------------------------------------------------------------------
template <bool TERN, bool GU, bool M16>
int launch_mma(tb_ctx* ctx, const MmArgs& a)
{
    constexpr int smem = mm_smem_bytes(TERN, M16 ? 16 : 8);
    auto kern = k_gemv_mma<TERN, GU, M16>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    e = tb_launch(ctx, kern, dim3(a.grid), dim3(MM_THREADS), (size_t)smem, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "gemv_mma launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

template <bool TERN>
int launch_mma_kind(tb_ctx* ctx, const MmArgs& a, bool gu)
{
    const bool m16 = a.B > 8;
    if (gu) return m16 ? launch_mma<TERN, true, true>(ctx, a) : launch_mma<TERN, true, false>(ctx, a);
    return m16 ? launch_mma<TERN, false, true>(ctx, a) : launch_mma<TERN, false, false>(ctx, a);
}

// cuTensorMapEncodeTiled from the driver, resolved once through the runtime
PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

// 2-D tensor map over a row-major [rows][cols] matrix of `esize`-byte elements
int encode_2d(tb_ctx* ctx, CUtensorMap* map, const void* base, CUtensorMapDataType dt, int esize, int64_t cols,
              int64_t rows, int box_cols, int box_rows, CUtensorMapSwizzle swz)
{
    PFN_cuTensorMapEncodeTiled_v12000 enc = tmap_encoder();
    if (!enc) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)(cols * esize)};
    const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return tb_fail(ctx, TB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return TB_OK;
}

}  // namespace

int tb_encode_2d(tb_ctx* ctx, CUtensorMap* map, const void* base, CUtensorMapDataType dt, int esize, int64_t cols,
                 int64_t rows, int box_cols, int box_rows, CUtensorMapSwizzle swz)
{
    return encode_2d(ctx, map, base, dt, esize, cols, rows, box_cols, box_rows, swz);
}

size_t tb_gemv_mma_act_bytes(int64_t K, int batch)
{
    const size_t ts = batch > 8 ? 16 : 8;
    return (size_t)(K / 32) * ts * 40;
}

bool tb_gemv_mma_fits(int64_t K, const int64_t* Ns, int count, int batch)
{
    if (batch < 2 || batch > 16 || K <= 0 || K % 256 != 0 || K > 65536) return false;
    for (int i = 0; i < count; i++)
        if (Ns[i] <= 0 || Ns[i] % 8 != 0 || Ns[i] >= (1LL << 28)) return false;
    return true;
}

// quantize x (optionally RMSNorm-ed) into buf ([G][TS][32] slots, then [G][TS]
// {xs, kc}; tb_gemv_mma_act_bytes(K, batch) bytes, 16-byte aligned), then
// y_i (+)= W_i . x for `count` matrices (gateup: swi = silu(W_0 . x) * (W_1 . x)).
int tb_gemv_mma_impl(tb_ctx* ctx, int count, float* const* ys, const uint32_t* const* packs,
                     const uint16_t* const* scales, const int64_t* Ns, const float* x, const uint16_t* normw,
                     float eps, int64_t K, int batch, int acc, bool tern, bool gateup, void* buf, bool quantize,
                     void* obuf, bool otern)
{
    TB_REQUIRE(ctx, count >= 1 && count <= 3 && (!gateup || count == 2), "bad matrix count %d", count);
    TB_REQUIRE(ctx, tb_gemv_mma_fits(K, Ns, count, batch),
               "gemv_mma: needs batch 2..16, K %% 256 == 0 and rows %% 8 == 0 (batch=%d K=%lld)", batch, (long long)K);
    TB_REQUIRE(ctx, (!quantize || (x && TB_ALIGNED(x, 16))) && buf && TB_ALIGNED(buf, 16),
               "x and buf must be 16-byte aligned");
    TB_REQUIRE(ctx, !obuf || (gateup && Ns[0] % 32 == 0 && TB_ALIGNED(obuf, 16)),
               "a quantized output needs gate/up rows in whole 32-groups");
    TB_REQUIRE(ctx, !normw || TB_ALIGNED(normw, 16), "norm weight must be 16-byte aligned");
    for (int i = 0; i < count; i++) {
        TB_REQUIRE(ctx, packs[i] && scales[i] && ys[i], "null weight or output pointer");
        TB_REQUIRE(ctx, TB_ALIGNED(packs[i], 16) && TB_ALIGNED(scales[i], 16), "pack and scales must be 16-byte aligned");
    }
    if (gateup) TB_REQUIRE(ctx, Ns[0] == Ns[1], "gate and up must have the same rows");
    const int ts = batch > 8 ? 16 : 8, G = (int)(K / 32);
    unsigned char* xa = static_cast<unsigned char*>(buf);
    uint2* xk = reinterpret_cast<uint2*>(xa + (size_t)G * ts * 32);
    if (quantize) {
        const int gsplit = std::max(1, std::min(G / 8, std::max(1, 2 * ctx->num_sms / ts)));
        cudaError_t e = tern ? tb_launch(ctx, k_quant_mma<true>, dim3(ts, gsplit), dim3(256), 0, x, normw, eps,
                                         (int)K, batch, ts, xa, xk)
                             : tb_launch(ctx, k_quant_mma<false>, dim3(ts, gsplit), dim3(256), 0, x, normw, eps,
                                         (int)K, batch, ts, xa, xk);
        if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "quant_mma launch: %s", cudaGetErrorString(e));
    }
    MmArgs a{};
    a.count = count;
    a.K = (int)K;
    a.G = G;
    a.B = batch;
    a.acc = acc ? 1 : 0;
    a.xa = xa;
    a.xk = xk;
    a.err = ctx->dev_error;
    int tiles = 0;
    // the even split of the units over the grid, in items whose boxes (8 * nu rows)
    // hold no row past the item: each CTA takes tpc units, in as few items of
    // equal size as fit the stage (8 tiles; gate/up 4 pairs)
    int units = 0;
    for (int i = 0; i < count; i++) units += gateup ? 0 : (int)(Ns[i] / 8);
    if (gateup) units = (int)(Ns[0] / 8);
    const int maxnu = gateup ? MM_MAXT / 2 : MM_MAXT;
    // a quantized swi output: every item is one whole 32-row group (4 pairs)
    a.ualign = obuf ? 4 : 1;
    const int quanta = units / a.ualign;
    const int tpc = ((quanta + ctx->num_sms - 1) / ctx->num_sms) * a.ualign;
    const int nitem = (tpc + maxnu - 1) / maxnu;
    a.nu = (tpc + nitem - 1) / nitem;
    a.grid = (quanta + tpc / a.ualign - 1) / (tpc / a.ualign);
    if (obuf) {
        a.oxa = static_cast<unsigned char*>(obuf);
        a.oxk = reinterpret_cast<uint2*>(a.oxa + (size_t)(Ns[0] / 32) * ts * 32);
        a.otern = otern ? 1 : 0;
    }
    const int box_rows = 8 * a.nu;
    const int64_t wrow = tern ? K / 4 : K / 2;
    for (int i = 0; i < 3; i++) {
        if (i < count) {
            a.m[i] = MmMat{ys[i], (int)Ns[i], tiles};
            if (!gateup) tiles += (int)(Ns[i] / 8);
            int rc = encode_2d(ctx, &a.tw[i], packs[i], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, wrow, Ns[i], 128, box_rows,
                               CU_TENSOR_MAP_SWIZZLE_128B);
            if (!rc) rc = encode_2d(ctx, &a.tsc[i], scales[i], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, G, Ns[i], MM_KS,
                                    box_rows, CU_TENSOR_MAP_SWIZZLE_NONE);
            if (rc) return rc;
        } else {
            a.m[i] = MmMat{nullptr, 0, 1 << 30};
        }
    }
    if (gateup) {
        a.m[1].tile_begin = 0;
        tiles = (int)(Ns[0] / 8);
    }
    a.units = tiles;
    return tern ? launch_mma_kind<true>(ctx, a, gateup) : launch_mma_kind<false>(ctx, a, gateup);
}

extern "C" {

// linearQ's T > 1 DP4A route at 2..16 rows (qwen3.js:1600-1607), one weight read:
// y (+)= W . rmsnorm?(x); the quantized rows go to context scratch.
TB_API int tb_gemv_int4_mma(tb_ctx* ctx, float* y, const float* x, const uint16_t* norm_w16, float eps,
                            const uint32_t* pack, const uint16_t* scales, int64_t N, int64_t K, int T, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    void* buf = tb_ctx_scratch(ctx, tb_gemv_mma_act_bytes(K, T));
    if (!buf) return TB_ERR_NOMEM;
    return tb_gemv_mma_impl(ctx, 1, &y, &pack, &scales, &N, x, norm_w16, eps, K, T, acc, false, false, buf);
}

// rmsnormQ + the q/k/v projGemv triple (qwen3.js:3981-3984) at 2..16 rows: one
// quantization, one launch over the concatenated rows of `count` (<= 3) matrices
TB_API int tb_gemv_int4_mma_multi(tb_ctx* ctx, int count, float* const* ys, const uint32_t* const* packs,
                                  const uint16_t* const* scales, const int64_t* Ns, const float* x,
                                  const uint16_t* norm_w16, float eps, int64_t K, int T, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, ys && packs && scales && Ns, "null array argument");
    void* buf = tb_ctx_scratch(ctx, tb_gemv_mma_act_bytes(K, T));
    if (!buf) return TB_ERR_NOMEM;
    return tb_gemv_mma_impl(ctx, count, ys, packs, scales, Ns, x, norm_w16, eps, K, T, acc, false, false, buf);
}

TB_API int tb_gateup_silu_int4_mma(tb_ctx* ctx, float* swi, const float* x, const uint16_t* norm_w16, float eps,
                                   const uint32_t* gpack, const uint16_t* gscales, const uint32_t* upack,
                                   const uint16_t* uscales, int64_t I, int64_t K, int T)
{
    if (!ctx) return TB_ERR_INVALID;
    void* buf = tb_ctx_scratch(ctx, tb_gemv_mma_act_bytes(K, T));
    if (!buf) return TB_ERR_NOMEM;
    float* ys[2] = {swi, swi};
    const uint32_t* packs[2] = {gpack, upack};
    const uint16_t* scs[2] = {gscales, uscales};
    const int64_t Ns[2] = {I, I};
    return tb_gemv_mma_impl(ctx, 2, ys, packs, scs, Ns, x, norm_w16, eps, K, T, 0, false, true, buf);
}

TB_API int tb_gemv_tern_wgsl_mma(tb_ctx* ctx, float* y, const float* x, const uint16_t* norm_w16, float eps,
                                 const uint32_t* pack, const uint16_t* scales, int64_t N, int64_t K, int T, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    void* buf = tb_ctx_scratch(ctx, tb_gemv_mma_act_bytes(K, T));
    if (!buf) return TB_ERR_NOMEM;
    return tb_gemv_mma_impl(ctx, 1, &y, &pack, &scales, &N, x, norm_w16, eps, K, T, acc, true, false, buf);
}

TB_API int tb_gateup_silu_tern_wgsl_mma(tb_ctx* ctx, float* swi, const float* x, const uint16_t* norm_w16,
                                        float eps, const uint32_t* gpack, const uint16_t* gscales,
                                        const uint32_t* upack, const uint16_t* uscales, int64_t I, int64_t K, int T)
{
    if (!ctx) return TB_ERR_INVALID;
    void* buf = tb_ctx_scratch(ctx, tb_gemv_mma_act_bytes(K, T));
    if (!buf) return TB_ERR_NOMEM;
    float* ys[2] = {swi, swi};
    const uint32_t* packs[2] = {gpack, upack};
    const uint16_t* scs[2] = {gscales, uscales};
    const int64_t Ns[2] = {I, I};
    return tb_gemv_mma_impl(ctx, 2, ys, packs, scs, Ns, x, norm_w16, eps, K, T, 0, true, true, buf);
}

}  // extern "C"
