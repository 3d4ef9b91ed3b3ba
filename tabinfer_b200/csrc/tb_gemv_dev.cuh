// tb_gemv_dev.cuh -- device code of the decode GEMVs shared by the standalone
// GEMV kernels (tb_gemv.cu) and the persistent decode-step kernel (tb_step.cu):
// the bulk-copy and mbarrier primitives, the activation staging (optional
// RMSNorm + the per-32 int8 quantization of QUANTQ8, models/qwen3.js:332-358,
// 569-621) and the per-group dot products.  One copy of this code means the
// two paths compute bit-identical activations and row sums.
#pragma once
#include "tb_act.cuh"

namespace {

constexpr int THREADS = 256;
constexpr int MAX_NST = 4;
constexpr int SMEM_HDR = 512;   // mbarriers (64 B) + reduction scratch (>= 72 floats)
constexpr uint32_t WAIT_TRIES = 1000;
constexpr int ERR_WAIT_TIMEOUT = 0x6d01;

enum Kind { KIND_Q8 = 0, KIND_GATEUP = 1, KIND_F32 = 2, KIND_TERN = 3, KIND_GATEUP_TERN = 4, KIND_F32D = 5 };
__host__ __device__ constexpr bool kind_tern(int k) { return k == KIND_TERN || k == KIND_GATEUP_TERN; }
__host__ __device__ constexpr bool kind_gateup(int k) { return k == KIND_GATEUP || k == KIND_GATEUP_TERN; }
enum ActSrc { ACT_PREQ = 0, ACT_F32 = 1, ACT_RMSNORM = 2 };

struct Mat {
    const uint32_t* pack;
    const uint16_t* scales;
    float* y;
    int N;
    int rb_begin;   // first row block of this matrix
};

struct Args {
    Mat m[4];
    int count, nrb, RB, K, acc;
    int wrow_bytes;        // packed weight bytes per row: K/2 (int4) or K/4 (ternary)
    int act_src;
    const float* x;        // f32 [B][K] (ACT_F32 / ACT_RMSNORM)
    const int8_t* xq;      // int8 [B][K]   (ACT_PREQ)
    const float* xs;       // f32 [B][K/32] (ACT_PREQ)
    const uint16_t* normw; // f16 [K]       (ACT_RMSNORM)
    float eps;
    int nst;
    int slot_bytes;        // bytes of one matrix's row block in a stage (weights, then scales)
    int act_bytes;         // staged activation (Q8 or f32 layout)
    int xbuf_bytes;        // f32 staging of raw rows for the Q8 prologue
    int nw_bytes;          // f16 RMSNorm weight, prefetched before the wait
    int* err;
};

// ---- mbarrier / bulk-copy primitives ------------------------------------------
__device__ __forceinline__ uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(saddr(dst)), "l"(src), "r"(bytes), "r"(saddr(bar)) : "memory");
}
// Bounded wait: try_wait suspends until the phase completes (woken at once) or
// its 1 ms hint runs out; WAIT_TRIES tries bound the whole wait to ~1 s.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity)
{
    for (uint32_t i = 0; i < WAIT_TRIES; i++) {
        uint32_t ok;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
                     " selp.u32 %0, 1, 0, p;\n}"
                     : "=r"(ok) : "r"(saddr(bar)), "r"(parity), "r"(1000000u) : "memory");
        if (ok) return true;
    }
    return false;
}


// ---- row-block bookkeeping --------------------------------------------------
struct Block {
    int mi, row0, nrows;
};
__device__ __forceinline__ Block block_of(const Args& a, int rb, bool gateup)
{
    int mi = 0;
    if (!gateup) {
#pragma unroll
        for (int i = 1; i < 4; i++) if (i < a.count && rb >= a.m[i].rb_begin) mi = i;
    }
    const Mat& M = a.m[mi];
    int row0 = (rb - M.rb_begin) * a.RB;
    return Block{mi, row0, min(a.RB, M.N - row0)};
}

// Scales of a block travel by bulk copy when their byte count is a multiple of 16.
__device__ __forceinline__ bool scales_bulk(int nrows, int G) { return ((nrows * G * 2) & 15) == 0; }

__device__ void issue_block(const Args& a, int rb, unsigned char* stage, uint64_t* bar, bool gateup)
{
    const int G = a.K >> 5;
    const Block bl = block_of(a, rb, gateup);
    const uint32_t wb = (uint32_t)bl.nrows * a.wrow_bytes;
    const uint32_t sb = (uint32_t)bl.nrows * G * 2;
    const bool sbulk = scales_bulk(bl.nrows, G);
    const int nm = gateup ? 2 : 1;
    mbar_expect_tx(bar, nm * (wb + (sbulk ? sb : 0u)));
    for (int s = 0; s < nm; s++) {
        const Mat& M = a.m[gateup ? s : bl.mi];
        unsigned char* dst = stage + s * a.slot_bytes;
        bulk_g2s(dst, reinterpret_cast<const unsigned char*>(M.pack) + (size_t)bl.row0 * a.wrow_bytes, wb, bar);
        if (sbulk) bulk_g2s(dst + (size_t)a.RB * a.wrow_bytes, M.scales + (size_t)bl.row0 * G, sb, bar);
    }
}

// ---- activation staging -------------------------------------------------------
// All of an activation row is requested at once (coalesced float4 loads, many in
// flight per thread) before any of it is used: the prologue costs one memory
// round trip, not one per 32-group.

// Index of element i of row b in the swizzled f32 layout (per (b, g) 8 float4,
// float4 index XOR-swizzled by (g & 7)).
__device__ __forceinline__ int swz_index(int G, int b, int i)
{
    const int f = i >> 2, g = f >> 3, j = f & 7;
    return ((b * G + g) * 8 + (j ^ (g & 7))) * 4 + (i & 3);
}

// Copy nb rows of K4 float4 from global into the swizzled shared layout and
// accumulate each row's sum of squares in the canonical order (thread t:
// float4 t, t+256, ... of the row).  Loads are issued in batches of 8 per
// thread before any store, so a batch costs one memory round trip.  COH: the
// rows were written by other CTAs of a still-running kernel, so they are read
// through L2 (ld.global.cg) instead of the read-only path.
template <int B, bool COH = false>
__device__ __forceinline__ void load_rows_swz(const float4* __restrict__ src, int nb, int K4, float4* dst, float* ss)
{
    constexpr int LPT = 8;
    const int tid = threadIdx.x;
    const int kpt = (K4 + THREADS - 1) / THREADS;   // float4 per thread per row
    const int n_items = nb * kpt;
#pragma unroll
    for (int b = 0; b < B; b++) ss[b] = 0.0f;
    for (int u0 = 0; u0 < n_items; u0 += LPT) {
        float4 v[LPT];
#pragma unroll
        for (int u = 0; u < LPT; u++) {
            const int it = u0 + u, bb = it / kpt, f = (it - bb * kpt) * THREADS + tid;
            if (it < n_items && f < K4) v[u] = COH ? __ldcg(src + (size_t)bb * K4 + f) : __ldg(src + (size_t)bb * K4 + f);
        }
#pragma unroll
        for (int u = 0; u < LPT; u++) {
            const int it = u0 + u, bb = it / kpt, f = (it - bb * kpt) * THREADS + tid;
            if (it < n_items && f < K4) {
                const int g = f >> 3, j = f & 7;
                dst[bb * K4 + g * 8 + (j ^ (g & 7))] = v[u];
#pragma unroll
                for (int b = 0; b < B; b++)
                    if (b == bb) ss[b] = sumsq_f4(v[u], ss[b]);
            }
        }
    }
}

// Q8 layout per (b, g): lo = (e0,o0,e1,o1), hi = (e2,o2,e3,o3) (e_w / o_w = even /
// odd k of weight word w, one int8 per byte), s8 = 8*sum(x), sf = scale.
// NAT (ternary weights): lo / hi = x[0..15] / x[16..31] in natural order and
// s8 = sum(x).
template <int B, bool NAT, bool COH = false>
__device__ void stage_q8(const Args& a, unsigned char* act, float* xbuf, int xbuf_floats, float* red,
                         const uint16_t* nws)
{
    const int G = a.K >> 5;
    uint4* xlo = reinterpret_cast<uint4*>(act);
    uint4* xhi = xlo + B * G;
    int* xs8 = reinterpret_cast<int*>(xhi + B * G);
    float* xsf = reinterpret_cast<float*>(xs8 + B * G);
    const int tid = threadIdx.x;
    if (a.act_src == ACT_PREQ) {
        for (int i = tid; i < B * G; i += THREADS) {
            const int b = i / G, g = i - b * G;
            const uint4* src = reinterpret_cast<const uint4*>(a.xq + (size_t)b * a.K + g * 32);
            const uint4 p = src[0], q = src[1];
            const uint32_t w[8] = {p.x, p.y, p.z, p.w, q.x, q.y, q.z, q.w};
            uint32_t e[4], o[4];
            int s = 0;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                e[j] = __byte_perm(w[2 * j], w[2 * j + 1], 0x6420);
                o[j] = __byte_perm(w[2 * j], w[2 * j + 1], 0x7531);
                s = __dp4a((int)w[2 * j], 0x01010101, s);
                s = __dp4a((int)w[2 * j + 1], 0x01010101, s);
            }
            if (NAT) {
                xlo[i] = p;
                xhi[i] = q;
                xs8[i] = s;
            } else {
                xlo[i] = make_uint4(e[0], o[0], e[1], o[1]);
                xhi[i] = make_uint4(e[2], o[2], e[3], o[3]);
                xs8[i] = 8 * s;
            }
            xsf[i] = a.xs[(size_t)b * G + g];
        }
        return;
    }
    // f32 rows -> swizzled shared copy (one burst of loads, the RMSNorm sums of
    // squares accumulated on the way in, canonical order of tb_act.cuh); then
    // 2 threads per (row, 32-group), one pass: thread h of the pair owns k =
    // 16h..16h+15, i.e. exactly the permuted dp4a half `lo` (h = 0) or `hi`.
    const int K4 = a.K >> 2;
    const int rows_per_chunk = max(1, xbuf_floats / a.K);
    float4* xb4 = reinterpret_cast<float4*>(xbuf);
    const int h2 = tid & 1;
    for (int b0 = 0; b0 < B; b0 += rows_per_chunk) {
        const int nb = min(rows_per_chunk, B - b0);
        const float4* src = reinterpret_cast<const float4*>(a.x + (size_t)b0 * a.K);
        float ss[B], inv[B];
        load_rows_swz<B, COH>(src, nb, K4, xb4, ss);
        if (a.act_src == ACT_RMSNORM) {
            block256_reduce_rows<B>(ss, red, inv);   // includes the __syncthreads for xb4
#pragma unroll
            for (int b = 0; b < B; b++) inv[b] = rms_inv(inv[b], a.K, a.eps);
        } else {
            __syncthreads();
#pragma unroll
            for (int b = 0; b < B; b++) inv[b] = 1.0f;
        }
        // both threads of a pair run the same number of passes (shuffles stay converged)
        for (int base = 0; base < nb * G * 2; base += THREADS) {
            const int item = (base + tid) >> 1;
            const bool live = item < nb * G;
            const int bb = live ? item / G : 0, g = live ? item - bb * G : 0;
            float v[16];
            {
                const float4* xg = xb4 + bb * K4 + g * 8;
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    const float4 t = xg[(4 * h2 + q) ^ (g & 7)];
                    v[4 * q] = t.x; v[4 * q + 1] = t.y; v[4 * q + 2] = t.z; v[4 * q + 3] = t.w;
                }
            }
            if (a.act_src == ACT_RMSNORM) {
                float ib = inv[0];
#pragma unroll
                for (int b = 1; b < B; b++) if (bb == b) ib = inv[b];
                const uint4* wq = reinterpret_cast<const uint4*>(nws + g * 32 + 16 * h2);
#pragma unroll
                for (int q = 0; q < 2; q++) {
                    const uint4 wv = wq[q];
                    const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                    for (int h = 0; h < 4; h++) {
                        const int k = 8 * q + 2 * h;
                        v[k] = __fmul_rn(__fmul_rn(v[k], ib), tb_h2f((uint16_t)(ww[h] & 0xffffu)));
                        v[k + 1] = __fmul_rn(__fmul_rn(v[k + 1], ib), tb_h2f((uint16_t)(ww[h] >> 16)));
                    }
                }
            }
            float m[4];
#pragma unroll
            for (int i = 0; i < 4; i++) m[i] = fmaxf(fmaxf(fabsf(v[i]), fabsf(v[i + 4])), fmaxf(fabsf(v[i + 8]), fabsf(v[i + 12])));
            float mx = fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3]));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
            const float scale = q8_scale(mx), is = q8_inv(scale);
            uint32_t wd[4];
            int sum = 0;
            if (NAT) {
#pragma unroll
                for (int w = 0; w < 4; w++) {
                    uint32_t n = 0;
#pragma unroll
                    for (int h = 0; h < 4; h++) {
                        const int qv = q8_quant(v[4 * w + h], is);
                        sum += qv;
                        n |= ((uint32_t)qv & 0xffu) << (8 * h);
                    }
                    wd[w] = n;
                }
            } else {
#pragma unroll
                for (int w = 0; w < 2; w++) {
                    uint32_t e = 0, o = 0;
#pragma unroll
                    for (int h = 0; h < 4; h++) {
                        const int qe = q8_quant(v[8 * w + 2 * h], is), qo = q8_quant(v[8 * w + 2 * h + 1], is);
                        sum += qe + qo;
                        e |= ((uint32_t)qe & 0xffu) << (8 * h);
                        o |= ((uint32_t)qo & 0xffu) << (8 * h);
                    }
                    wd[2 * w] = e;
                    wd[2 * w + 1] = o;
                }
            }
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            if (live) {
                const int i = (b0 + bb) * G + g;
                (h2 ? xhi : xlo)[i] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
                if (h2 == 0) { xs8[i] = NAT ? sum : 8 * sum; xsf[i] = scale; }
            }
        }
        __syncthreads();   // xbuf and red are reused by the next chunk
    }
}

// One f32 row (gemvQ, batch 1) as four int8 digit vectors, so the int4 dot
// runs on dp4a instead of a float conversion per weight.  Per 32-group: sc =
// max|x|/127, d1 = rn(x/sc), then each next digit rounds the remaining residual
// at 128 times finer steps: x = sc*(d1 + d2/128 + d3/128^2 + d4/128^3) within
// sc/2^22 (1.9e-9 of the group's largest magnitude, below f32 rounding).  The
// digit vectors are stored in the permuted Q8 layout of stage_q8; c1 = 8*sum d1
// and c234 = 8*(16384*sum d2 + 128*sum d3 + sum d4) remove the nibble bias (the
// weight is nib - 8); xsf = sc/2^21.  The group dot is then, in exact integers,
// t1 = dot(nib, d1) - c1 and t234 = 16384*dot(nib, d2) + 128*dot(nib, d3) +
// dot(nib, d4) - c234, and (s16 * xsf) * (2^21*t1 + t234) with two f32 roundings.
// Layout: per digit d a lo and a hi uint4 plane [8][G], c1 [G], c234 [G] (int), xsf [G].
constexpr int F32D_ND = 4;
constexpr int F32D_BYTES_PER_GROUP = 2 * F32D_ND * 16 + 3 * 4;
__device__ void stage_f32d(const Args& a, unsigned char* act, float* xbuf, float* red, const uint16_t* nws)
{
    const int G = a.K >> 5, K4 = a.K >> 2;
    uint4* xd = reinterpret_cast<uint4*>(act);       // [2*ND][G]
    int* c1 = reinterpret_cast<int*>(xd + 2 * F32D_ND * G);
    int* c234 = c1 + G;
    float* xsf = reinterpret_cast<float*>(c234 + G);
    const int tid = threadIdx.x, h2 = tid & 1;
    float4* xb4 = reinterpret_cast<float4*>(xbuf);
    float ss[1], inv[1];
    load_rows_swz<1>(reinterpret_cast<const float4*>(a.x), 1, K4, xb4, ss);
    if (a.act_src == ACT_RMSNORM) {
        block256_reduce_rows<1>(ss, red, inv);   // includes the __syncthreads for xb4
        inv[0] = rms_inv(inv[0], a.K, a.eps);
    } else {
        __syncthreads();
        inv[0] = 1.0f;
    }
    // 2 threads per 32-group: thread h2 of the pair owns k = 16 h2 .. 16 h2 + 15
    for (int base = 0; base < G * 2; base += THREADS) {
        const int item = (base + tid) >> 1;
        const bool live = item < G;
        const int g = live ? item : 0;
        float v[16];
        {
            const float4* xg = xb4 + g * 8;
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float4 t = xg[(4 * h2 + q) ^ (g & 7)];
                v[4 * q] = t.x; v[4 * q + 1] = t.y; v[4 * q + 2] = t.z; v[4 * q + 3] = t.w;
            }
        }
        if (a.act_src == ACT_RMSNORM) {
            const uint4* wq = reinterpret_cast<const uint4*>(nws + g * 32 + 16 * h2);
#pragma unroll
            for (int q = 0; q < 2; q++) {
                const uint4 wv = wq[q];
                const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
                for (int h = 0; h < 4; h++) {
                    const int k = 8 * q + 2 * h;
                    v[k] = __fmul_rn(__fmul_rn(v[k], inv[0]), tb_h2f((uint16_t)(ww[h] & 0xffffu)));
                    v[k + 1] = __fmul_rn(__fmul_rn(v[k + 1], inv[0]), tb_h2f((uint16_t)(ww[h] >> 16)));
                }
            }
        }
        float mx = 0.0f;
#pragma unroll
        for (int i = 0; i < 16; i++) mx = fmaxf(mx, fabsf(v[i]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        // digit d: step sc / 128^d and its inverse (exact power-of-two scalings)
        float stp[F32D_ND], istp[F32D_ND];
        stp[0] = q8_scale(mx);
        istp[0] = q8_inv(stp[0]);
#pragma unroll
        for (int d = 1; d < F32D_ND; d++) {
            stp[d] = __fmul_rn(stp[d - 1], 0.0078125f);
            istp[d] = __fmul_rn(istp[d - 1], 128.0f);
        }
        uint32_t dw[F32D_ND][4];
        int sums[F32D_ND] = {};
#pragma unroll
        for (int w = 0; w < 2; w++) {
            uint32_t e[F32D_ND] = {}, o[F32D_ND] = {};
#pragma unroll
            for (int h = 0; h < 4; h++) {
#pragma unroll
                for (int par = 0; par < 2; par++) {
                    float r = v[8 * w + 2 * h + par];
#pragma unroll
                    for (int d = 0; d < F32D_ND; d++) {
                        const int q = max(-127, min(127, __float2int_rn(__fmul_rn(r, istp[d]))));
                        r = __fsub_rn(r, __fmul_rn(stp[d], (float)q));
                        sums[d] += q;
                        const uint32_t b = ((uint32_t)q & 0xffu) << (8 * h);
                        if (par) o[d] |= b; else e[d] |= b;
                    }
                }
            }
#pragma unroll
            for (int d = 0; d < F32D_ND; d++) { dw[d][2 * w] = e[d]; dw[d][2 * w + 1] = o[d]; }
        }
#pragma unroll
        for (int d = 0; d < F32D_ND; d++) sums[d] += __shfl_xor_sync(0xffffffffu, sums[d], 1);
        if (live) {
#pragma unroll
            for (int d = 0; d < F32D_ND; d++)
                xd[(2 * d + h2) * G + g] = make_uint4(dw[d][0], dw[d][1], dw[d][2], dw[d][3]);
            if (h2 == 0) {
                c1[g] = 8 * sums[0];
                c234[g] = 8 * (16384 * sums[1] + 128 * sums[2] + sums[3]);
                xsf[g] = stp[F32D_ND - 1];   // sc / 128^3 = sc / 2^21
            }
        }
    }
    __syncthreads();
}

// The four-digit activation of one 32-group (stage_f32d).
struct XD {
    uint4 d[F32D_ND][2];     // digit vector, lo / hi half of the permuted layout
    int c1, c234;
    float sf;
};
__device__ __forceinline__ void load_xd(XD& x, const unsigned char* act, int G, int g)
{
    const uint4* xd = reinterpret_cast<const uint4*>(act);
#pragma unroll
    for (int d = 0; d < F32D_ND; d++) {
        x.d[d][0] = xd[(2 * d) * G + g];
        x.d[d][1] = xd[(2 * d + 1) * G + g];
    }
    const int* c1 = reinterpret_cast<const int*>(xd + 2 * F32D_ND * G);
    x.c1 = c1[g];
    x.c234 = c1[G + g];
    x.sf = reinterpret_cast<const float*>(c1 + 2 * G)[g];
}
// int4 word quadruple (32 nibbles) against the four digit vectors: exact
// integer sums, two f32 roundings, one FMA a group
__device__ __forceinline__ void item_f32d(const uint4 w, const float s, const XD& x, float* acc)
{
    const uint32_t nl[4] = {w.x & 0x0f0f0f0fu, w.y & 0x0f0f0f0fu, w.z & 0x0f0f0f0fu, w.w & 0x0f0f0f0fu};
    const uint32_t nh[4] = {(w.x >> 4) & 0x0f0f0f0fu, (w.y >> 4) & 0x0f0f0f0fu, (w.z >> 4) & 0x0f0f0f0fu,
                            (w.w >> 4) & 0x0f0f0f0fu};
    int dd[F32D_ND];
#pragma unroll
    for (int d = 0; d < F32D_ND; d++) {
        const uint4 lo = x.d[d][0], hi = x.d[d][1];
        int p0 = 0, p1 = 0;
        p0 = __dp4a((int)nl[0], (int)lo.x, p0);
        p1 = __dp4a((int)nh[0], (int)lo.y, p1);
        p0 = __dp4a((int)nl[1], (int)lo.z, p0);
        p1 = __dp4a((int)nh[1], (int)lo.w, p1);
        p0 = __dp4a((int)nl[2], (int)hi.x, p0);
        p1 = __dp4a((int)nh[2], (int)hi.y, p1);
        p0 = __dp4a((int)nl[3], (int)hi.z, p0);
        p1 = __dp4a((int)nh[3], (int)hi.w, p1);
        dd[d] = p0 + p1;
    }
    // |dd| <= 32*15*127 = 60960: t234 < 2^31, 2^21 * t1 exact as a float
    const int t1 = dd[0] - x.c1;
    const int t234 = 16384 * dd[1] + 128 * dd[2] + dd[3] - x.c234;
    const float t = fmaf((float)t1, 2097152.0f, (float)t234);
    *acc = fmaf(s * x.sf, t, *acc);
}

// F32 layout: per (b, g) 8 float4, float4 index XOR-swizzled by (g & 7).
template <int B>
__device__ void stage_f32(const Args& a, unsigned char* act, float* red, const uint16_t* nws)
{
    const int G = a.K >> 5, K4 = a.K >> 2;
    float4* xsm = reinterpret_cast<float4*>(act);
    float ss[B], inv[B];
    load_rows_swz<B>(reinterpret_cast<const float4*>(a.x), B, K4, xsm, ss);
    if (a.act_src != ACT_RMSNORM) { __syncthreads(); return; }
    block256_reduce_rows<B>(ss, red, inv);
#pragma unroll
    for (int b = 0; b < B; b++) inv[b] = rms_inv(inv[b], a.K, a.eps);
    float* xf = reinterpret_cast<float*>(act);
    for (int i = threadIdx.x; i < a.K; i += THREADS) {
        const float w = tb_h2f(nws[i]);
#pragma unroll
        for (int b = 0; b < B; b++) {
            float* p = xf + swz_index(G, b, i);
            *p = __fmul_rn(__fmul_rn(*p, inv[b]), w);
        }
    }
    __syncthreads();
}

// ---- per-item math ----------------------------------------------------------------
template <int B>
__device__ __forceinline__ void item_q8(const uint4 w, const float s, const unsigned char* act, int G, int g, float* acc)
{
    const uint4* xlo = reinterpret_cast<const uint4*>(act);
    const uint4* xhi = xlo + B * G;
    const int* xs8 = reinterpret_cast<const int*>(xhi + B * G);
    const float* xsf = reinterpret_cast<const float*>(xs8 + B * G);
    const uint32_t l0 = w.x & 0x0f0f0f0fu, h0 = (w.x >> 4) & 0x0f0f0f0fu;
    const uint32_t l1 = w.y & 0x0f0f0f0fu, h1 = (w.y >> 4) & 0x0f0f0f0fu;
    const uint32_t l2 = w.z & 0x0f0f0f0fu, h2 = (w.z >> 4) & 0x0f0f0f0fu;
    const uint32_t l3 = w.w & 0x0f0f0f0fu, h3 = (w.w >> 4) & 0x0f0f0f0fu;
#pragma unroll
    for (int b = 0; b < B; b++) {
        const int i = b * G + g;
        const uint4 xl = xlo[i], xh = xhi[i];
        // four independent chains (the integer sum is the same in any order)
        int d0 = -xs8[i], d1 = 0, d2 = 0, d3 = 0;
        d0 = __dp4a((int)l0, (int)xl.x, d0);
        d1 = __dp4a((int)h0, (int)xl.y, d1);
        d2 = __dp4a((int)l1, (int)xl.z, d2);
        d3 = __dp4a((int)h1, (int)xl.w, d3);
        d0 = __dp4a((int)l2, (int)xh.x, d0);
        d1 = __dp4a((int)h2, (int)xh.y, d1);
        d2 = __dp4a((int)l3, (int)xh.z, d2);
        d3 = __dp4a((int)h3, (int)xh.w, d3);
        const int d = (d0 + d1) + (d2 + d3);
        acc[b] = fmaf(s * xsf[i], (float)d, acc[b]);
    }
}

// The int8 activation of one 32-group for all B rows, loaded once and shared by
// the several weight rows a warp carries.
template <int B>
struct XQ {
    uint4 lo[B], hi[B];
    int s8[B];
    float sf[B];
};
template <int B>
__device__ __forceinline__ void load_xq(XQ<B>& x, const unsigned char* act, int G, int g)
{
    const uint4* xlo = reinterpret_cast<const uint4*>(act);
    const uint4* xhi = xlo + B * G;
    const int* xs8 = reinterpret_cast<const int*>(xhi + B * G);
    const float* xsf = reinterpret_cast<const float*>(xs8 + B * G);
#pragma unroll
    for (int b = 0; b < B; b++) {
        const int i = b * G + g;
        x.lo[b] = xlo[i];
        x.hi[b] = xhi[i];
        x.s8[b] = xs8[i];
        x.sf[b] = xsf[i];
    }
}
// int4 word quadruple (32 nibbles) against the permuted int8 layout
template <int B>
__device__ __forceinline__ void item_q8x(const uint4 w, const float s, const XQ<B>& x, float* acc)
{
    const uint32_t l0 = w.x & 0x0f0f0f0fu, h0 = (w.x >> 4) & 0x0f0f0f0fu;
    const uint32_t l1 = w.y & 0x0f0f0f0fu, h1 = (w.y >> 4) & 0x0f0f0f0fu;
    const uint32_t l2 = w.z & 0x0f0f0f0fu, h2 = (w.z >> 4) & 0x0f0f0f0fu;
    const uint32_t l3 = w.w & 0x0f0f0f0fu, h3 = (w.w >> 4) & 0x0f0f0f0fu;
#pragma unroll
    for (int b = 0; b < B; b++) {
        // four independent chains (the integer sum is the same in any order)
        int d0 = -x.s8[b], d1 = 0, d2 = 0, d3 = 0;
        d0 = __dp4a((int)l0, (int)x.lo[b].x, d0);
        d1 = __dp4a((int)h0, (int)x.lo[b].y, d1);
        d2 = __dp4a((int)l1, (int)x.lo[b].z, d2);
        d3 = __dp4a((int)h1, (int)x.lo[b].w, d3);
        d0 = __dp4a((int)l2, (int)x.hi[b].x, d0);
        d1 = __dp4a((int)h2, (int)x.hi[b].y, d1);
        d2 = __dp4a((int)l3, (int)x.hi[b].z, d2);
        d3 = __dp4a((int)h3, (int)x.hi[b].w, d3);
        const int d = (d0 + d1) + (d2 + d3);
        acc[b] = fmaf(s * x.sf[b], (float)d, acc[b]);
    }
}
// ternary group (two code words) against the natural-order int8 layout
template <int B>
__device__ __forceinline__ void item_ternx(const uint2 w, const float s, const XQ<B>& x, float* acc)
{
    constexpr uint32_t M = 0x03030303u;
    const uint32_t a0 = w.x & M, a1 = (w.x >> 2) & M, a2 = (w.x >> 4) & M, a3 = (w.x >> 6) & M;
    const uint32_t c0 = w.y & M, c1 = (w.y >> 2) & M, c2 = (w.y >> 4) & M, c3 = (w.y >> 6) & M;
#pragma unroll
    for (int b = 0; b < B; b++) {
        // four independent chains (the integer sum is the same in any order)
        int d0 = -x.s8[b], d1 = 0, d2 = 0, d3 = 0;
        d0 = __dp4a((int)a0, (int)x.lo[b].x, d0);
        d1 = __dp4a((int)a1, (int)x.lo[b].y, d1);
        d2 = __dp4a((int)a2, (int)x.lo[b].z, d2);
        d3 = __dp4a((int)a3, (int)x.lo[b].w, d3);
        d0 = __dp4a((int)c0, (int)x.hi[b].x, d0);
        d1 = __dp4a((int)c1, (int)x.hi[b].y, d1);
        d2 = __dp4a((int)c2, (int)x.hi[b].z, d2);
        d3 = __dp4a((int)c3, (int)x.hi[b].w, d3);
        const int d = (d0 + d1) + (d2 + d3);
        acc[b] = fmaf(s * x.sf[b], (float)d, acc[b]);
    }
}

// One ternary 32-group (two code words) against the natural-order int8 row:
// sum (c-1)*x = sum_s dp4a((word >> 2s) & 0x03030303, x word s) - sum(x).
template <int B>
__device__ __forceinline__ void item_tern(const uint2 w, const float s, const unsigned char* act, int G, int g, float* acc)
{
    const uint4* xlo = reinterpret_cast<const uint4*>(act);
    const uint4* xhi = xlo + B * G;
    const int* xsum = reinterpret_cast<const int*>(xhi + B * G);
    const float* xsf = reinterpret_cast<const float*>(xsum + B * G);
    constexpr uint32_t M = 0x03030303u;
    const uint32_t a0 = w.x & M, a1 = (w.x >> 2) & M, a2 = (w.x >> 4) & M, a3 = (w.x >> 6) & M;
    const uint32_t c0 = w.y & M, c1 = (w.y >> 2) & M, c2 = (w.y >> 4) & M, c3 = (w.y >> 6) & M;
#pragma unroll
    for (int b = 0; b < B; b++) {
        const int i = b * G + g;
        const uint4 xl = xlo[i], xh = xhi[i];
        // four independent chains (the integer sum is the same in any order)
        int d0 = -xsum[i], d1 = 0, d2 = 0, d3 = 0;
        d0 = __dp4a((int)a0, (int)xl.x, d0);
        d1 = __dp4a((int)a1, (int)xl.y, d1);
        d2 = __dp4a((int)a2, (int)xl.z, d2);
        d3 = __dp4a((int)a3, (int)xl.w, d3);
        d0 = __dp4a((int)c0, (int)xh.x, d0);
        d1 = __dp4a((int)c1, (int)xh.y, d1);
        d2 = __dp4a((int)c2, (int)xh.z, d2);
        d3 = __dp4a((int)c3, (int)xh.w, d3);
        const int d = (d0 + d1) + (d2 + d3);
        acc[b] = fmaf(s * xsf[i], (float)d, acc[b]);
    }
}

// One weight word (8 nibbles, k = 8wi..8wi+7) against x[k..k+7] = (xa, xb).
__device__ __forceinline__ float2 word_f32(uint32_t word, float4 xa, float4 xb, float2 d)
{
    const float2 M2 = make_float2(-8388616.0f, -8388616.0f);   // -(2^23 + 8)
    const uint32_t lo = word & 0x0f0f0f0fu, hi = (word >> 4) & 0x0f0f0f0fu;
    // 0x4B0000nn is the float 2^23 + nn; adding -(2^23+8) leaves nn - 8 exactly
    const float2 n01 = fadd2(make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7540)),
                                         __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7540))), M2);
    const float2 n23 = fadd2(make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7541)),
                                         __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7541))), M2);
    const float2 n45 = fadd2(make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7542)),
                                         __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7542))), M2);
    const float2 n67 = fadd2(make_float2(__uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7543)),
                                         __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7543))), M2);
    d = ffma2(n01, make_float2(xa.x, xa.y), d);
    d = ffma2(n23, make_float2(xa.z, xa.w), d);
    d = ffma2(n45, make_float2(xb.x, xb.y), d);
    d = ffma2(n67, make_float2(xb.z, xb.w), d);
    return d;
}

template <int B>
__device__ __forceinline__ void item_f32(const uint4 w, const float s, const unsigned char* act, int G, int g, float* acc)
{
    const float4* xsm = reinterpret_cast<const float4*>(act);
    const int sw = g & 7;
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int b = 0; b < B; b++) {
        const float4* xr = xsm + (b * G + g) * 8;
        float2 d = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int wi = 0; wi < 4; wi++) d = word_f32(ww[wi], xr[(2 * wi) ^ sw], xr[(2 * wi + 1) ^ sw], d);
        acc[b] = fmaf(s, d.x + d.y, acc[b]);
    }
}

}  // namespace
