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

namespace {

constexpr int ATT_WARPS = 4;
constexpr int ATT_THREADS = ATT_WARPS * 32;
constexpr int ATT_MAXG = 8;       // q heads per kv head handled by one CTA
constexpr int ATT_MAXSPLIT = 1024; // splits per decode call
constexpr float NEG_BIG = -3.0e38f;

__device__ __forceinline__ int8_t snorm8(float v)
{
    float c = fminf(1.0f, fmaxf(-1.0f, v));
    return (int8_t)floorf(__fadd_rn(0.5f, __fmul_rn(127.0f, c)));
}

// Error word codes written by the attention kernels when a device-resident
// position is outside the cache (the host cannot check it).
constexpr int ERR_ATTN_POS = 0x6a01;

// ---- attnPrepQ8 math (qwen3.js:2228-2296) -----------------------------------
// RoPE angle of dimension j (split-half pairs j, j + hd/2) at position pos, in
// double: pos * theta^(-2 fi / hd).
__device__ __forceinline__ void rope_cs(int j, int hd, long long pos, float theta, float* c, float* s)
{
    const int half = hd >> 1;
    const int fi = j < half ? j : j - half;
    const double ang = (double)pos * pow((double)theta, -2.0 * (double)fi / (double)hd);
    double sd, cd;
    sincos(ang, &sd, &cd);
    *c = (float)cd;
    *s = (float)sd;
}

// Per-head RMSNorm (w16) + RoPE of x (thread j holds element j of the head,
// threads j >= hd hold nothing); every thread of the block calls it.  rk: hd
// floats of shared memory, red: 8.
__device__ __forceinline__ float norm_rope(float x, const uint16_t* w16, int hd, float eps, float c, float s, float* rk,
                                           float* red)
{
    const int j = threadIdx.x, lane = j & 31, wid = j >> 5, nw = hd >> 5;
    const float ss = warp_sum(j < hd ? x * x : 0.0f);
    if (lane == 0 && wid < nw) red[wid] = ss;
    __syncthreads();
    float t = 0.0f;
    for (int i = 0; i < nw; i++) t += red[i];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)hd), eps)));
    if (j < hd) rk[j] = __fmul_rn(__fmul_rn(x, inv), tb_h2f(w16[j]));
    __syncthreads();
    float y = 0.0f;
    if (j < hd) {
        const int half = hd >> 1;
        const float partner = j < half ? rk[j + half] : rk[j - half];
        const float rot = j < half ? -partner : partner;
        y = fmaf(rk[j], c, rot * s);
    }
    __syncthreads();   // rk and red may be reused
    return y;
}

// snorm int8 of one 32-group per warp (pack4x8snorm of x / max(1e-12, maxabs))
// into row dq / scales ds (element j of the head at dq[j], group scale at ds[j/32])
__device__ __forceinline__ void quant_row(float x, int hd, int8_t* dq, float* ds)
{
    const int j = threadIdx.x, lane = j & 31;
    if ((j >> 5) >= (hd >> 5)) return;
    const float m = fmaxf(1e-12f, warp_max(fabsf(x)));
    dq[j] = snorm8(__fdiv_rn(x, m));
    if (lane == 0) ds[j >> 5] = m;
}

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

// ---- split-KV decode --------------------------------------------------------
struct AttnArgs {
    const float* qr;       // [nHq*hd]
    const int8_t* Kq;
    const float* Ks;
    const int8_t* Vq;
    const float* Vs;
    float* PO;             // [nHq][nsplit][hd]
    float* PML;            // [nHq][nsplit][2]
    float* out;            // [nHq*hd]
    unsigned* counters;    // [B][nKv] split arrivals, zero between calls
    const int* dpos;       // [B] device positions (context S_b = dpos[b] + 1), or null: S for all
    int* err;              // device error word
    long long cache_rows;  // rows of each sequence's cache
    int S, nHq, nKv, nsplit;
    int grid_z;            // sequences
};

// k_attn_decode mode EARLY (the decode step): the position and every cache row
// below S-1 were written by earlier steps, so each warp's first tile is fetched
// before griddepcontrol.wait unless it holds row S-1, which the preceding prep
// kernel writes.

// ---- cp.async (16-byte and 8-byte global -> shared copies, per thread) -----
__device__ __forceinline__ void cp_async16(void* sdst, const void* gsrc)
{
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(sdst)),
                 "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async8(void* sdst, const void* gsrc)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"((uint32_t)__cvta_generic_to_shared(sdst)),
                 "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Shared-memory layout of k_attn_decode<HD, GRP> (dynamic, bytes).  Each warp
// owns NST stages; a stage holds one tile of 32 keys: K rows, V rows (HD bytes
// each, 16-byte chunk i of key j stored at chunk i ^ (j % KV16) so the per-key
// 16-byte copies and reads are bank-conflict free), then the 32 keys' K and V
// group scales.
template <int HD, int GRP>
struct DecLayout {
    static constexpr int KV16 = HD / 16, NG = HD / 32, NST = 2;
    static constexpr int ST_K = 0, ST_V = 32 * HD, ST_KS = 64 * HD, ST_VS = 64 * HD + 32 * NG * 4;
    static constexpr int STAGE = 64 * HD + 64 * NG * 4;
    static constexpr int OFF_QS = 0;                                  // float [GRP][HD]
    static constexpr int OFF_PS = OFF_QS + GRP * HD * 4;              // float [W][32 keys][NG][GRP]
    static constexpr int OFF_WM = OFF_PS + ATT_WARPS * 32 * NG * GRP * 4;   // float [W][GRP]
    static constexpr int OFF_WL = OFF_WM + ATT_WARPS * GRP * 4;       // float [W][GRP]
    static constexpr int OFF_ST = (OFF_WL + ATT_WARPS * GRP * 4 + 127) / 128 * 128;
    static constexpr int BYTES = OFF_ST + ATT_WARPS * NST * STAGE;
    // after the key loop the stages are reused for the warps' outputs, float [W][GRP][HD]
    static_assert(ATT_WARPS * GRP * HD * 4 <= ATT_WARPS * NST * STAGE, "merge buffer must fit in the stages");
    static_assert(STAGE % 16 == 0 && ST_KS % 16 == 0 && ST_VS % 16 == 0, "stage alignment");
    // the combining CTA keeps its split weights [GRP][nsplit] there too
    static_assert(GRP * ATT_MAXSPLIT * 4 + (GRP * HD / 4 > ATT_THREADS ? GRP * HD / 4 : ATT_THREADS) * 16 <=
                      ATT_WARPS * NST * STAGE,
                  "split weights and column partials must fit in the stages");
};

// hd fixed at compile time (64 or 128); GRP = q heads per kv head.
// CTA = 4 warps over one (kv head, split).  Warp w takes the 32-key tiles
// w, w+4, w+8, ... of the split and runs a two-stage cp.async pipeline over
// them: while tile j is scored, tile j+1's K rows, V rows and scales are in
// flight.  Lane = key for the scores (K row from shared memory against q held
// in shared memory, packed f32x2 FMAs); the lane's key then writes
// p * vscale / 127 per V group, and P.V runs lane = 4 dims (2 for hd 64)
// over the tile's keys.  Softmax is online per warp; the 4 warps merge at the
// end into the split's partial (PO, PML).
template <int HD, int GRP, bool EARLY>
__global__ void __launch_bounds__(ATT_THREADS) k_attn_decode(const AttnArgs a)
{
    using L = DecLayout<HD, GRP>;
    constexpr int KV16 = L::KV16, NG = L::NG, NST = L::NST;
    constexpr int DPL = HD / 32;                // dims per lane in P.V
    extern __shared__ __align__(128) uint8_t smem[];
    float* qs = reinterpret_cast<float*>(smem + L::OFF_QS);
    float* ps_all = reinterpret_cast<float*>(smem + L::OFF_PS);
    float* wm = reinterpret_cast<float*>(smem + L::OFF_WM);
    float* wl = reinterpret_cast<float*>(smem + L::OFF_WL);

    const int hk = blockIdx.x, split = blockIdx.y, zb = blockIdx.z;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const long long row_elems = (long long)a.nKv * HD, row_groups = row_elems / 32;
    // this CTA's sequence: its cache, q row, partials, output and counters
    const int8_t* Kq = a.Kq + zb * a.cache_rows * row_elems;
    const int8_t* Vq = a.Vq + zb * a.cache_rows * row_elems;
    const float* Ks = a.Ks + zb * a.cache_rows * row_groups;
    const float* Vs = a.Vs + zb * a.cache_rows * row_groups;
    const float* qrow = a.qr + (long long)zb * a.nHq * HD;
    float* PO = a.PO + (long long)zb * a.nHq * a.nsplit * HD;
    float* PML = a.PML + (long long)zb * a.nHq * a.nsplit * 2;
    float* outp = a.out + (long long)zb * a.nHq * HD;
    unsigned* counter = a.counters + (long long)zb * a.nKv + hk;
    if (!EARLY) {
        tb_pdl_wait();
        tb_pdl_trigger();
    }
    int S = a.S;
    if (a.dpos) {
        S = a.dpos[zb] + 1;
        if (S < 1 || S > a.cache_rows) {
            if (threadIdx.x == 0) atomicExch(a.err, ERR_ATTN_POS);
            S = 0;   // every split empty: the output row is written as zeros
        }
    }
    const int per = (S + a.nsplit - 1) / a.nsplit;
    const int c0 = split * per, c1 = min(S, c0 + per);
    const int span = c1 - c0;
    const int ntile = span > wid * 32 ? (span - wid * 32 + ATT_WARPS * 32 - 1) / (ATT_WARPS * 32) : 0;
    uint8_t* stages = smem + L::OFF_ST + wid * NST * L::STAGE;
    float* ps = ps_all + wid * 32 * NG * GRP;

    // tile j of this warp -> stage s; always commits a group (possibly empty).
    // Rows are copied coalesced: in copy r, lanes 8q..8q+7 (4q..4q+3 for hd 64)
    // move the KV16 16-byte chunks of key r*RPI + q.  Scales: lane = key.
    auto issue = [&](int j, int s) {
        constexpr int RPI = 32 / KV16;                  // rows per copy instruction
        const int tb0 = c0 + (wid + ATT_WARPS * j) * 32;
        uint8_t* st = stages + s * L::STAGE;
        const int ch = lane % KV16;
#pragma unroll
        for (int r = 0; r < KV16; r++) {
            const int kr = r * RPI + lane / KV16;
            if (tb0 + kr < c1) {
                const long long src = (long long)(tb0 + kr) * row_elems + hk * HD + ch * 16;
                const int dst = (kr * KV16 + (ch ^ (kr & (KV16 - 1)))) * 16;
                cp_async16(st + L::ST_K + dst, Kq + src);
                cp_async16(st + L::ST_V + dst, Vq + src);
            }
        }
        const int t = tb0 + lane;
        if (t < c1) {
            float* ksd = reinterpret_cast<float*>(st + L::ST_KS) + lane * NG;
            float* vsd = reinterpret_cast<float*>(st + L::ST_VS) + lane * NG;
            const float* ksr = Ks + (long long)t * row_groups + hk * NG;
            const float* vsr = Vs + (long long)t * row_groups + hk * NG;
            if (NG * 4 == 16) {
                cp_async16(ksd, ksr);
                cp_async16(vsd, vsr);
            } else {
#pragma unroll
                for (int g = 0; g < NG; g += 2) { cp_async8(ksd + g, ksr + g); cp_async8(vsd + g, vsr + g); }
            }
        }
        cp_async_commit();
    };

    const float qscale = rsqrtf((float)HD) * (1.0f / 127.0f);
    if constexpr (EARLY) {
        const int last = S - 1, t00 = c0 + wid * 32;
        const bool first_new = ntile > 0 && t00 <= last && last < t00 + 32;
        if (!first_new) issue(0, 0);
        tb_pdl_wait();
        tb_pdl_trigger();
        if (first_new) issue(0, 0);
    } else {
        issue(0, 0);
    }
    for (int i = threadIdx.x; i < GRP * HD; i += ATT_THREADS) qs[i] = qrow[(long long)hk * GRP * HD + i];
    __syncthreads();

    float m[GRP], l[GRP];
    float2 o[GRP][DPL / 2];
#pragma unroll
    for (int h = 0; h < GRP; h++) {
        m[h] = NEG_BIG; l[h] = 0.0f;
#pragma unroll
        for (int i = 0; i < DPL / 2; i++) o[h][i] = make_float2(0.0f, 0.0f);
    }
    const int gsel = (lane * DPL) / 32;               // V group of this lane's dims
    const int vc = (lane * DPL) >> 4, vcw = ((lane * DPL) & 15) / DPL;   // 16-byte chunk, word in chunk

    for (int j = 0; j < ntile; j++) {
        issue(j + 1, (j + 1) % NST);
        cp_async_wait<NST - 1>();
        __syncwarp();
        const uint8_t* st = stages + (j % NST) * L::STAGE;
        const int t0 = c0 + (wid + ATT_WARPS * j) * 32;
        const bool valid = t0 + lane < c1;
        const int nk = min(32, c1 - t0);

        // ---- scores: lane = key
        float s[GRP];
#pragma unroll
        for (int h = 0; h < GRP; h++) s[h] = 0.0f;
        if (valid) {
            const uint4* kd = reinterpret_cast<const uint4*>(st + L::ST_K) + lane * KV16;
            const float* ksd = reinterpret_cast<const float*>(st + L::ST_KS) + lane * NG;
#pragma unroll
            for (int g = 0; g < NG; g++) {
                float2 acc[GRP];
#pragma unroll
                for (int h = 0; h < GRP; h++) acc[h] = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int i2 = 0; i2 < 2; i2++) {
                    const int i = g * 2 + i2;
                    const uint4 w4 = kd[i ^ (lane & (KV16 - 1))];
                    const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                    for (int wq = 0; wq < 4; wq++) {
                        const float2 k01 = sbytes_f2(ww[wq], 0), k23 = sbytes_f2(ww[wq], 1);
                        const int d = i * 16 + wq * 4;
#pragma unroll
                        for (int h = 0; h < GRP; h++) {
                            const float4 q4 = *reinterpret_cast<const float4*>(qs + h * HD + d);
                            acc[h] = ffma2(make_float2(q4.x, q4.y), k01, acc[h]);
                            acc[h] = ffma2(make_float2(q4.z, q4.w), k23, acc[h]);
                        }
                    }
                }
                const float ksc = ksd[g];
#pragma unroll
                for (int h = 0; h < GRP; h++) s[h] = fmaf(acc[h].x + acc[h].y, ksc, s[h]);
            }
        }
        // ---- online softmax (per lane partial l; m warp-uniform)
        float pr[GRP];
#pragma unroll
        for (int h = 0; h < GRP; h++) {
            const float sc = valid ? s[h] * qscale : NEG_BIG;
            const float mn = fmaxf(m[h], warp_max(sc));
            const float corr = __expf(m[h] - mn);
            pr[h] = valid ? __expf(sc - mn) : 0.0f;
            l[h] = fmaf(l[h], corr, pr[h]);
            m[h] = mn;
#pragma unroll
            for (int i = 0; i < DPL / 2; i++) o[h][i] = make_float2(o[h][i].x * corr, o[h][i].y * corr);
        }
        // ---- this key's weights per V group: p * vscale / 127
        {
            const float* vsd = reinterpret_cast<const float*>(st + L::ST_VS) + lane * NG;
#pragma unroll
            for (int g = 0; g < NG; g++) {
                const float vsc = valid ? vsd[g] * (1.0f / 127.0f) : 0.0f;
#pragma unroll
                for (int h = 0; h < GRP; h++) ps[(lane * NG + g) * GRP + h] = pr[h] * vsc;
            }
        }
        __syncwarp();
        // ---- P.V: lane = DPL dims
        const uint4* vt = reinterpret_cast<const uint4*>(st + L::ST_V);
#pragma unroll 4
        for (int kk = 0; kk < nk; kk++) {
            const uint4* vrow = vt + kk * KV16 + (vc ^ (kk & (KV16 - 1)));
            const uint32_t vw = DPL == 4 ? reinterpret_cast<const uint32_t*>(vrow)[vcw]
                                         : (uint32_t)reinterpret_cast<const uint16_t*>(vrow)[vcw];
            const float* pp = ps + (kk * NG + gsel) * GRP;
            float pw[GRP];
#pragma unroll
            for (int h = 0; h < GRP; h++) pw[h] = pp[h];
            const float2 v01 = sbytes_f2(vw, 0);
#pragma unroll
            for (int h = 0; h < GRP; h++) o[h][0] = ffma2(v01, make_float2(pw[h], pw[h]), o[h][0]);
            if (DPL == 4) {
                const float2 v23 = sbytes_f2(vw, 1);
#pragma unroll
                for (int h = 0; h < GRP; h++) o[h][DPL / 2 - 1] = ffma2(v23, make_float2(pw[h], pw[h]), o[h][DPL / 2 - 1]);
            }
        }
        __syncwarp();   // stage j % NST and ps are rewritten next iteration
    }
    cp_async_wait<0>();
    __syncthreads();    // every warp is done with its stages: reuse them for the merge

    // ---- merge warps
    float* wo = reinterpret_cast<float*>(smem + L::OFF_ST);     // [W][GRP][HD]
#pragma unroll
    for (int h = 0; h < GRP; h++) {
        const float lt = warp_sum(l[h]);
        if (lane == 0) { wm[wid * GRP + h] = m[h]; wl[wid * GRP + h] = lt; }
#pragma unroll
        for (int i = 0; i < DPL / 2; i++)
            *reinterpret_cast<float2*>(wo + (wid * GRP + h) * HD + lane * DPL + 2 * i) = o[h][i];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < GRP * HD; i += ATT_THREADS) {
        const int h = i / HD, d = i - h * HD;
        float M = NEG_BIG;
#pragma unroll
        for (int w = 0; w < ATT_WARPS; w++) M = fmaxf(M, wm[w * GRP + h]);
        float Ls = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < ATT_WARPS; w++) {
            const float e = __expf(wm[w * GRP + h] - M);
            Ls = fmaf(wl[w * GRP + h], e, Ls);
            O = fmaf(wo[(w * GRP + h) * HD + d], e, O);
        }
        if (a.nsplit == 1) {
            outp[(long long)(hk * GRP + h) * HD + d] = Ls > 0.0f ? O / Ls : 0.0f;
        } else {
            const long long pidx = (long long)(hk * GRP + h) * a.nsplit + split;
            PO[pidx * HD + d] = O;
            if (d == 0) { PML[pidx * 2] = M; PML[pidx * 2 + 1] = Ls; }
        }
    }
    if (a.nsplit == 1) return;

    // ---- the last split of this kv head to finish combines all of them
    //      (ATTN_DEC_COMBINE, qwen3.js:2048-2069): out = sum_i e_i O_i / sum_i e_i l_i,
    //      e_i = exp(m_i - max m).  Partials are read through L2 (ld.cg).
    __threadfence();
    __syncthreads();
    int* last = reinterpret_cast<int*>(wm);          // wm/wl are free again after the loop above
    if (threadIdx.x == 0) *last = atomicAdd(counter, 1u) == (unsigned)(a.nsplit - 1);
    __syncthreads();
    if (!*last) return;
    __threadfence();
    float* wts = reinterpret_cast<float*>(smem + L::OFF_ST);    // [GRP][nsplit]
    float* lsum = wl;                                            // [GRP]
    for (int h = wid; h < GRP; h += ATT_WARPS) {
        const float* pml = PML + (long long)(hk * GRP + h) * a.nsplit * 2;
        float M = NEG_BIG;
        for (int i = lane; i < a.nsplit; i += 32) M = fmaxf(M, __ldcg(pml + 2 * i));
        M = warp_max(M);
        float Ls = 0.0f;
        for (int i = lane; i < a.nsplit; i += 32) {
            const float e = __expf(__ldcg(pml + 2 * i) - M);
            wts[h * a.nsplit + i] = e;
            Ls = fmaf(__ldcg(pml + 2 * i + 1), e, Ls);
        }
        Ls = warp_sum(Ls);
        if (lane == 0) lsum[h] = Ls;
    }
    __syncthreads();
    // float4 columns (head h, dims 4c..4c+3); when there are fewer columns than
    // threads, P threads share a column, each summing every P-th split with 8
    // loads in flight, and the P partials are added in part order.
    constexpr int NCOL = GRP * HD / 4;
    constexpr int P = NCOL >= ATT_THREADS ? 1 : ATT_THREADS / NCOL;
    float4* part = reinterpret_cast<float4*>(wts + GRP * ATT_MAXSPLIT);     // [P][NCOL]
    for (int i = threadIdx.x; i < NCOL * P; i += ATT_THREADS) {
        const int col = i % NCOL, pp = i / NCOL;
        const int h = col / (HD / 4), c4 = col - h * (HD / 4);
        const float4* po = reinterpret_cast<const float4*>(PO + (long long)(hk * GRP + h) * a.nsplit * HD) + c4;
        const float* w = wts + h * a.nsplit;
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        int k = pp;
        for (; k + 7 * P < a.nsplit; k += 8 * P) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = __ldcg(po + (long long)(k + u * P) * (HD / 4));
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const float e = w[k + u * P];
                acc.x = fmaf(v[u].x, e, acc.x); acc.y = fmaf(v[u].y, e, acc.y);
                acc.z = fmaf(v[u].z, e, acc.z); acc.w = fmaf(v[u].w, e, acc.w);
            }
        }
        for (; k < a.nsplit; k += P) {
            const float4 v = __ldcg(po + (long long)k * (HD / 4));
            const float e = w[k];
            acc.x = fmaf(v.x, e, acc.x); acc.y = fmaf(v.y, e, acc.y);
            acc.z = fmaf(v.z, e, acc.z); acc.w = fmaf(v.w, e, acc.w);
        }
        part[pp * NCOL + col] = acc;
    }
    __syncthreads();
    for (int col = threadIdx.x; col < NCOL; col += ATT_THREADS) {
        const int h = col / (HD / 4), c4 = col - h * (HD / 4);
        float4 O = part[col];
        for (int pp = 1; pp < P; pp++) {
            const float4 v = part[pp * NCOL + col];
            O.x += v.x; O.y += v.y; O.z += v.z; O.w += v.w;
        }
        const float Ls = lsum[h];
        const float4 res = Ls > 0.0f ? make_float4(O.x / Ls, O.y / Ls, O.z / Ls, O.w / Ls)
                                     : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        reinterpret_cast<float4*>(outp + (long long)(hk * GRP + h) * HD)[c4] = res;
    }
    if (threadIdx.x == 0) *counter = 0u;     // ready for the next call
}

template <int HD, int GRP, bool EARLY>
int launch_decode(tb_ctx* ctx, const AttnArgs& a)
{
    constexpr int bytes = DecLayout<HD, GRP>::BYTES;
    auto kern = k_attn_decode<HD, GRP, EARLY>;
    static bool attr_set[64] = {};   // per device and instantiation; setting it twice is harmless
    if (ctx->device >= 64 || !attr_set[ctx->device]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "attn_decode attribute: %s", cudaGetErrorString(e));
        if (ctx->device < 64) attr_set[ctx->device] = true;
    }
    cudaError_t e = tb_launch(ctx, kern, dim3(a.nKv, a.nsplit, a.grid_z), dim3(ATT_THREADS), bytes, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "attn_decode launch: %s", cudaGetErrorString(e));
    return TB_OK;
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
// CTA, and enough CTAs (nKv * nsplit) for ~2 per SM (the decode kernel's
// shared-memory occupancy) at long context.
int tb_attn_auto_nsplit(tb_ctx* ctx, int64_t S, int64_t nKv)
{
    long long by_keys = (S + 127) / 128;
    long long by_fill = (2LL * ctx->num_sms + nKv - 1) / nKv;
    long long n = std::min(by_keys, by_fill);
    return (int)std::max(1LL, std::min(n, 1024LL));
}

// batch sequences (grid.z); sequence b's cache starts cache_rows rows after
// sequence b-1's; with dpos, S_b = dpos[b] + 1 is read on the device.
int tb_attn_decode_impl(tb_ctx* ctx, float* out, const float* qr, const int8_t* Kq, const float* Ks,
                        const int8_t* Vq, const float* Vs, int64_t S, int64_t nHq, int64_t nKv, int64_t hd,
                        int nsplit, float* PO, float* PML, unsigned* counters, int64_t batch,
                        int64_t cache_rows, const int32_t* dpos, bool early)
{
    AttnArgs a{qr, Kq, Ks, Vq, Vs, PO, PML, out, counters, (const int*)dpos, ctx->dev_error,
               (long long)(cache_rows > 0 ? cache_rows : S), (int)S, (int)nHq, (int)nKv, nsplit};
    a.grid_z = (int)batch;
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
//    heads x hd 128, fits up to 126 splits); larger requests are rejected with
//    TB_ERR_INVALID before anything is enqueued.
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
    if (nsplit == 0) nsplit = tb_attn_auto_nsplit(ctx, S, nKv);
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
