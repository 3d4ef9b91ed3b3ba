// tb_attn_dev.cuh -- device code of the int8-KV decode attention shared by the
// standalone kernels (tb_attn.cu) and the persistent decode-step kernel
// (tb_step.cu): the attnPrepQ8 math (qwen3.js:2228-2296), the KV quantization
// (pack4x8snorm, qwen3.js:2180-2210), and one split of the split-KV decode with
// the combine of ATTN_DEC_COMBINE (qwen3.js:2048-2069).  One copy of this code
// means the two paths compute bit-identical attention.
#pragma once
#include "tb_act.cuh"

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

// Barrier of the threads sharing a computation: bar 0 is the whole CTA, bar id >
// 0 a group of nthr threads (one split unit) of a larger CTA.
__device__ __forceinline__ void unit_sync(int bar, int nthr = ATT_THREADS)
{
    if (bar == 0) __syncthreads();
    else asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthr) : "memory");
}

// Per-head RMSNorm (w16) + RoPE of x (thread j holds element j of the head,
// threads j >= hd hold nothing); every thread of the block (bar 0) or of the
// 128-thread group (bar > 0) calls it.  rk: hd floats of shared memory, red: 8.
__device__ __forceinline__ float norm_rope(float x, const uint16_t* w16, int hd, float eps, float c, float s, float* rk,
                                           float* red, int j = threadIdx.x, int bar = 0, int nthr = ATT_THREADS)
{
    const int lane = j & 31, wid = j >> 5, nw = hd >> 5;
    const float ss = warp_sum(j < hd ? x * x : 0.0f);
    if (lane == 0 && wid < nw) red[wid] = ss;
    unit_sync(bar, nthr);
    float t = 0.0f;
    for (int i = 0; i < nw; i++) t += red[i];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)hd), eps)));
    if (j < hd) rk[j] = __fmul_rn(__fmul_rn(x, inv), tb_h2f(w16[j]));
    unit_sync(bar, nthr);
    float y = 0.0f;
    if (j < hd) {
        const int half = hd >> 1;
        const float partner = j < half ? rk[j + half] : rk[j - half];
        const float rot = j < half ? -partner : partner;
        y = fmaf(rk[j], c, rot * s);
    }
    unit_sync(bar, nthr);    // rk and red may be reused
    return y;
}

// norm_rope of several heads at once, the same arithmetic per head: thread t
// holds element t % hd of head slot t / hd (nthr threads, nthr % hd == 0, hd %
// 32 == 0); each head's warp sums are added in warp order as above.  rk: nthr
// floats, red: nthr / 32.
__device__ __forceinline__ float norm_rope_heads(float x, const uint16_t* w16, int hd, float eps, float c, float s,
                                                 float* rk, float* red, int t, int bar, int nthr)
{
    const int lane = t & 31, nw = hd >> 5, slot = t / hd, j = t - slot * hd;
    const float ss = warp_sum(x * x);
    if (lane == 0) red[t >> 5] = ss;
    unit_sync(bar, nthr);
    float tot = 0.0f;
    for (int i = 0; i < nw; i++) tot += red[slot * nw + i];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)hd), eps)));
    rk[t] = __fmul_rn(__fmul_rn(x, inv), tb_h2f(w16[j]));
    unit_sync(bar, nthr);
    const int half = hd >> 1;
    const float partner = j < half ? rk[t + half] : rk[t - half];
    const float rot = j < half ? -partner : partner;
    const float y = fmaf(rk[t], c, rot * s);
    unit_sync(bar, nthr);
    return y;
}

// snorm int8 of one 32-group per warp (pack4x8snorm of x / max(1e-12, maxabs))
// into row dq / scales ds (element j of the head at dq[j], group scale at ds[j/32])
__device__ __forceinline__ void quant_row(float x, int hd, int8_t* dq, float* ds, int j = threadIdx.x)
{
    const int lane = j & 31;
    if ((j >> 5) >= (hd >> 5)) return;
    const float m = fmaxf(1e-12f, warp_max(fabsf(x)));
    dq[j] = snorm8(__fdiv_rn(x, m));
    if (lane == 0) ds[j >> 5] = m;
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
    // optional: the heads' outputs also QUANTQ8'd in the tensor-core GEMVs' fragment
    // order (row slot = sequence, ts slots), for the o projection that follows
    unsigned char* mxa;
    uint2* mxk;
    int mts, mtern;
};

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

// Shared-memory layout of one split unit (4 warps; dynamic, bytes).  Each warp
// owns NST stages; a stage holds one tile of 32 keys: K rows, V rows (HD bytes
// each, 16-byte chunk i of key j stored at chunk i ^ (j % KV16) so the per-key
// 16-byte copies and reads are bank-conflict free), then the 32 keys' K and V
// group scales.
template <int HD, int GRP, int NST_, int W = ATT_WARPS>
struct DecLayout {
    static constexpr int KV16 = HD / 16, NG = HD / 32, NST = NST_, NT = 32 * W;
    // splits the combining unit can weigh (its [GRP][nsplit] weights live in the stages)
    static constexpr int MAXSPLIT = NST == 1 ? 256 : ATT_MAXSPLIT;
    static constexpr int ST_K = 0, ST_V = 32 * HD, ST_KS = 64 * HD, ST_VS = 64 * HD + 32 * NG * 4;
    static constexpr int STAGE = 64 * HD + 64 * NG * 4;
    static constexpr int OFF_QS = 0;                                  // float [GRP][HD]
    static constexpr int OFF_PS = OFF_QS + GRP * HD * 4;              // float [W][32 keys][NG][GRP]
    static constexpr int OFF_WM = OFF_PS + W * 32 * NG * GRP * 4;   // float [W][GRP]
    static constexpr int OFF_WL = OFF_WM + W * GRP * 4;       // float [W][GRP]
    static constexpr int OFF_ST = (OFF_WL + W * GRP * 4 + 127) / 128 * 128;
    // q's four int8 digits [GRP][4][HD] replace q itself (OFF_QS) once it is split, and
    // their steps [GRP][NG] sit in the merge scratch (OFF_WM, unused until the merge)
    static_assert(GRP * 4 * HD <= GRP * HD * 4 && GRP * NG <= 2 * W * GRP, "q digits must fit");
    static constexpr int BYTES = OFF_ST + W * NST * STAGE;
    // after the key loop the stages are reused for the warps' outputs, float [W][GRP][HD]
    static_assert(W * GRP * HD * 4 <= W * NST * STAGE, "merge buffer must fit in the stages");
    static_assert(STAGE % 16 == 0 && ST_KS % 16 == 0 && ST_VS % 16 == 0, "stage alignment");
    // the combining unit keeps its split weights [GRP][nsplit] there too
    static_assert(GRP * MAXSPLIT * 4 + (GRP * HD / 4 > NT ? GRP * HD / 4 : NT) * 16 <= W * NST * STAGE,
                  "split weights and column partials must fit in the stages");
};

// One (kv head, split) of the split-KV decode, run by 4 warps (tid 0..127).
// Warp w takes the 32-key tiles w, w+4, w+8, ... of the split: with NST = 2 a
// cp.async pipeline (tile j+1 in flight while tile j is scored), with NST = 1
// one stage (tile j+1 requested after tile j is consumed).  Lane = key for the
// scores (K row from shared memory against q held in shared memory, packed
// f32x2 FMAs); the lane's key then writes p * vscale / 127 per V group, and
// P.V runs lane = 4 dims (2 for hd 64) over the tile's keys.  Softmax is online
// per warp; the 4 warps merge at the end into the split's partial (PO, PML);
// the last split of the kv head to finish combines all of them.
//
// prefetch(early) requests each warp's first tile -- with early, not the tile
// holding row S-1 (written by the step's own prep); run(early) requests that
// one and does the rest.  The position (dpos) must not change in between.
// attnPrepQ8 folded into a unit (the persistent decode step): the unit computes
// its GRP q heads' norm + RoPE into shared memory itself, and the unit whose
// split holds row pos = S-1 also writes that row of the cache (k: norm + RoPE +
// int8, v: int8), before any warp requests it.
struct PrepIn {
    const float *q, *k, *v;          // this step's projections
    const uint16_t *qn, *kn;         // q / k norm weights
    const float* cs;                 // cos [HD], sin [HD] at pos
    float eps;
};

template <int HD, int GRP, int NST, int W = ATT_WARPS>
struct DecUnit {
    using L = DecLayout<HD, GRP, NST, W>;
    static constexpr int KV16 = L::KV16, NG = L::NG, NT = 32 * W;
    static constexpr int DPL = HD / 32;                // dims per lane in P.V

    const AttnArgs& a;
    uint8_t* smem;
    int hk, split, zb, tid, lane, wid, bar;
    // persistent step: the unit runs the prep, and row S-1 of a first tile is
    // written into the stage by the prep instead of copied (inject)
    const PrepIn* prep = nullptr;
    bool inject = false;
    // persistent step: the combining unit also stores its heads' outputs QUANTQ8'd
    // in the GEMV activation layout (qG groups), so the o phase copies instead of
    // quantizing
    unsigned char* qout = nullptr;
    int qG = 0;
    bool qnat = false;                  // qout in the ternary GEMVs' natural-order layout
    // the multi-kernel batched step: the outputs also in the tensor-core GEMVs' fragment
    // order (a.mxa; groups of 8 lanes, so GRP * HD / 4 is a multiple of 32)
    unsigned long long* tr = nullptr;   // optional %globaltimer stamps of the unit's stages (8 slots)

    __device__ void ts(int k) const
    {
        if (tr && tid == 0) {
            unsigned long long t;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
            tr[k] = t;
        }
    }
    long long row_elems, row_groups;
    const int8_t* Kq;
    const int8_t* Vq;
    const float* Ks;
    const float* Vs;
    int S, c0, c1, ntile;

    __device__ DecUnit(const AttnArgs& a_, uint8_t* smem_, int hk_, int split_, int zb_, int tid_, int bar_)
        : a(a_), smem(smem_), hk(hk_), split(split_), zb(zb_), tid(tid_), lane(tid_ & 31), wid(tid_ >> 5), bar(bar_)
    {
        row_elems = (long long)a.nKv * HD;
        row_groups = row_elems / 32;
        Kq = a.Kq + zb * a.cache_rows * row_elems;
        Vq = a.Vq + zb * a.cache_rows * row_elems;
        Ks = a.Ks + zb * a.cache_rows * row_groups;
        Vs = a.Vs + zb * a.cache_rows * row_groups;
        S = a.S;
        if (a.dpos) {
            S = a.dpos[zb] + 1;
            if (S < 1 || S > a.cache_rows) {
                if (tid == 0) atomicExch(a.err, ERR_ATTN_POS);
                S = 0;   // every split empty: the output row is written as zeros
            }
        }
        const int per = (S + a.nsplit - 1) / a.nsplit;
        c0 = split * per;
        c1 = min(S, c0 + per);
        const int span = c1 - c0;
        ntile = span > wid * 32 ? (span - wid * 32 + W * 32 - 1) / (W * 32) : 0;
    }

    __device__ uint8_t* stages() const { return smem + L::OFF_ST + wid * NST * L::STAGE; }

    // tile j of this warp -> stage s; always commits a group (possibly empty).
    // Rows are copied coalesced: in copy r, lanes 8q..8q+7 (4q..4q+3 for hd 64)
    // move the KV16 16-byte chunks of key r*RPI + q.  Scales: lane = key.
    __device__ void issue(int j, int s, int skip = -1) const
    {
        constexpr int RPI = 32 / KV16;                  // rows per copy instruction
        const int tb0 = c0 + (wid + W * j) * 32;
        uint8_t* st = stages() + s * L::STAGE;
        const int ch = lane % KV16;
#pragma unroll
        for (int r = 0; r < KV16; r++) {
            const int kr = r * RPI + lane / KV16;
            if (tb0 + kr < c1 && tb0 + kr != skip) {
                const long long src = (long long)(tb0 + kr) * row_elems + hk * HD + ch * 16;
                const int dst = (kr * KV16 + (ch ^ (kr & (KV16 - 1)))) * 16;
                cp_async16(st + L::ST_K + dst, Kq + src);
                cp_async16(st + L::ST_V + dst, Vq + src);
            }
        }
        const int t = tb0 + lane;
        if (t < c1 && t != skip) {
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
    }

    // does this warp's first tile hold row S-1?
    __device__ bool first_new() const
    {
        const int last = S - 1, t00 = c0 + wid * 32;
        return ntile > 0 && t00 <= last && last < t00 + 32;
    }

    __device__ void prefetch(bool early) const
    {
        if (!(early && first_new())) issue(0, 0);
        else if (inject) issue(0, 0, S - 1);     // every row but S-1, which the prep writes
    }

    __device__ void run(bool early) const
    {
        float* qs = reinterpret_cast<float*>(smem + L::OFF_QS);
        float* ps_all = reinterpret_cast<float*>(smem + L::OFF_PS);
        float* wm = reinterpret_cast<float*>(smem + L::OFF_WM);
        float* wl = reinterpret_cast<float*>(smem + L::OFF_WL);
        const float* qrow = a.qr + (long long)zb * a.nHq * HD;
        float* PO = a.PO + (long long)zb * a.nHq * a.nsplit * HD;
        float* PML = a.PML + (long long)zb * a.nHq * a.nsplit * 2;
        float* outp = a.out + (long long)zb * a.nHq * HD;
        unsigned* counter = a.counters + (long long)zb * a.nKv + hk;
        uint8_t* stg = stages();
        float* ps = ps_all + wid * 32 * NG * GRP;

        const float qscale = rsqrtf((float)HD) * (1.0f / 127.0f);
        ts(0);
        if (prep) {
            // the stages may still be receiving prefetched tiles: work in ps / wm
            float* rk = ps_all;
            float* red = wm;
            const int j = tid % HD, slot = tid / HD;
            constexpr int SLOTS = NT / HD;             // heads prepared side by side
            const float c = prep->cs[j], sn = prep->cs[HD + j];
            for (int h0 = 0; h0 < GRP; h0 += SLOTS) {
                const int h = h0 + slot;
                const long long o = (long long)zb * a.nHq * HD + (long long)(hk * GRP + (h < GRP ? h : 0)) * HD;
                const float x = h < GRP ? __ldcg(prep->q + o + j) : 0.0f;
                const float y = norm_rope_heads(x, prep->qn, HD, prep->eps, c, sn, rk, red, tid, bar, NT);
                if (h < GRP) qs[h * HD + j] = y;
            }
            ts(1);
            const int last = S - 1;
            // the warp whose FIRST tile holds row S-1 gets it straight into its stage
            const int wl = S > 0 ? (last - c0) >> 5 : W;
            const bool into_stage = inject && early && S > 0 && c0 <= last && last < c1 && wl < W;
            if (S > 0 && c0 <= last && last < c1) {
                // k (norm + RoPE) in head slot 0, v in slot 1 (or after k with one slot)
                const long long o = (long long)zb * a.nKv * HD + (long long)hk * HD;
                const long long row = (long long)last * row_elems + (long long)hk * HD;
                for (int part = 0; part < 2; part += SLOTS) {
                    const int which = part + slot;       // 0: k, 1: v
                    const float x = which < 2 ? __ldcg((which ? prep->v : prep->k) + o + j) : 0.0f;
                    const float kr = norm_rope_heads(x, prep->kn, HD, prep->eps, c, sn, rk, red, tid, bar, NT);
                    const float val = which == 0 ? kr : x;
                    // quant_row's values, into the cache and (into_stage) the stage of warp wl
                    const float m = fmaxf(1e-12f, warp_max(fabsf(val)));
                    const int8_t q8 = snorm8(__fdiv_rn(val, m));
                    if (which < 2) {
                        const_cast<int8_t*>(which ? Vq : Kq)[row + j] = q8;
                        if (lane == 0) const_cast<float*>(which ? Vs : Ks)[row / 32 + (j >> 5)] = m;
                        if (into_stage) {
                            uint8_t* st = smem + L::OFF_ST + wl * NST * L::STAGE;
                            const int kr_ = last - (c0 + wl * 32), ch = j >> 4;
                            const int off = (kr_ * KV16 + (ch ^ (kr_ & (KV16 - 1)))) * 16 + (j & 15);
                            st[(which ? L::ST_V : L::ST_K) + off] = (uint8_t)q8;
                            if (lane == 0)
                                reinterpret_cast<float*>(st + (which ? L::ST_VS : L::ST_KS))[kr_ * NG + (j >> 5)] = m;
                        }
                    }
                }
                if (!into_stage) __threadfence();    // the row reaches L2 before a warp's cp.async reads it
            }
            unit_sync(bar, NT);
            ts(2);
            if (early && first_new() && !inject) issue(0, 0);
        } else {
            if (early && first_new()) issue(0, 0);
            for (int i = tid; i < GRP * HD; i += NT) qs[i] = __ldcg(qrow + (long long)hk * GRP * HD + i);
            unit_sync(bar, NT);
        }

        // ---- q as four int8 digits per (head, 32-group): q = sc (d1 + d2/128 + d3/128^2 +
        // d4/128^3), sc = max|q|/127, each digit the rounded residual (below f32 rounding).
        // The scores then run on the tensor cores with K as the raw int8 operand.
        constexpr int NN8 = (GRP * 4 + 7) / 8;            // 8-column tiles of (head, digit)
        uint32_t qb[NN8][NG][2];                          // B fragments: column g, dims 4t.. / 16+4t..
        float qst[NN8][NG][2];                            // digit steps of this thread's two columns
        {
            int8_t* qd = reinterpret_cast<int8_t*>(smem + L::OFF_QS);   // overwrites q
            float* qsc = wm;
            constexpr int PPW = (GRP * NG + W - 1) / W;                  // (head, group) pairs a warp
            float qv[PPW];
#pragma unroll
            for (int i = 0; i < PPW; i++) {
                const int pr = wid + i * W;
                qv[i] = pr < GRP * NG ? qs[(pr / NG) * HD + 32 * (pr % NG) + lane] : 0.0f;
            }
            unit_sync(bar, NT);          // every q value is in registers: q's area takes the digits
#pragma unroll
            for (int i = 0; i < PPW; i++) {
                const int pr = wid + i * W;
                if (pr >= GRP * NG) break;
                const int h = pr / NG, G = pr - h * NG;
                float r = qv[i];
                float stp = q8_scale(warp_max(fabsf(r))), istp = q8_inv(stp);
                if (lane == 0) qsc[h * NG + G] = stp;
#pragma unroll
                for (int d = 0; d < 4; d++) {
                    const int q = max(-127, min(127, __float2int_rn(__fmul_rn(r, istp))));
                    r = __fsub_rn(r, __fmul_rn(stp, (float)q));
                    qd[(h * 4 + d) * HD + 32 * G + lane] = (int8_t)q;
                    stp = __fmul_rn(stp, 0.0078125f);
                    istp = __fmul_rn(istp, 128.0f);
                }
            }
            unit_sync(bar, NT);
            const int g8 = lane >> 2, t4 = lane & 3;
#pragma unroll
            for (int nt = 0; nt < NN8; nt++) {
                const int hb = (8 * nt + g8) >> 2, db = (8 * nt + g8) & 3;     // this thread's B column
                const int hc = 2 * nt + (t4 >> 1);                              // its D columns' head
#pragma unroll
                for (int G = 0; G < NG; G++) {
                    const int8_t* src = qd + (hb * 4 + db) * HD + 32 * G + 4 * t4;
                    qb[nt][G][0] = hb < GRP ? *reinterpret_cast<const uint32_t*>(src) : 0u;
                    qb[nt][G][1] = hb < GRP ? *reinterpret_cast<const uint32_t*>(src + 16) : 0u;
                    const float sc = hc < GRP ? qsc[hc * NG + G] : 0.0f;
                    // digits 2(t&1) and 2(t&1)+1: sc / 128^d (exact power-of-two steps)
                    qst[nt][G][0] = (t4 & 1) ? __fmul_rn(sc, 1.0f / 16384.0f) : sc;
                    qst[nt][G][1] = (t4 & 1) ? __fmul_rn(sc, 1.0f / 2097152.0f) : __fmul_rn(sc, 0.0078125f);
                }
            }
        }

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
            if constexpr (NST > 1) issue(j + 1, (j + 1) % NST);
            cp_async_wait<NST - 1>();
            __syncwarp();
            const uint8_t* st = stg + (j % NST) * L::STAGE;
            const int t0 = c0 + (wid + W * j) * 32;
            const bool valid = t0 + lane < c1;
            const int nk = min(32, c1 - t0);

            // ---- scores on the tensor cores: D[key][(head, digit)] = sum_32 K * digit per
            // group (mma m16n8k32, K the int8 A operand straight from the swizzled tile,
            // seeded with 2^23 + 2^22 so the int32 sum converts exactly), scaled by the
            // digit steps and the key's group scale; the two digit pairs of a head meet by
            // one shuffle, and lane = key picks its scores up from shared memory
            float s[GRP];
            {
                const int g8 = lane >> 2, t4 = lane & 3;
                const uint8_t* kb = st + L::ST_K;
                const float* ksd = reinterpret_cast<const float*>(st + L::ST_KS);
                float part[2][NN8][2];
#pragma unroll
                for (int mt = 0; mt < 2; mt++)
#pragma unroll
                    for (int nt = 0; nt < NN8; nt++) part[mt][nt][0] = part[mt][nt][1] = 0.0f;
#pragma unroll
                for (int G = 0; G < NG; G++) {
#pragma unroll
                    for (int mt = 0; mt < 2; mt++) {
                        const int k0 = 16 * mt + g8, k1 = k0 + 8;
                        const int c0 = 2 * G, c1 = 2 * G + 1;
                        uint32_t af[4];
                        af[0] = *reinterpret_cast<const uint32_t*>(kb + k0 * HD + ((c0 ^ (k0 & (KV16 - 1))) << 4) + 4 * t4);
                        af[1] = *reinterpret_cast<const uint32_t*>(kb + k1 * HD + ((c0 ^ (k1 & (KV16 - 1))) << 4) + 4 * t4);
                        af[2] = *reinterpret_cast<const uint32_t*>(kb + k0 * HD + ((c1 ^ (k0 & (KV16 - 1))) << 4) + 4 * t4);
                        af[3] = *reinterpret_cast<const uint32_t*>(kb + k1 * HD + ((c1 ^ (k1 & (KV16 - 1))) << 4) + 4 * t4);
                        const float ks0 = ksd[k0 * NG + G], ks1 = ksd[k1 * NG + G];
#pragma unroll
                        for (int nt = 0; nt < NN8; nt++) {
                            int dd[4];
                            asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
                                "{%8,%9}, {%10,%10,%10,%10};"
                                : "=r"(dd[0]), "=r"(dd[1]), "=r"(dd[2]), "=r"(dd[3])
                                : "r"(af[0]), "r"(af[1]), "r"(af[2]), "r"(af[3]), "r"(qb[nt][G][0]),
                                  "r"(qb[nt][G][1]), "r"(0x4B400000));
                            const float2 v0 = fadd2(make_float2(__int_as_float(dd[0]), __int_as_float(dd[1])),
                                                    make_float2(-12582912.0f, -12582912.0f));
                            const float2 v1 = fadd2(make_float2(__int_as_float(dd[2]), __int_as_float(dd[3])),
                                                    make_float2(-12582912.0f, -12582912.0f));
                            const float w0 = fmaf(v0.y, qst[nt][G][1], v0.x * qst[nt][G][0]);
                            const float w1 = fmaf(v1.y, qst[nt][G][1], v1.x * qst[nt][G][0]);
                            part[mt][nt][0] = fmaf(ks0, w0, part[mt][nt][0]);
                            part[mt][nt][1] = fmaf(ks1, w1, part[mt][nt][1]);
                        }
                    }
                }
                float* scs = ps;      // [32 keys][GRP] scores, before ps holds the V weights
#pragma unroll
                for (int mt = 0; mt < 2; mt++)
#pragma unroll
                    for (int nt = 0; nt < NN8; nt++) {
                        const float p0 = part[mt][nt][0] + __shfl_xor_sync(0xffffffffu, part[mt][nt][0], 1);
                        const float p1 = part[mt][nt][1] + __shfl_xor_sync(0xffffffffu, part[mt][nt][1], 1);
                        const int h = 2 * nt + (t4 >> 1);
                        if ((t4 & 1) == 0 && h < GRP) {
                            scs[(16 * mt + g8) * GRP + h] = p0;
                            scs[(16 * mt + g8 + 8) * GRP + h] = p1;
                        }
                    }
                __syncwarp();
#pragma unroll
                for (int h = 0; h < GRP; h++) s[h] = scs[lane * GRP + h];
                __syncwarp();         // ps is rewritten below
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
                    for (int h = 0; h < GRP; h++)
                        o[h][DPL / 2 - 1] = ffma2(v23, make_float2(pw[h], pw[h]), o[h][DPL / 2 - 1]);
                }
            }
            __syncwarp();   // stage j % NST and ps are rewritten next
            if constexpr (NST == 1) {
                if (j + 1 < ntile) issue(j + 1, 0);
            }
        }
        cp_async_wait<0>();
        unit_sync(bar, NT);    // every warp is done with its stages: reuse them for the merge
        ts(3);

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
        unit_sync(bar, NT);
        for (int i = tid; i < GRP * HD; i += NT) {
            const int h = i / HD, d = i - h * HD;
            float M = NEG_BIG;
#pragma unroll
            for (int w = 0; w < W; w++) M = fmaxf(M, wm[w * GRP + h]);
            float Ls = 0.0f, O = 0.0f;
#pragma unroll
            for (int w = 0; w < W; w++) {
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
        if (a.nsplit == 1) {
            if (qout || a.mxa) {     // the heads' outputs, written above by this unit, QUANTQ8'd
                unit_sync(bar, NT);
                constexpr int NC = GRP * HD / 4;
                for (int col = tid; col < NC; col += NT) {
                    const int h = col / (HD / 4), c4 = col - h * (HD / 4);
                    const float4 r = __ldcg(reinterpret_cast<const float4*>(outp + (long long)(hk * GRP + h) * HD) + c4);
                    const float e4[4] = {r.x, r.y, r.z, r.w};
                    const int gq = ((hk * GRP + h) * (HD / 4) + c4) >> 3;
                    if (qout) q8_store_group4(e4, gq, true, qout, qG, qnat);
                    else mma_store_group4(e4, gq, zb, a.mts, a.mtern != 0, a.mxa, a.mxk);
                }
            }
            return;
        }
        ts(4);

        // ---- the last split of this kv head to finish combines all of them
        //      (ATTN_DEC_COMBINE, qwen3.js:2048-2069): out = sum_i e_i O_i / sum_i e_i l_i,
        //      e_i = exp(m_i - max m).  Partials are read through L2 (ld.cg).  The
        //      arrival is one acquire-release add by thread 0 after the unit's barrier:
        //      it publishes the unit's partial (every thread's stores precede the
        //      barrier) and, in the last unit, makes every other unit's visible.
        unit_sync(bar, NT);
        int* last = reinterpret_cast<int*>(wm);          // wm/wl are free again after the loop above
        if (tid == 0) {
            unsigned old;
            asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(counter) : "memory");
            *last = old == (unsigned)(a.nsplit - 1);
        }
        unit_sync(bar, NT);
        ts(5);
        if (tr && tid == 0) tr[7] = *last;
        if (!*last) return;
        float* wts = reinterpret_cast<float*>(smem + L::OFF_ST);    // [GRP][nsplit]
        float* lsum = wl;                                            // [GRP]
        // float4 columns (head h, dims 4c..4c+3); when there are fewer columns than
        // threads, P threads share a column, each summing every P-th split, and the
        // P partials are added in part order.  With one (column, part) per thread
        // and at most 8 splits a thread, its partials are requested here, before
        // the split weights are known (the sums keep their order).
        constexpr int NCOL = GRP * HD / 4;
        constexpr int P = NCOL >= NT ? 1 : NT / NCOL;
        constexpr int PRE = 8;
        const bool pre = NCOL * P == NT && a.nsplit <= PRE * P;
        float4 pv[PRE];
        if (pre) {
            const int col = tid % NCOL, pp = tid / NCOL;
            const int h = col / (HD / 4), c4 = col - h * (HD / 4);
            const float4* po = reinterpret_cast<const float4*>(PO + (long long)(hk * GRP + h) * a.nsplit * HD) + c4;
#pragma unroll
            for (int u = 0; u < PRE; u++)
                if (pp + u * P < a.nsplit) pv[u] = __ldcg(po + (long long)(pp + u * P) * (HD / 4));
        }
        for (int h = wid; h < GRP && a.nsplit > 256; h += W) {   // many splits: two passes
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
        for (int h = wid; h < GRP && a.nsplit <= 256; h += W) {
            // each split's (m, l) pair read once (at most 8 a lane)
            const float2* pml = reinterpret_cast<const float2*>(PML + (long long)(hk * GRP + h) * a.nsplit * 2);
            float2 ml[8];
            float M = NEG_BIG;
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int i = lane + 32 * u;
                ml[u] = i < a.nsplit ? __ldcg(pml + i) : make_float2(NEG_BIG, 0.0f);
                M = fmaxf(M, ml[u].x);
            }
            M = warp_max(M);
            float Ls = 0.0f;
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const int i = lane + 32 * u;
                if (i < a.nsplit) {
                    const float e = __expf(ml[u].x - M);
                    wts[h * a.nsplit + i] = e;
                    Ls = fmaf(ml[u].y, e, Ls);
                }
            }
            Ls = warp_sum(Ls);
            if (lane == 0) lsum[h] = Ls;
        }
        unit_sync(bar, NT);
        float4* part = reinterpret_cast<float4*>(wts + GRP * L::MAXSPLIT);     // [P][NCOL]
        if (pre) {
            const int col = tid % NCOL, pp = tid / NCOL;
            const int h = col / (HD / 4);
            const float* w = wts + h * a.nsplit;
            float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
            for (int u = 0; u < PRE; u++) {
                const int k = pp + u * P;
                if (k < a.nsplit) {
                    const float e = w[k];
                    acc.x = fmaf(pv[u].x, e, acc.x); acc.y = fmaf(pv[u].y, e, acc.y);
                    acc.z = fmaf(pv[u].z, e, acc.z); acc.w = fmaf(pv[u].w, e, acc.w);
                }
            }
            part[pp * NCOL + col] = acc;
        }
        for (int i = pre ? NCOL * P : tid; i < NCOL * P; i += NT) {
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
        unit_sync(bar, NT);
        for (int col = tid; col < NCOL; col += NT) {
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
            if (qout || a.mxa) {     // 8 consecutive columns = one 32-group, 8 consecutive lanes
                const float e4[4] = {res.x, res.y, res.z, res.w};
                const int gq = ((hk * GRP + h) * (HD / 4) + c4) >> 3;
                if (qout) q8_store_group4(e4, gq, true, qout, qG, qnat);
                else mma_store_group4(e4, gq, zb, a.mts, a.mtern != 0, a.mxa, a.mxk);
            }
        }
        if (tid == 0) *counter = 0u;     // ready for the next call
        ts(6);
    }
};

}  // namespace
