// tb_step.cu -- the Qwen3 decode step (forward at T = 1, models/qwen3.js:3938-4069)
// for one sequence on one GPU as ONE persistent kernel: one CTA per SM, the
// layers' phases separated by grid barriers instead of kernel boundaries.
//
// Why: a decode step is ~170 small dependent kernels whose time is latency (each
// kernel's launch wait, its activation staging behind its own weight stream),
// not bandwidth.  Here every CTA owns a fixed slice of rows of every matrix and
// requests the weights of its NEXT phases into shared memory (cp.async.bulk,
// mbarrier completion) while the current phase runs, so when a barrier opens the
// weights are on chip and the phase costs the barrier, the activation staging and
// the arithmetic.
//
// Phases of layer l (barrier after each):
//   A  RMSNorm + QUANTQ8 of x, q/k/v rows (head-aligned 32-row blocks); the
//      last CTA of a head runs attnPrepQ8 for it (q: norm + RoPE into qr;
//      k: norm + RoPE + int8 row into the cache; v: int8 row)
//   B  split-KV attention: (kv head, split) units on 4-warp groups, two per CTA;
//      the last split of a kv head combines (DecUnit, the standalone kernel's code)
//   C  QUANTQ8 of the attention output, o rows, += residual
//   D  RMSNorm + QUANTQ8 of x, gate/up rows, SwiGLU
//   E  QUANTQ8 of swi, down rows, += residual
// Shared-memory buffers and what they hold, requested as soon as they are free:
//   R  A(l) -> C(l) -> A(l+1)   (requested at the end of A(l) / C(l))
//   P  B(l) key/value tiles (cp.async) -> D(l) gate/up (requested at the end of
//      B(l)) -> B(l+1) tiles (requested at the end of D(l))
//   Q  E(l) -> E(l+1)           (requested at the end of E(l))
// Every phase uses the standalone kernels' device code (tb_gemv_dev.cuh,
// tb_attn_dev.cuh) with the same split count, so the step is bit-identical to
// the multi-kernel step.  Barrier and copy waits are bounded; a CTA that gives up
// records the error, raises the launch's abort word, drains its copies and
// returns, and the others leave at their next barrier.
#include "tb_internal.h"
#include "tb_gemv_dev.cuh"
#include "tb_attn_dev.cuh"

namespace {

constexpr int ERR_STEP_BARRIER = 0x5101;
constexpr int ERR_STEP_COPY = 0x5102;
constexpr long long STEP_WAIT_LIMIT = 1LL << 21;   // barrier polls of ~0.5 us: ~1 s
constexpr int RBA = 32;                              // rows of a phase-A block (a head has hd/32 blocks)
constexpr int STEP_HD = 128;

struct StepLayer {
    const uint32_t* p[7];    // q, k, v, o, gate, up, down packs
    const uint16_t* s[7];    // their f16 scales
    const uint16_t *ln1, *ln2, *qn, *kn;
    int8_t *Kq, *Vq;
    float *Ks, *Vs;
};
enum { WQ = 0, WK, WV, WO, WG, WU, WD };

struct StepArgs {
    const StepLayer* layers;
    int L, H, nHq, nKv, I, nsplit, max_seq;
    float eps, theta;
    const uint32_t* ids;
    const int32_t* pos;
    const uint16_t* embed;
    float *x, *q, *k, *v, *qr, *attn, *swi, *PO, *PML;
    unsigned* counters;      // [nKv] split arrivals (zero between steps)
    unsigned* head_ctr;      // [nHq + 2 nKv] phase-A block arrivals (zero between steps)
    unsigned* bar_count;     // grid barrier: arrivals, generation
    unsigned* bar_gen;
    unsigned* abort_word;    // == this launch's tag: a CTA gave up in this launch
    int* err;
    // shared-memory layout (bytes)
    int off_P, off_Q, off_R, off_xbuf, off_act, off_misc;
    int xbuf_floats;
    int rpC, rpD;            // rows per CTA of o / down (rpC) and gate / up (rpD)
};

// ---- grid barrier ---------------------------------------------------------------
__device__ __forceinline__ void st_release_gpu(unsigned* p, unsigned v)
{
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

struct Ctl {
    unsigned gen;            // barrier generation seen by this CTA (thread 0)
    unsigned tag;            // this launch: the generation every CTA saw at its start, + 1
    int abort;               // this CTA stops
    unsigned pend;           // bulk copies in flight: bit b = buffer b (P, Q, R)
    unsigned par;            // mbarrier parity per buffer
};

// Every CTA arrives; the last one resets the count and publishes the next
// generation; the others poll it (acquire).  Returns false when the launch is
// being abandoned.
__device__ bool grid_sync(const StepArgs& a, Ctl* ctl)
{
    __threadfence();          // every thread's stores of this phase, before the arrival
    __syncthreads();
    if (threadIdx.x == 0 && !ctl->abort) {
        __threadfence();
        const unsigned target = ctl->gen + 1u;
        if (atomicAdd(a.bar_count, 1u) == gridDim.x - 1) {
            atomicExch(a.bar_count, 0u);
            __threadfence();
            st_release_gpu(a.bar_gen, target);
        } else {
            long long it = 0;
            while (ld_acquire_gpu(a.bar_gen) != target) {
                ++it;
                if ((it & 255) == 0 && *reinterpret_cast<volatile unsigned*>(a.abort_word) == ctl->tag) {
                    ctl->abort = 1;
                    break;
                }
                if (it > STEP_WAIT_LIMIT) {
                    atomicExch(a.err, ERR_STEP_BARRIER);
                    atomicExch(a.abort_word, ctl->tag);
                    ctl->abort = 1;
                    break;
                }
                if (it > 2048) __nanosleep(32);
            }
        }
        ctl->gen = target;
    }
    __syncthreads();
    return !ctl->abort;
}

// ---- weight requests ---------------------------------------------------------
enum { BUF_P = 0, BUF_Q = 1, BUF_R = 2 };

// rows [r0, r0+n) of a matrix with K columns -> dst: packed rows, then their scales
__device__ __forceinline__ uint32_t mat_bytes(int n, int K) { return (uint32_t)n * (K / 2 + K / 16); }
__device__ __forceinline__ void req_rows(unsigned char* dst, const uint32_t* pack, const uint16_t* sc, int r0, int n,
                                         int K, uint64_t* bar)
{
    if (n <= 0) return;
    bulk_g2s(dst, reinterpret_cast<const unsigned char*>(pack) + (size_t)r0 * (K / 2), (uint32_t)n * (K / 2), bar);
    bulk_g2s(dst + (size_t)n * (K / 2), sc + (size_t)r0 * (K / 32), (uint32_t)n * (K / 16), bar);
}

__device__ __forceinline__ int rowsC0(const StepArgs& a) { return min(a.H, (int)blockIdx.x * a.rpC); }
__device__ __forceinline__ int rowsC(const StepArgs& a) { return max(0, min(a.H, ((int)blockIdx.x + 1) * a.rpC) - rowsC0(a)); }
__device__ __forceinline__ int rowsD0(const StepArgs& a) { return min(a.I, (int)blockIdx.x * a.rpD); }
__device__ __forceinline__ int rowsD(const StepArgs& a) { return max(0, min(a.I, ((int)blockIdx.x + 1) * a.rpD) - rowsD0(a)); }

// phase-A block of this CTA: matrix, first row in it, head (q heads, then k, then v)
struct BlockA {
    int mat, row0, head;
    bool live;
};
__device__ __forceinline__ BlockA block_a(const StepArgs& a)
{
    const int qrows = a.nHq * STEP_HD, kvrows = a.nKv * STEP_HD;
    const int r = (int)blockIdx.x * RBA;
    BlockA b{0, 0, 0, r < qrows + 2 * kvrows};
    if (r < qrows) { b.mat = WQ; b.row0 = r; }
    else if (r < qrows + kvrows) { b.mat = WK; b.row0 = r - qrows; }
    else { b.mat = WV; b.row0 = r - qrows - kvrows; }
    b.head = r / STEP_HD;
    return b;
}

// Thread 0: request a phase's rows into a buffer (after the CTA finished reading it).
__device__ void request(const StepArgs& a, Ctl* ctl, int buf, int phase, int l, unsigned char* smem, uint64_t* bars)
{
    const StepLayer& Ly = a.layers[l];
    uint64_t* bar = bars + buf;
    unsigned char* dst = smem + (buf == BUF_P ? a.off_P : buf == BUF_Q ? a.off_Q : a.off_R);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    uint32_t bytes = 0;
    if (phase == 0) {          // A: one 32-row block + ln1
        const BlockA b = block_a(a);
        if (b.live) bytes = mat_bytes(RBA, a.H);
        bytes += (uint32_t)a.H * 2;
        mbar_expect_tx(bar, bytes);
        if (b.live) req_rows(dst, Ly.p[b.mat], Ly.s[b.mat], b.row0, RBA, a.H, bar);
        bulk_g2s(dst + (b.live ? mat_bytes(RBA, a.H) : 0u), Ly.ln1, (uint32_t)a.H * 2, bar);
    } else if (phase == 2) {   // C: o rows
        const int n = rowsC(a), K = a.nHq * STEP_HD;
        bytes = mat_bytes(n, K);
        if (bytes == 0) return;
        mbar_expect_tx(bar, bytes);
        req_rows(dst, Ly.p[WO], Ly.s[WO], rowsC0(a), n, K, bar);
    } else if (phase == 3) {   // D: gate rows, up rows, ln2
        const int n = rowsD(a);
        bytes = 2 * mat_bytes(n, a.H) + (uint32_t)a.H * 2;
        mbar_expect_tx(bar, bytes);
        req_rows(dst, Ly.p[WG], Ly.s[WG], rowsD0(a), n, a.H, bar);
        req_rows(dst + mat_bytes(n, a.H), Ly.p[WU], Ly.s[WU], rowsD0(a), n, a.H, bar);
        bulk_g2s(dst + 2 * mat_bytes(n, a.H), Ly.ln2, (uint32_t)a.H * 2, bar);
    } else {                   // E: down rows
        const int n = rowsC(a);
        bytes = mat_bytes(n, a.I);
        if (bytes == 0) return;
        mbar_expect_tx(bar, bytes);
        req_rows(dst, Ly.p[WD], Ly.s[WD], rowsC0(a), n, a.I, bar);
    }
    ctl->pend |= 1u << buf;
}

// All threads: wait for a buffer's copies (bounded).
__device__ bool await_buf(const StepArgs& a, Ctl* ctl, int buf, uint64_t* bars)
{
    if (!(ctl->pend & (1u << buf))) return true;      // nothing was requested (no rows here)
    const bool ok = mbar_wait(bars + buf, (ctl->par >> buf) & 1u);
    __syncthreads();
    if (threadIdx.x == 0) {
        ctl->par ^= 1u << buf;
        ctl->pend &= ~(1u << buf);
        if (!ok) {
            atomicExch(a.err, ERR_STEP_COPY);
            atomicExch(a.abort_word, ctl->tag);
            ctl->abort = 1;
        }
    }
    __syncthreads();
    return !ctl->abort;
}

// ---- one phase's GEMV over the CTA's rows (the standalone consumer loop, B = 1) --
// w_s: [n][G] 16-byte weight groups, then [n][G] f16 scales
template <int NM>
__device__ void gemv_rows(const unsigned char* act, const unsigned char* w0, const unsigned char* w1, int n, int G,
                          float* y, int row0, bool residual)
{
    constexpr int RPW = 4, NW = THREADS / 32;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    for (int r0 = wid; r0 < n; r0 += NW * RPW) {
        float acc[RPW][NM];
#pragma unroll
        for (int q = 0; q < RPW; q++)
#pragma unroll
            for (int s = 0; s < NM; s++) acc[q][s] = 0.0f;
#pragma unroll
        for (int s = 0; s < NM; s++) {
            const unsigned char* slot = s ? w1 : w0;
            const uint4* wq = reinterpret_cast<const uint4*>(slot);
            const uint16_t* sbase = reinterpret_cast<const uint16_t*>(slot + (size_t)n * G * 16);
            for (int g = lane; g < G; g += 32) {
                XQ<1> xg;
                load_xq<1>(xg, act, G, g);
#pragma unroll
                for (int q = 0; q < RPW; q++) {
                    const int r = r0 + q * NW;
                    if (r < n) item_q8x<1>(wq[r * G + g], tb_h2f(sbase[r * G + g]), xg, &acc[q][s]);
                }
            }
        }
#pragma unroll
        for (int q = 0; q < RPW; q++)
#pragma unroll
            for (int s = 0; s < NM; s++) acc[q][s] = warp_sum(acc[q][s]);
        if (lane == 0) {
#pragma unroll
            for (int q = 0; q < RPW; q++) {
                const int r = r0 + q * NW;
                if (r >= n) continue;
                float* yp = y + row0 + r;
                if (NM == 2) {
                    const float g = acc[q][0], u = acc[q][NM - 1];
                    *yp = __fdiv_rn(g, 1.0f + expf(-g)) * u;
                } else {
                    *yp = (residual ? __ldcg(yp) : 0.0f) + acc[q][0];
                }
            }
        }
    }
}

// QUANTQ8 (optionally RMSNorm first) of a whole f32 row written by other CTAs
__device__ __forceinline__ void stage(const StepArgs& sa, unsigned char* smem, const float* x, int K, bool norm,
                                      const uint16_t* nws, float* red)
{
    Args a{};
    a.K = K;
    a.act_src = norm ? ACT_RMSNORM : ACT_F32;
    a.x = x;
    a.eps = sa.eps;
    stage_q8<1, false, true>(a, smem + sa.off_act, reinterpret_cast<float*>(smem + sa.off_xbuf), sa.xbuf_floats, red,
                             nws);
    __syncthreads();
}

__device__ __forceinline__ AttnArgs attn_args(const StepArgs& a, const StepLayer& Ly)
{
    AttnArgs t{};
    t.qr = a.qr; t.Kq = Ly.Kq; t.Ks = Ly.Ks; t.Vq = Ly.Vq; t.Vs = Ly.Vs;
    t.PO = a.PO; t.PML = a.PML; t.out = a.attn; t.counters = a.counters; t.dpos = a.pos; t.err = a.err;
    t.cache_rows = a.max_seq; t.S = 0; t.nHq = a.nHq; t.nKv = a.nKv; t.nsplit = a.nsplit; t.grid_z = 1;
    return t;
}

// attention units of this CTA: unit u = blockIdx.x + gridDim.x * (2 i + group)
template <int GRP>
__device__ void attn_prefetch(const StepArgs& a, int l, unsigned char* smem)
{
    using U = DecUnit<STEP_HD, GRP, 1>;
    const int grp = threadIdx.x >> 7, gtid = threadIdx.x & 127;
    const int u = blockIdx.x + gridDim.x * grp;
    if (u >= a.nKv * a.nsplit) return;
    const AttnArgs t = attn_args(a, a.layers[l]);
    U unit(t, smem + a.off_P + grp * U::L::BYTES, u % a.nKv, u / a.nKv, 0, gtid, 1 + grp);
    unit.prefetch(true);
}

template <int GRP>
__device__ void attn_run(const StepArgs& a, int l, unsigned char* smem)
{
    using U = DecUnit<STEP_HD, GRP, 1>;
    const int grp = threadIdx.x >> 7, gtid = threadIdx.x & 127;
    const AttnArgs t = attn_args(a, a.layers[l]);
    for (int i = 0;; i++) {
        const int u = blockIdx.x + gridDim.x * (2 * i + grp);
        if (u >= a.nKv * a.nsplit) break;
        U unit(t, smem + a.off_P + grp * U::L::BYTES, u % a.nKv, u / a.nKv, 0, gtid, 1 + grp);
        if (i > 0) unit.prefetch(false);
        unit.run(i == 0);
    }
}

// attnPrepQ8 of one head, by the whole CTA (thread j = element j), as k_attn_prep
__device__ void prep_head(const StepArgs& a, const StepLayer& Ly, int head, int pos, const float* cs, float* rk,
                          float* red)
{
    const int j = threadIdx.x, hd = STEP_HD;
    const bool isQ = head < a.nHq, isK = !isQ && head < a.nHq + a.nKv;
    const int hh = isQ ? head : (isK ? head - a.nHq : head - a.nHq - a.nKv);
    const float* src = isQ ? a.q : (isK ? a.k : a.v);
    float x = j < hd ? __ldcg(src + (long long)hh * hd + j) : 0.0f;
    if (isQ || isK) {
        const float c = j < hd ? cs[j] : 0.0f, s = j < hd ? cs[hd + j] : 0.0f;
        x = norm_rope(x, isQ ? Ly.qn : Ly.kn, hd, a.eps, c, s, rk, red);
        if (isQ) {
            if (j < hd) a.qr[(long long)hh * hd + j] = x;
            return;
        }
    }
    if (pos < 0 || pos >= a.max_seq) return;   // reported by the attention units
    const long long row = (long long)pos * a.nKv * hd + (long long)hh * hd;
    quant_row(x, hd, (isK ? Ly.Kq : Ly.Vq) + row, (isK ? Ly.Ks : Ly.Vs) + row / 32);
}

template <int GRP>
__global__ void __launch_bounds__(THREADS, 1) k_decode_step(const StepArgs a)
{
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* misc = smem + a.off_misc;
    uint64_t* bars = reinterpret_cast<uint64_t*>(misc);              // 3 mbarriers
    Ctl* ctl = reinterpret_cast<Ctl*>(misc + 64);
    float* red = reinterpret_cast<float*>(misc + 128);               // >= 72 floats
    float* cs = reinterpret_cast<float*>(misc + 512);                // cos [hd], sin [hd]
    float* rk = cs + 2 * STEP_HD;                                    // [hd]
    int* flag = reinterpret_cast<int*>(rk + STEP_HD);
    const int tid = threadIdx.x;
    const int pos = a.pos[0];

    if (tid == 0) {
        // no barrier of this launch can complete before every CTA has read the
        // generation, so all CTAs read the same value: it tags the launch
        ctl->gen = ld_acquire_gpu(a.bar_gen);
        ctl->tag = ctl->gen + 1u;
        ctl->abort = 0;
        ctl->pend = 0;
        ctl->par = 0;
        for (int b = 0; b < 3; b++) mbar_init(&bars[b], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (tid < STEP_HD) {
        float c, s;
        rope_cs(tid, STEP_HD, pos, a.theta, &c, &s);
        cs[tid] = c;
        cs[STEP_HD + tid] = s;
    }
    __syncthreads();
    if (tid == 0) {
        request(a, ctl, BUF_R, 0, 0, smem, bars);
        request(a, ctl, BUF_Q, 4, 0, smem, bars);
    }
    attn_prefetch<GRP>(a, 0, smem);
    // embed: this CTA's rows of x (the o / down row slice)
    {
        const int r0 = rowsC0(a), n = rowsC(a);
        const uint32_t id = a.ids[0];
        for (int i = tid; i < n; i += THREADS) a.x[r0 + i] = tb_h2f(a.embed[(long long)id * a.H + r0 + i]);
    }
    if (!grid_sync(a, ctl)) goto drain;

    for (int l = 0; l < a.L; l++) {
        const StepLayer& Ly = a.layers[l];
        const bool more = l + 1 < a.L;
        // ---- A: rmsnorm + quant of x, q/k/v rows, prep of completed heads
        {
            if (!await_buf(a, ctl, BUF_R, bars)) goto drain;
            const BlockA b = block_a(a);
            const unsigned char* wR = smem + a.off_R;
            const uint16_t* nws = reinterpret_cast<const uint16_t*>(wR + (b.live ? mat_bytes(RBA, a.H) : 0));
            if (b.live) {
                stage(a, smem, a.x, a.H, true, nws, red);
                float* y = b.mat == WQ ? a.q : (b.mat == WK ? a.k : a.v);
                gemv_rows<1>(smem + a.off_act, wR, nullptr, RBA, a.H / 32, y, b.row0, false);
                __threadfence();      // this block's rows, before its arrival at the head
                __syncthreads();
                if (tid == 0) {
                    __threadfence();
                    const unsigned bph = STEP_HD / RBA;
                    *flag = atomicAdd(a.head_ctr + b.head, 1u) == bph - 1;
                }
                __syncthreads();
                if (*flag) {
                    __threadfence();
                    prep_head(a, Ly, b.head, pos, cs, rk, red);
                    __syncthreads();
                    if (tid == 0) a.head_ctr[b.head] = 0u;
                }
            }
            __syncthreads();
            if (tid == 0) request(a, ctl, BUF_R, 2, l, smem, bars);
            if (!grid_sync(a, ctl)) goto drain;
        }
        // ---- B: attention (prep'd q, cache row pos written in A)
        {
            attn_run<GRP>(a, l, smem);
            __syncthreads();
            if (tid == 0) request(a, ctl, BUF_P, 3, l, smem, bars);
            if (!grid_sync(a, ctl)) goto drain;
        }
        // ---- C: quant of the attention output, o rows += x
        {
            if (!await_buf(a, ctl, BUF_R, bars)) goto drain;
            const int n = rowsC(a);
            if (n > 0) {
                stage(a, smem, a.attn, a.nHq * STEP_HD, false, nullptr, red);
                gemv_rows<1>(smem + a.off_act, smem + a.off_R, nullptr, n, a.nHq * STEP_HD / 32, a.x, rowsC0(a), true);
            }
            __syncthreads();
            if (tid == 0 && more) request(a, ctl, BUF_R, 0, l + 1, smem, bars);
            if (!grid_sync(a, ctl)) goto drain;
        }
        // ---- D: rmsnorm + quant of x, gate/up rows, swiglu
        {
            if (!await_buf(a, ctl, BUF_P, bars)) goto drain;
            const int n = rowsD(a);
            const unsigned char* wP = smem + a.off_P;
            if (n > 0) {
                const uint16_t* nws = reinterpret_cast<const uint16_t*>(wP + 2 * mat_bytes(n, a.H));
                stage(a, smem, a.x, a.H, true, nws, red);
                gemv_rows<2>(smem + a.off_act, wP, wP + mat_bytes(n, a.H), n, a.H / 32, a.swi, rowsD0(a), false);
            }
            __syncthreads();
            if (more) attn_prefetch<GRP>(a, l + 1, smem);
            if (!grid_sync(a, ctl)) goto drain;
        }
        // ---- E: quant of swi, down rows += x
        {
            if (!await_buf(a, ctl, BUF_Q, bars)) goto drain;
            const int n = rowsC(a);
            if (n > 0) {
                stage(a, smem, a.swi, a.I, false, nullptr, red);
                gemv_rows<1>(smem + a.off_act, smem + a.off_Q, nullptr, n, a.I / 32, a.x, rowsC0(a), true);
            }
            __syncthreads();
            if (tid == 0 && more) request(a, ctl, BUF_Q, 4, l + 1, smem, bars);
            if (more && !grid_sync(a, ctl)) goto drain;
        }
    }
drain:
    // copies still in flight land before the CTA's shared memory is released
    cp_async_wait<0>();
    __syncthreads();
    if (tid == 0) {
        for (int b = 0; b < 3; b++)
            if (ctl->pend & (1u << b)) mbar_wait(&bars[b], (ctl->par >> b) & 1u);
    }
}

}  // namespace

// ---- host side ---------------------------------------------------------------------
struct tb_step_plan {
    StepArgs a;
    int smem = 0, grid = 0, grp = 0;
};

// Layout and feasibility of the persistent step for these sizes on this device;
// returns TB_ERR_UNSUPPORTED when it does not apply (the caller keeps the
// multi-kernel step).
int tb_step_plan_make(tb_ctx* ctx, int L, int H, int nHq, int nKv, int hd, int I, int nsplit, int max_seq,
                      tb_step_plan** out)
{
    *out = nullptr;
    const int G = ctx->num_sms;
    const int grp = nKv > 0 ? nHq / nKv : 0;
    if (hd != STEP_HD || nKv <= 0 || nHq % nKv || (grp != 1 && grp != 2 && grp != 4 && grp != 8))
        return TB_ERR_UNSUPPORTED;
    // K % 256: every slice's scales (n * K/16 bytes) are whole 16-byte chunks for the bulk copies
    if (H % 256 || I % 256 || (nHq * hd) % 256 || H > 8192 || I > 16384) return TB_ERR_UNSUPPORTED;
    if ((nHq + 2 * nKv) * hd / RBA > G) return TB_ERR_UNSUPPORTED;   // one phase-A block per CTA
    if (nsplit < 1 || nsplit > 256) return TB_ERR_UNSUPPORTED;
    StepArgs a{};
    a.L = L; a.H = H; a.nHq = nHq; a.nKv = nKv; a.I = I; a.nsplit = nsplit; a.max_seq = max_seq;
    a.rpC = (H + G - 1) / G;
    a.rpD = (I + G - 1) / G;
    auto mb = [](int n, int K) { return (size_t)n * (K / 2 + K / 16); };
    size_t unit_bytes = 0;
    switch (grp) {
    case 1: unit_bytes = DecLayout<STEP_HD, 1, 1>::BYTES; break;
    case 2: unit_bytes = DecLayout<STEP_HD, 2, 1>::BYTES; break;
    case 4: unit_bytes = DecLayout<STEP_HD, 4, 1>::BYTES; break;
    default: unit_bytes = DecLayout<STEP_HD, 8, 1>::BYTES; break;
    }
    auto up = [](size_t v) { return (v + 127) & ~size_t(127); };
    const size_t bP = up(std::max(2 * unit_bytes, 2 * mb(a.rpD, H) + (size_t)H * 2));
    const size_t bQ = up(mb(a.rpC, I));
    const size_t bR = up(std::max(mb(RBA, H) + (size_t)H * 2, mb(a.rpC, nHq * hd)));
    const int Kmax = std::max(std::max(H, I), nHq * hd);
    const size_t xbuf = up((size_t)Kmax * 4);
    const size_t act = up((size_t)(Kmax / 32) * 40);
    const size_t misc = 512 + 3 * STEP_HD * 4 + 128;
    a.off_P = 0;
    a.off_Q = (int)bP;
    a.off_R = (int)(bP + bQ);
    a.off_xbuf = (int)(bP + bQ + bR);
    a.off_act = (int)(bP + bQ + bR + xbuf);
    a.off_misc = (int)(bP + bQ + bR + xbuf + act);
    a.xbuf_floats = (int)(xbuf / 4);
    const size_t total = (size_t)a.off_misc + misc;
    int maxsm = 0;
    cudaDeviceGetAttribute(&maxsm, cudaDevAttrMaxSharedMemoryPerBlockOptin, ctx->device);
    if (total > (size_t)maxsm) return TB_ERR_UNSUPPORTED;
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, ctx->device);
    if (!coop) return TB_ERR_UNSUPPORTED;
    tb_step_plan* p = new tb_step_plan;
    p->a = a;
    p->smem = (int)total;
    p->grid = G;
    p->grp = grp;
    *out = p;
    return TB_OK;
}

void tb_step_plan_free(tb_step_plan* p) { delete p; }

size_t tb_step_plan_smem(const tb_step_plan* p) { return (size_t)p->smem; }

// Fill the per-step pointers and launch (cooperative: every CTA resident).
int tb_step_launch(tb_ctx* ctx, tb_step_plan* p, const tb_step_io* io)
{
    StepArgs a = p->a;
    a.layers = reinterpret_cast<const StepLayer*>(io->layers);
    a.eps = io->eps; a.theta = io->theta;
    a.ids = io->ids; a.pos = io->pos; a.embed = io->embed;
    a.x = io->x; a.q = io->q; a.k = io->k; a.v = io->v; a.qr = io->qr; a.attn = io->attn; a.swi = io->swi;
    a.PO = io->PO; a.PML = io->PML; a.counters = io->counters; a.head_ctr = io->ctrl;
    a.bar_count = io->ctrl + 64; a.bar_gen = io->ctrl + 96; a.abort_word = io->ctrl + 128;
    a.err = ctx->dev_error;
    void (*kern)(const StepArgs) = nullptr;
    switch (p->grp) {
    case 1: kern = k_decode_step<1>; break;
    case 2: kern = k_decode_step<2>; break;
    case 4: kern = k_decode_step<4>; break;
    default: kern = k_decode_step<8>; break;
    }
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p->smem);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "decode step attribute: %s", cudaGetErrorString(e));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p->grid);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = p->smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "decode step launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

size_t tb_step_layer_bytes() { return sizeof(StepLayer); }

void tb_step_layer_fill(void* dst, const uint32_t* const* packs, const uint16_t* const* scales, const uint16_t* ln1,
                        const uint16_t* ln2, const uint16_t* qn, const uint16_t* kn, int8_t* Kq, float* Ks, int8_t* Vq,
                        float* Vs)
{
    StepLayer s{};
    for (int i = 0; i < 7; i++) { s.p[i] = packs[i]; s.s[i] = scales[i]; }
    s.ln1 = ln1; s.ln2 = ln2; s.qn = qn; s.kn = kn;
    s.Kq = Kq; s.Ks = Ks; s.Vq = Vq; s.Vs = Vs;
    memcpy(dst, &s, sizeof s);
}
