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
//   A  RMSNorm + QUANTQ8 of x, q/k/v rows (32-row blocks)
//   B  split-KV attention: one 8-warp (kv head, split) unit per CTA (DecUnit,
//      the standalone kernel's code); each unit runs attnPrepQ8 for its own q
//      heads (norm + RoPE) and the unit holding row pos writes that cache row
//      (k: norm + RoPE + int8, v: int8, also straight into its tile); the last
//      split of a kv head combines and stores the heads' outputs QUANTQ8'd
//   C  the attention output (QUANTQ8'd by the combining units), o rows, += residual
//   D  RMSNorm + QUANTQ8 of x, gate/up rows, SwiGLU
//   E  QUANTQ8 of swi, down rows, += residual
// Shared-memory buffers and what they hold; each is requested once it is free,
// right after the next phase's own activation loads (so neither those loads nor
// the barriers queue behind the bulk copies), at least one phase ahead:
//   R  A(l) -> C(l) (requested at the start of B(l)) -> A(l+1) (during D(l))
//   P  B(l) key/value tiles (cp.async, during E(l-1)) -> D(l) gate/up (during C(l))
//   Q  E(l) (during A(l))
// Every phase uses the standalone kernels' device code (tb_gemv_dev.cuh,
// tb_attn_dev.cuh) with the same split count, so the step is bit-identical to
// the multi-kernel step.  Under tensor parallelism over peer memory each rank
// runs this kernel on its shard: the o and down rows are partial sums, and CTA c
// exchanges its slice of them with CTA c of every rank inside the kernel (each
// row pushed to every peer's inbox as one 8-byte (epoch, value) packet, a
// bounded wait on local loads, then x + part_0 + ... + part_{P-1} in rank order,
// the sum of the exchange kernel k_tp_allreduce), so the step is one kernel per
// rank and the same bits as the multi-kernel TP step.  The layer weights are all int4 G32
// or all ternary in the WebGPU layout (TERN: 8 code bytes a 32-group, the
// activations QUANTQ8'd in natural order, item_ternx instead of item_q8x), as
// gemvTern / gemvQ8 of the multi-kernel step.  Barrier and copy waits are bounded; a CTA that gives up
// records the error, raises the launch's abort word, drains its copies and
// returns, and the others leave at their next barrier.
#include "tb_internal.h"
#include "tb_gemv_dev.cuh"
#include "tb_attn_dev.cuh"

namespace {

constexpr int ERR_STEP_BARRIER = 0x5101;
constexpr int ERR_STEP_COPY = 0x5102;
constexpr int ERR_STEP_TP = 0x5103;
constexpr int ERR_STEP_TP_POISONED = 0x5104;   // refused: an earlier exchange wait of this rank gave up
constexpr int ERR_STEP_PACKET = 0x5105;        // a phase-boundary packet wait gave up
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
    unsigned char* attnq;    // the attention output QUANTQ8'd in the GEMV activation layout
    unsigned* counters;      // [nKv] split arrivals (zero between steps)
    unsigned long long* bar_count;   // grid barrier: arrivals since the model was made (monotonic)
    unsigned* abort_word;    // == this launch's tag: a CTA gave up in this launch
    unsigned* head_cnt;      // [L][nKv] phase-A blocks of each kv head written (zeroed by every launch)
    // phase-boundary packets (epoch << 32 | f32 bits): x rows after o (one GPU)
    unsigned long long* xpk; // [H]
    int* err;
    // optional phase trace: per CTA 1 + 38 * L %globaltimer stamps (kernel start;
    // per layer and phase: weights ready, activation row loaded, activation
    // staged, phase done, barrier passed; then per layer 8 slots of the CTA's
    // first attention unit: start, q prep, k/v prep, tiles done, partial
    // written, arrival counted, end, last-split flag; then per layer and phase
    // the moment the phase's next-buffer request was issued)
    unsigned long long* trace;
    // shared-memory layout (bytes)
    int off_P, off_Q, off_R, off_act, off_misc, off_layers;
    int rpC, rpD;            // rows per CTA of o / down (rpC) and gate / up (rpD)
    int tern;                // layer weights: 0 int4 G32, 1 ternary in the WebGPU layout
    // tensor parallel (P > 1): the o and down rows are partial sums over this rank's
    // heads / intermediate slice; CTA c exchanges its rows with CTA c of every rank
    // through the ranks' exchange arenas (peer memory over NVLink)
    int P, rank;
    float* xpart;                                 // this rank's part[2][H]
    unsigned long long* peer_inbox[TB_TP_MAX];    // every rank's inbox [TB_TP_MAX][2][H]
    const unsigned long long* my_inbox;           // this rank's inbox
    unsigned* poison;                             // this rank's poison word
};

__device__ __forceinline__ void stamp(const StepArgs& a, int slot)
{
    if (a.trace && threadIdx.x == 0) {
        unsigned long long t;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
        a.trace[(size_t)blockIdx.x * (1 + 38 * a.L) + slot] = t;
    }
}
#define STAMP(ph, k) stamp(a, 1 + 25 * l + 5 * (ph) + (k))
#define STAMP_REQ(ph) stamp(a, 1 + 33 * a.L + 5 * l + (ph))

// ---- grid barrier ---------------------------------------------------------------
__device__ __forceinline__ void red_release_add(unsigned long long* p, unsigned long long v)
{
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p)
{
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add_u32(unsigned* p, unsigned v)
{
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p)
{
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Phase-boundary packets: (epoch << 32) | f32 bits, one 8-byte store a value.  A
// reader polls until the epoch is the one it expects, so a value and the news
// that it is ready arrive in the same load (no barrier, no second round trip).
__device__ __forceinline__ void st_relaxed_gpu_u64(unsigned long long* p, unsigned long long v)
{
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void ld_relaxed_gpu_v2u64(const unsigned long long* p, unsigned long long& a,
                                                     unsigned long long& b)
{
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

struct Ctl {
    unsigned long long base; // arrivals before this launch (a multiple of the grid)
    unsigned nb;             // barriers of this launch so far
    unsigned tag;            // this launch (base / grid + 1), marks its abort
    int abort;               // this CTA stops
    unsigned pend;           // bulk copies in flight: bit b = buffer b (P, Q, R)
    unsigned par;            // mbarrier parity per buffer
};

// Every CTA adds its arrival (release) to one monotonic counter and polls it
// (acquire) until the whole grid has arrived: one fire-and-forget add and the
// polls, no reset.  Returns false when the launch is being abandoned.
__device__ bool grid_sync(const StepArgs& a, Ctl* ctl)
{
    __syncthreads();          // the CTA's stores of this phase happen before thread 0's release
    if (threadIdx.x == 0 && !ctl->abort) {
        ctl->nb++;
        const unsigned long long target = ctl->base + (unsigned long long)ctl->nb * gridDim.x;
        red_release_add(a.bar_count, 1ull);
        {
            long long it = 0;
            while (ld_acquire_u64(a.bar_count) < target) {
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
    }
    __syncthreads();
    return !ctl->abort;
}

// ---- weight requests ---------------------------------------------------------
enum { BUF_P = 0, BUF_Q = 1, BUF_R = 2 };

// rows [r0, r0+n) of a matrix with K columns -> dst: packed rows (K/2 bytes a
// row of int4, K/4 of ternary codes), then their f16 scales (one per 32-group)
__device__ __forceinline__ uint32_t row_bytes(const StepArgs& a, int K) { return (uint32_t)(K >> (a.tern ? 2 : 1)); }
__device__ __forceinline__ uint32_t mat_bytes(const StepArgs& a, int n, int K)
{
    return (uint32_t)n * (row_bytes(a, K) + K / 16);
}
__device__ __forceinline__ void req_rows(const StepArgs& a, unsigned char* dst, const uint32_t* pack,
                                         const uint16_t* sc, int r0, int n, int K, uint64_t* bar)
{
    if (n <= 0) return;
    const uint32_t wb = row_bytes(a, K);
    bulk_g2s(dst, reinterpret_cast<const unsigned char*>(pack) + (size_t)r0 * wb, (uint32_t)n * wb, bar);
    bulk_g2s(dst + (size_t)n * wb, sc + (size_t)r0 * (K / 32), (uint32_t)n * (K / 16), bar);
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
    const StepLayer& Ly = reinterpret_cast<const StepLayer*>(smem + a.off_layers)[l];
    uint64_t* bar = bars + buf;
    unsigned char* dst = smem + (buf == BUF_P ? a.off_P : buf == BUF_Q ? a.off_Q : a.off_R);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    uint32_t bytes = 0;
    if (phase == 0) {          // A: one 32-row block + ln1
        const BlockA b = block_a(a);
        if (b.live) bytes = mat_bytes(a, RBA, a.H);
        bytes += (uint32_t)a.H * 2;
        mbar_expect_tx(bar, bytes);
        if (b.live) req_rows(a, dst, Ly.p[b.mat], Ly.s[b.mat], b.row0, RBA, a.H, bar);
        bulk_g2s(dst + (b.live ? mat_bytes(a, RBA, a.H) : 0u), Ly.ln1, (uint32_t)a.H * 2, bar);
    } else if (phase == 2) {   // C: o rows
        const int n = rowsC(a), K = a.nHq * STEP_HD;
        bytes = mat_bytes(a, n, K);
        if (bytes == 0) return;
        mbar_expect_tx(bar, bytes);
        req_rows(a, dst, Ly.p[WO], Ly.s[WO], rowsC0(a), n, K, bar);
    } else if (phase == 3) {   // D: gate rows, up rows, ln2
        const int n = rowsD(a);
        bytes = 2 * mat_bytes(a, n, a.H) + (uint32_t)a.H * 2;
        mbar_expect_tx(bar, bytes);
        req_rows(a, dst, Ly.p[WG], Ly.s[WG], rowsD0(a), n, a.H, bar);
        req_rows(a, dst + mat_bytes(a, n, a.H), Ly.p[WU], Ly.s[WU], rowsD0(a), n, a.H, bar);
        bulk_g2s(dst + 2 * mat_bytes(a, n, a.H), Ly.ln2, (uint32_t)a.H * 2, bar);
    } else {                   // E: down rows
        const int n = rowsC(a);
        bytes = mat_bytes(a, n, a.I);
        if (bytes == 0) return;
        mbar_expect_tx(bar, bytes);
        req_rows(a, dst, Ly.p[WD], Ly.s[WD], rowsC0(a), n, a.I, bar);
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
// own: this CTA's rows of the residual x kept in shared memory (their only
// writer is this CTA), so y = own + W.a needs no read of y from memory
template <int NM, int RPW, bool TERN>
__device__ void gemv_rows_r(const unsigned char* act, const unsigned char* w0, const unsigned char* w1, int n, int G,
                            float* y, int row0, float* own, unsigned long long* pk, unsigned pe)
{
    constexpr int NW = THREADS / 32;
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
            const uint16_t* sbase = reinterpret_cast<const uint16_t*>(slot + (size_t)n * G * (TERN ? 8 : 16));
            for (int g = lane; g < G; g += 32) {
                XQ<1> xg;
                load_xq<1>(xg, act, G, g);
#pragma unroll
                for (int q = 0; q < RPW; q++) {
                    const int r = r0 + q * NW;
                    if (r >= n) continue;
                    if (TERN)
                        item_ternx<1>(reinterpret_cast<const uint2*>(slot)[r * G + g], tb_h2f(sbase[r * G + g]), xg,
                                      &acc[q][s]);
                    else
                        item_q8x<1>(reinterpret_cast<const uint4*>(slot)[r * G + g], tb_h2f(sbase[r * G + g]), xg,
                                    &acc[q][s]);
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
                float v;
                if (NM == 2) {
                    const float g = acc[q][0], u = acc[q][NM - 1];
                    v = __fdiv_rn(g, 1.0f + expf(-g)) * u;
                } else if (own) {
                    v = own[r] + acc[q][0];
                    own[r] = v;
                } else {
                    v = 0.0f + acc[q][0];
                }
                *yp = v;
                // the same value as an epoch-tagged packet for the next phase's readers
                if (pk) st_relaxed_gpu_u64(pk + row0 + r, ((unsigned long long)pe << 32) | __float_as_uint(v));
            }
        }
    }
}

// rows per warp chosen so the CTA's rows take one pass (a row's sum does not
// depend on which warp computes it)
template <int NM, bool TERN>
__device__ void gemv_rows(const unsigned char* act, const unsigned char* w0, const unsigned char* w1, int n, int G,
                          float* y, int row0, float* own, unsigned long long* pk = nullptr, unsigned pe = 0)
{
    const int rpw = (n + THREADS / 32 - 1) / (THREADS / 32);
    if (rpw <= 2) gemv_rows_r<NM, 2, TERN>(act, w0, w1, n, G, y, row0, own, pk, pe);
    else if (rpw <= 4) gemv_rows_r<NM, 4, TERN>(act, w0, w1, n, G, y, row0, own, pk, pe);
    else if (rpw <= 6) gemv_rows_r<NM, 6, TERN>(act, w0, w1, n, G, y, row0, own, pk, pe);
    else gemv_rows_r<NM, 8, TERN>(act, w0, w1, n, G, y, row0, own, pk, pe);
}

// QUANTQ8 (optionally RMSNorm first) of a whole f32 row written by other CTAs,
// into the int8 layout of stage_q8<1, NAT> with the same bits (NAT: the
// ternary GEMVs' natural order; else the permuted int4 dp4a order): thread
// t holds float4s f = t, t+256, ... in registers (the canonical sum-of-squares
// order), 8 consecutive threads (one warp-aligned 32-group) find the group
// maximum and sum with shuffles, and pairs of threads assemble the even / odd
// byte words of a weight word.  Every thread is busy and there is one
// round trip to memory.  K % 32 == 0, K <= 8192.
template <bool NAT>
__device__ void stage(const StepArgs& sa, unsigned char* smem, const float* x, int K, bool norm, const uint16_t* nws,
                      float* red, int slot)
{
    constexpr int MAXF = 8;
    const int tid = threadIdx.x, G = K >> 5, K4 = K >> 2;
    const int nf = (K4 + THREADS - 1) / THREADS;
    float4 v[MAXF];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXF; i++) {
        const int f = i * THREADS + tid;
        v[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (i < nf && f < K4) v[i] = __ldcg(reinterpret_cast<const float4*>(x) + f);
    }
#pragma unroll
    for (int i = 0; i < MAXF; i++)
        if (i < nf && i * THREADS + tid < K4) ss = sumsq_f4(v[i], ss);
    if (sa.trace && tid == 0) {   // the row has arrived in thread 0's registers
        asm volatile("" ::"f"(ss));
        stamp(sa, slot);
    }
    float inv = 1.0f;
    if (norm) {
        float tot;
        block256_reduce_rows<1>(&ss, red, &tot);
        inv = rms_inv(tot, K, sa.eps);
    }
#pragma unroll
    for (int i = 0; i < MAXF; i++) {
        if (i >= nf) break;
        const int f = i * THREADS + tid;
        const bool live = f < K4;              // whole 32-groups (8 consecutive f) are live or not
        float e[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
        if (norm && live) {
#pragma unroll
            for (int j = 0; j < 4; j++) e[j] = __fmul_rn(__fmul_rn(e[j], inv), tb_h2f(nws[4 * f + j]));
        }
        q8_store_group4(e, f >> 3, live, smem + sa.off_act, G, NAT);      // f & 7 == lane & 7
    }
    __syncthreads();
    stamp(sa, slot + 1);
}

// stage() for a row that arrives as packets (pk[k] = (e << 32) | bits of x[k],
// written by other CTAs in the previous phase with no barrier in between): each
// thread polls its own float4s' packets (relaxed loads at gpu scope, two packets
// a 16-byte load) until all carry epoch e, bounded, then stages exactly as
// stage() does.  false: this CTA gave up (or saw another CTA give up); the
// launch is abandoned.
template <bool NAT>
__device__ bool stage_pk(const StepArgs& sa, Ctl* ctl, unsigned char* smem, const unsigned long long* pk, unsigned e,
                         int K, bool norm, const uint16_t* nws, float* red, int slot)
{
    constexpr int MAXF = 8;
    const int tid = threadIdx.x, G = K >> 5, K4 = K >> 2;
    const int nf = (K4 + THREADS - 1) / THREADS;
    float4 v[MAXF];
    unsigned pending = 0;
#pragma unroll
    for (int i = 0; i < MAXF; i++) {
        v[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (i < nf && i * THREADS + tid < K4) pending |= 1u << i;
    }
    long long it = 0;
    while (pending && !*reinterpret_cast<volatile int*>(&ctl->abort)) {
#pragma unroll
        for (int i = 0; i < MAXF; i++) {
            if (!((pending >> i) & 1u)) continue;
            const unsigned long long* q = pk + 4 * (i * THREADS + tid);
            unsigned long long p0, p1, p2, p3;
            ld_relaxed_gpu_v2u64(q, p0, p1);
            ld_relaxed_gpu_v2u64(q + 2, p2, p3);
            if ((unsigned)(p0 >> 32) == e && (unsigned)(p1 >> 32) == e && (unsigned)(p2 >> 32) == e &&
                (unsigned)(p3 >> 32) == e) {
                v[i] = make_float4(__uint_as_float((unsigned)p0), __uint_as_float((unsigned)p1),
                                   __uint_as_float((unsigned)p2), __uint_as_float((unsigned)p3));
                pending &= ~(1u << i);
            }
        }
        if (!pending) break;
        ++it;
        if ((it & 255) == 0 && *reinterpret_cast<volatile unsigned*>(sa.abort_word) == ctl->tag) {
            ctl->abort = 1;
            break;
        }
        if (it > STEP_WAIT_LIMIT) {
            atomicExch(sa.err, ERR_STEP_PACKET);
            atomicExch(sa.abort_word, ctl->tag);
            ctl->abort = 1;
            break;
        }
        if (it > 64) __nanosleep(32);
    }
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < MAXF; i++)
        if (i < nf && i * THREADS + tid < K4) ss = sumsq_f4(v[i], ss);
    if (sa.trace && tid == 0) {   // the row has arrived in thread 0's registers
        asm volatile("" ::"f"(ss));
        stamp(sa, slot);
    }
    float inv = 1.0f;
    if (norm) {
        float tot;
        block256_reduce_rows<1>(&ss, red, &tot);
        inv = rms_inv(tot, K, sa.eps);
    }
#pragma unroll
    for (int i = 0; i < MAXF; i++) {
        if (i >= nf) break;
        const int f = i * THREADS + tid;
        const bool live = f < K4;              // whole 32-groups (8 consecutive f) are live or not
        float e4[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
        if (norm && live) {
#pragma unroll
            for (int j = 0; j < 4; j++) e4[j] = __fmul_rn(__fmul_rn(e4[j], inv), tb_h2f(nws[4 * f + j]));
        }
        q8_store_group4(e4, f >> 3, live, smem + sa.off_act, G, NAT);      // f & 7 == lane & 7
    }
    __syncthreads();
    stamp(sa, slot + 1);
    return !ctl->abort;
}

// ---- tensor-parallel exchange of the o / down rows ----------------------------------
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v)
{
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p)
{
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// After this CTA stored its partial rows of exchange xi (rows rowsC0 .. +rowsC)
// into its own arena's part[xi & 1] and the caller's __syncthreads: push every
// row to every other rank as one 8-byte packet (e << 32) | f32 bits into that
// rank's inbox[this rank][xi & 1][row] (plain NVLink stores, no fence: the epoch
// travels in the same store as the value, so a packet is complete the moment it
// is seen), then wait (bounded) until this rank's inbox holds epoch e for every
// other rank's rows of this CTA -- local loads only -- and form
// x + part_0 + ... + part_{P-1} in rank order, the sum k_tp_allreduce forms,
// into the CTA's residual rows and x.
// e = (barriers before this launch) + xi + 1: a launch passes 4L >= 2L + 1
// barriers and has 2L exchanges, so epochs grow across launches; a slot holds
// epoch e - 2 or e, never more (a rank sends exchange xi + 2 only after it
// received every rank's xi + 1, sent after that rank consumed xi), so the wait
// is for equality.  A wait that gives up aborts the launch; the abort poisons
// the rank (checked at the start of every launch), because the ranks' epochs
// may disagree from then on until tb_qwen3_tp_reset.
__device__ bool tp_exchange(const StepArgs& a, Ctl* ctl, int xi, float* own, float* vals)
{
    const unsigned e = (unsigned)(ctl->base / gridDim.x) + (unsigned)xi + 1u;
    const int tid = threadIdx.x, r0 = rowsC0(a), n = rowsC(a), par = xi & 1;
    const float* part = a.xpart + (size_t)par * a.H + r0;
    const int pairs = a.P * n;
    if (!ctl->abort) {
        for (int j = tid; j < pairs; j += THREADS) {
            const int s = j / n, i = j - s * n;
            const float v = part[i];
            if (s == a.rank) {
                vals[s * 64 + i] = v;
            } else {
                st_relaxed_sys_u64(a.peer_inbox[s] + ((size_t)a.rank * 2 + par) * a.H + r0 + i,
                                   ((unsigned long long)e << 32) | __float_as_uint(v));
            }
        }
        for (int j = tid; j < pairs; j += THREADS) {
            const int s = j / n, i = j - s * n;
            if (s == a.rank) continue;
            const unsigned long long* slot = a.my_inbox + ((size_t)s * 2 + par) * a.H + r0 + i;
            unsigned long long pk;
            long long it = 0;
            while ((unsigned)((pk = ld_relaxed_sys_u64(slot)) >> 32) != e) {
                ++it;
                if ((it & 255) == 0 && *reinterpret_cast<volatile unsigned*>(a.abort_word) == ctl->tag) {
                    ctl->abort = 1;
                    break;
                }
                if (it > STEP_WAIT_LIMIT) {
                    atomicExch(a.err, ERR_STEP_TP);
                    atomicExch(a.abort_word, ctl->tag);
                    ctl->abort = 1;
                    break;
                }
                if (it > 2048) __nanosleep(32);
            }
            vals[s * 64 + i] = __uint_as_float((unsigned)pk);
        }
    }
    __syncthreads();
    if (ctl->abort) return false;
    for (int i = tid; i < n; i += THREADS) {
        float v = own[i];
        for (int s = 0; s < a.P; s++) v += vals[s * 64 + i];
        own[i] = v;
        a.x[r0 + i] = v;
    }
    return true;
}

// the context S = pos + 1 was read and checked at the kernel's start (0 when pos
// is outside the cache: every split empty), so the units read no position
__device__ __forceinline__ AttnArgs attn_args(const StepArgs& a, const StepLayer& Ly, int S)
{
    AttnArgs t{};
    t.qr = a.qr; t.Kq = Ly.Kq; t.Ks = Ly.Ks; t.Vq = Ly.Vq; t.Vs = Ly.Vs;
    t.PO = a.PO; t.PML = a.PML; t.out = a.attn; t.counters = a.counters; t.dpos = nullptr; t.err = a.err;
    t.cache_rows = a.max_seq; t.S = S; t.nHq = a.nHq; t.nKv = a.nKv; t.nsplit = a.nsplit; t.grid_z = 1;
    return t;
}
__device__ __forceinline__ int step_S(const StepArgs& a, int pos) { return pos >= 0 && pos < a.max_seq ? pos + 1 : 0; }

// Units on CTAs: slot u = blockIdx.x + gridDim.x * (2 i + group).  The (kv head,
// split) of slot u is rotated so the last splits (they hold row pos: prep of the
// k/v row, usually the combine) land on the slots gridDim-nKv .. gridDim-1, whose
// CTAs carry no second unit when there are fewer than 2 * gridDim units.
__device__ __forceinline__ int unit_rot(const StepArgs& a, int u)
{
    const int N = a.nKv * a.nsplit, G = gridDim.x;
    return N > G ? (u + N - G) % N : u;
}

// attention units: one 8-warp unit (the whole CTA) per CTA, unit u of CTA
// blockIdx.x + gridDim.x * i; one 32-key tile per warp (the plan checks it)
constexpr int UW = 8;

template <int GRP>
__device__ void attn_prefetch(const StepArgs& a, const StepLayer& Ly, unsigned char* smem)
{
    using U = DecUnit<STEP_HD, GRP, 1, UW>;
    const int u = blockIdx.x;
    if (u >= a.nKv * a.nsplit) return;
    const AttnArgs t = attn_args(a, Ly, step_S(a, a.pos[0]));
    const int r = unit_rot(a, u);
    U unit(t, smem + a.off_P, r % a.nKv, r / a.nKv, 0, threadIdx.x, 0);
    unit.inject = true;
    unit.prefetch(true);
}

// Phase B of layer l may start for kv head h once the phase-A blocks of its
// q heads and of its k and v rows are written: (GRP + 2) * hd / RBA arrivals on
// head_cnt[l][h] (a release add by each block's thread 0 after the block's
// rows), in place of a grid barrier.  Thread 0 polls (acquire, bounded); the
// CTA barrier then orders every thread's reads of those rows after it.
__device__ bool head_ready(const StepArgs& a, Ctl* ctl, int l, int h)
{
    if (threadIdx.x == 0 && !ctl->abort) {
        const unsigned need = (unsigned)(a.nHq / a.nKv + 2) * (STEP_HD / RBA);
        const unsigned* c = a.head_cnt + (size_t)l * a.nKv + h;
        long long it = 0;
        while (ld_acquire_u32(c) < need) {
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
    __syncthreads();
    return !ctl->abort;
}

template <int GRP, bool TERN>
__device__ void attn_run(const StepArgs& a, Ctl* ctl, const StepLayer& Ly, int l, unsigned char* smem, const float* cs,
                         int pos)
{
    using U = DecUnit<STEP_HD, GRP, 1, UW>;
    const AttnArgs t = attn_args(a, Ly, step_S(a, pos));
    const PrepIn pin{a.q, a.k, a.v, Ly.qn, Ly.kn, cs, a.eps};
    for (int i = 0;; i++) {
        const int u = blockIdx.x + gridDim.x * i;
        if (u >= a.nKv * a.nsplit) break;
        const int r = unit_rot(a, u);
        if (!head_ready(a, ctl, l, r % a.nKv)) return;
        U unit(t, smem + a.off_P, r % a.nKv, r / a.nKv, 0, threadIdx.x, 0);
        unit.prep = &pin;
        unit.qout = a.attnq;
        unit.qG = a.nHq * STEP_HD / 32;
        unit.qnat = TERN;
        if (a.trace && i == 0) unit.tr = a.trace + (size_t)blockIdx.x * (1 + 38 * a.L) + 1 + 25 * a.L + 8 * l;
        // the first unit's tiles were requested in an earlier phase (row pos is
        // written into its stage by the prep); a later unit requests them now,
        // the tile holding row pos only after the prep wrote that row
        unit.inject = i == 0;
        if (i > 0) unit.prefetch(true);
        unit.run(true);
        __syncthreads();
    }
}

template <int GRP, bool TERN>
__global__ void __launch_bounds__(THREADS, 1) k_decode_step(const StepArgs a)
{
    extern __shared__ __align__(128) unsigned char smem[];
    unsigned char* misc = smem + a.off_misc;
    uint64_t* bars = reinterpret_cast<uint64_t*>(misc);              // 3 mbarriers
    Ctl* ctl = reinterpret_cast<Ctl*>(misc + 64);
    float* red = reinterpret_cast<float*>(misc + 128);               // >= 72 floats
    float* cs = reinterpret_cast<float*>(misc + 512);                // cos [hd], sin [hd]
    float* xo = reinterpret_cast<float*>(misc + 2112);               // this CTA's rows of x [rpC <= 64]
    float* tpv = reinterpret_cast<float*>(misc + 2112 + 256);        // P > 1: exchanged rows [P][64]
    const int tid = threadIdx.x;
    if (a.P > 1) {
        // a rank poisoned by an earlier exchange that gave up runs nothing (no
        // barrier arrival, no copy, no packet) until tb_qwen3_tp_reset
        if (__syncthreads_or(tid == 0 && *reinterpret_cast<const volatile unsigned*>(a.poison) != 0u)) {
            if (tid == 0 && blockIdx.x == 0) atomicCAS(a.err, 0, ERR_STEP_TP_POISONED);   // keeps a first error
            return;
        }
    }
    const int pos = a.pos[0];
    if (tid == 0 && blockIdx.x == 0 && step_S(a, pos) == 0) atomicExch(a.err, ERR_ATTN_POS);
    stamp(a, 0);

    if (tid == 0) {
        // every launch adds a whole number of grids of arrivals, and no barrier of
        // this launch opens before every CTA arrived, so each CTA reads the count
        // at most grid - 1 arrivals into this launch: rounding down gives the base
        const unsigned long long c0 = ld_acquire_u64(a.bar_count);
        ctl->base = c0 - c0 % gridDim.x;
        ctl->nb = 0;
        ctl->tag = (unsigned)(ctl->base / gridDim.x) + 1u;
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
    // the per-layer pointer records, on chip for the whole launch
    StepLayer* sl = reinterpret_cast<StepLayer*>(smem + a.off_layers);
    for (int i = tid; i < a.L * (int)(sizeof(StepLayer) / 8); i += THREADS)
        reinterpret_cast<unsigned long long*>(sl)[i] = reinterpret_cast<const unsigned long long*>(a.layers)[i];
    __syncthreads();
    if (tid == 0) {
        request(a, ctl, BUF_R, 0, 0, smem, bars);
        request(a, ctl, BUF_Q, 4, 0, smem, bars);
    }
    attn_prefetch<GRP>(a, sl[0], smem);
    // this launch's head counters start at zero; the embed barrier below orders
    // the zeroing before any phase-A arrival
    for (int i = blockIdx.x * THREADS + tid; i < a.L * a.nKv; i += gridDim.x * THREADS) a.head_cnt[i] = 0u;
    // embed: this CTA's rows of x (the o / down row slice)
    {
        const int r0 = rowsC0(a), n = rowsC(a);
        const uint32_t id = a.ids[0];
        for (int i = tid; i < n; i += THREADS) {
            const float e = tb_h2f(a.embed[(long long)id * a.H + r0 + i]);
            xo[i] = e;
            a.x[r0 + i] = e;
        }
    }
    if (!grid_sync(a, ctl)) goto drain;

    // epochs of this launch's phase-boundary packets (x after o, one GPU): ebase +
    // 3l + 1.  Every launch that writes packets has passed the embed barrier, so its
    // base (grid barriers before it) exceeds an earlier one's and the epoch ranges
    // of two launches never meet; a reader waits for equality, and the earlier
    // writer of a slot (the layer before, the launch before) carries another epoch.
    // (Packets at the gate/up -> down and down -> q/k/v boundaries measured slower
    // than the barriers there: every CTA polling all 6144 swi / 2048 x values
    // loads L2 harder than one counter, and those boundaries stay barriers.)
    {
    const unsigned ebase = (unsigned)(ctl->base / gridDim.x) * (unsigned)(3 * a.L);
    for (int l = 0; l < a.L; l++) {
        const StepLayer& Ly = sl[l];
        const bool more = l + 1 < a.L;
        // ---- A: rmsnorm + quant of x, q/k/v rows, prep of completed heads
        {
            if (!await_buf(a, ctl, BUF_R, bars)) goto drain;
            STAMP(0, 0);
            const BlockA b = block_a(a);
            const unsigned char* wR = smem + a.off_R;
            const uint16_t* nws = reinterpret_cast<const uint16_t*>(wR + (b.live ? mat_bytes(a, RBA, a.H) : 0));
            if (b.live) stage<TERN>(a, smem, a.x, a.H, true, nws, red, 1 + 25 * l + 5 * 0 + 1);
            if (tid == 0 && l > 0) request(a, ctl, BUF_Q, 4, l, smem, bars);   // Q held E(l-1)
            STAMP_REQ(0);
            if (b.live) {
                float* y = b.mat == WQ ? a.q : (b.mat == WK ? a.k : a.v);
                gemv_rows<1, TERN>(smem + a.off_act, wR, nullptr, RBA, a.H / 32, y, b.row0, nullptr);
            }
            __syncthreads();           // the block's rows are written before thread 0's release
            STAMP(0, 3);
            if (b.live && tid == 0 && !ctl->abort) {
                const int kvh = b.mat == WQ ? b.row0 / STEP_HD / (a.nHq / a.nKv) : b.row0 / STEP_HD;
                red_release_add_u32(a.head_cnt + (size_t)l * a.nKv + kvh, 1u);
            }
            STAMP(0, 4);
        }
        // ---- B: attention (prep'd q, cache row pos written in A)
        {
            STAMP(1, 0);
            // (requests are issued after the phase's own critical loads, so the
            // barrier and the activation loads do not queue behind them)
            if (tid == 0) request(a, ctl, BUF_R, 2, l, smem, bars);
            STAMP_REQ(1);
            attn_run<GRP, TERN>(a, ctl, Ly, l, smem, cs, pos);
            __syncthreads();
            STAMP(1, 3);
            if (!grid_sync(a, ctl)) goto drain;
            STAMP(1, 4);
        }
        // ---- C: quant of the attention output, o rows += x
        {
            if (!await_buf(a, ctl, BUF_R, bars)) goto drain;
            STAMP(2, 0);
            const int n = rowsC(a);
            if (n > 0) {    // the combining units stored the quantized attention output
                const int nq = a.nHq * STEP_HD / 32 * 40 / 16;
                for (int i = tid; i < nq; i += THREADS)
                    reinterpret_cast<uint4*>(smem + a.off_act)[i] = __ldcg(reinterpret_cast<const uint4*>(a.attnq) + i);
                __syncthreads();
                STAMP(2, 2);
            }
            if (tid == 0) request(a, ctl, BUF_P, 3, l, smem, bars);
            STAMP_REQ(2);
            if (n > 0) {
                if (a.P > 1)    // this rank's partial rows -> its arena, then the exchange
                    gemv_rows<1, TERN>(smem + a.off_act, smem + a.off_R, nullptr, n, a.nHq * STEP_HD / 32, a.xpart,
                                       rowsC0(a), nullptr);
                else
                    gemv_rows<1, TERN>(smem + a.off_act, smem + a.off_R, nullptr, n, a.nHq * STEP_HD / 32, a.x,
                                       rowsC0(a), xo, a.xpk, ebase + 3 * l + 1);
            }
            __syncthreads();
            if (a.P > 1 && !tp_exchange(a, ctl, 2 * l, xo, tpv)) goto drain;
            STAMP(2, 3);
            // one GPU: phase D reads x as packets, no barrier; under TP, after the exchange
            if (a.P > 1 && !grid_sync(a, ctl)) goto drain;
            STAMP(2, 4);
        }
        // ---- D: rmsnorm + quant of x, gate/up rows, swiglu
        {
            if (!await_buf(a, ctl, BUF_P, bars)) goto drain;
            STAMP(3, 0);
            const int n = rowsD(a);
            const unsigned char* wP = smem + a.off_P;
            if (n > 0) {
                const uint16_t* nws = reinterpret_cast<const uint16_t*>(wP + 2 * mat_bytes(a, n, a.H));
                if (a.P == 1) {
                    if (!stage_pk<TERN>(a, ctl, smem, a.xpk, ebase + 3 * l + 1, a.H, true, nws, red,
                                        1 + 25 * l + 5 * 3 + 1))
                        goto drain;
                } else {
                    stage<TERN>(a, smem, a.x, a.H, true, nws, red, 1 + 25 * l + 5 * 3 + 1);
                }
            }
            if (tid == 0 && more) request(a, ctl, BUF_R, 0, l + 1, smem, bars);
            STAMP_REQ(3);
            if (n > 0) {
                gemv_rows<2, TERN>(smem + a.off_act, wP, wP + mat_bytes(a, n, a.H), n, a.H / 32, a.swi, rowsD0(a),
                                   nullptr);
            }
            __syncthreads();
            STAMP(3, 3);
            if (!grid_sync(a, ctl)) goto drain;
            STAMP(3, 4);
        }
        // ---- E: quant of swi, down rows += x
        {
            if (!await_buf(a, ctl, BUF_Q, bars)) goto drain;
            STAMP(4, 0);
            const int n = rowsC(a);
            if (n > 0) stage<TERN>(a, smem, a.swi, a.I, false, nullptr, red, 1 + 25 * l + 5 * 4 + 1);
            if (more) attn_prefetch<GRP>(a, sl[l + 1], smem);
            STAMP_REQ(4);
            if (n > 0) {
                if (a.P > 1)
                    gemv_rows<1, TERN>(smem + a.off_act, smem + a.off_Q, nullptr, n, a.I / 32, a.xpart + a.H,
                                       rowsC0(a), nullptr);
                else
                    gemv_rows<1, TERN>(smem + a.off_act, smem + a.off_Q, nullptr, n, a.I / 32, a.x, rowsC0(a), xo);
            }
            __syncthreads();
            if (a.P > 1 && !tp_exchange(a, ctl, 2 * l + 1, xo, tpv)) goto drain;
            STAMP(4, 3);
            if (more && !grid_sync(a, ctl)) goto drain;
            STAMP(4, 4);
        }
    }
    }
drain:
    // copies still in flight land before the CTA's shared memory is released
    cp_async_wait<0>();
    __syncthreads();
    if (tid == 0 && a.P > 1 && ctl->abort) atomicExch(a.poison, 1u);   // epochs may disagree from here on
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
                      int tern, int P, tb_step_plan** out)
{
    *out = nullptr;
    const int G = ctx->num_sms;
    const int grp = nKv > 0 ? nHq / nKv : 0;
    if (hd != STEP_HD || nKv <= 0 || nHq % nKv || (grp != 1 && grp != 2 && grp != 4 && grp != 8))
        return TB_ERR_UNSUPPORTED;
    // K % 256: every slice's scales (n * K/16 bytes) are whole 16-byte chunks for the bulk copies
    // K <= 8192: the activation staging holds a row in 8 float4 per thread
    if (H % 256 || I % 256 || (nHq * hd) % 256 || H > 8192 || I > 8192 || nHq * hd > 8192) return TB_ERR_UNSUPPORTED;
    if ((nHq + 2 * nKv) * hd / RBA > G) return TB_ERR_UNSUPPORTED;   // one phase-A block per CTA
    if (nsplit < 1 || nsplit > 256) return TB_ERR_UNSUPPORTED;
    StepArgs a{};
    a.L = L; a.H = H; a.nHq = nHq; a.nKv = nKv; a.I = I; a.nsplit = nsplit; a.max_seq = max_seq;
    a.tern = tern ? 1 : 0;
    a.P = P > 1 ? P : 1;
    if (a.P > TB_TP_MAX) return TB_ERR_UNSUPPORTED;
    // the exchange epochs (P > 1): a launch passes 1 + 3L + (L - 1) = 4L grid
    // barriers (the embed, after attention, after o's exchange, after gate/up,
    // after down's exchange but the last) and has 2L exchanges; epochs stay unique
    // across launches while 4L >= 2L + 1.  One GPU passes 3L (no barrier after o).
    if (4 * L < 2 * L + 1) return TB_ERR_UNSUPPORTED;
    a.rpC = (H + G - 1) / G;
    a.rpD = (I + G - 1) / G;
    if (a.rpC > 64) return TB_ERR_UNSUPPORTED;      // own rows of x kept in shared memory
    auto mb = [&](int n, int K) { return (size_t)n * ((K >> (a.tern ? 2 : 1)) + K / 16); };
    // one 8-warp unit per CTA with one 32-key tile per warp at the longest context
    const int per = (max_seq + nsplit - 1) / nsplit;
    if (nKv * nsplit > G || per > UW * 32) return TB_ERR_UNSUPPORTED;
    size_t unit_bytes = 0;
    switch (grp) {
    case 1: unit_bytes = DecLayout<STEP_HD, 1, 1, UW>::BYTES; break;
    case 2: unit_bytes = DecLayout<STEP_HD, 2, 1, UW>::BYTES; break;
    case 4: unit_bytes = DecLayout<STEP_HD, 4, 1, UW>::BYTES; break;
    default: unit_bytes = DecLayout<STEP_HD, 8, 1, UW>::BYTES; break;
    }
    auto up = [](size_t v) { return (v + 127) & ~size_t(127); };
    const size_t bP = up(std::max(unit_bytes, 2 * mb(a.rpD, H) + (size_t)H * 2));
    const size_t bQ = up(mb(a.rpC, I));
    const size_t bR = up(std::max(mb(RBA, H) + (size_t)H * 2, mb(a.rpC, nHq * hd)));
    const int Kmax = std::max(std::max(H, I), nHq * hd);
    const size_t act = up((size_t)(Kmax / 32) * 40);
    // barriers, control, reduction, rope table, own rows of x, exchanged rows (P > 1)
    const size_t misc = 2112 + 64 * 4 + (a.P > 1 ? (size_t)TB_TP_MAX * 64 * 4 : 0);
    a.off_P = 0;
    a.off_Q = (int)bP;
    a.off_R = (int)(bP + bQ);
    a.off_act = (int)(bP + bQ + bR);
    a.off_misc = (int)(bP + bQ + bR + act);
    a.off_layers = (int)(bP + bQ + bR + act + misc);
    const size_t total = (size_t)a.off_layers + (size_t)L * sizeof(StepLayer);
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
    a.attnq = io->attnq;
    a.PO = io->PO; a.PML = io->PML; a.counters = io->counters;
    a.bar_count = reinterpret_cast<unsigned long long*>(io->ctrl + 64); a.abort_word = io->ctrl + 128;
    a.head_cnt = io->head_cnt;
    a.xpk = io->pk;
    TB_REQUIRE(ctx, a.head_cnt != nullptr && a.xpk != nullptr, "decode step: no head counters / packet buffers");
    a.err = ctx->dev_error;
    a.trace = reinterpret_cast<unsigned long long*>(io->trace);
    const int P = io->P > 1 ? io->P : 1;
    TB_REQUIRE(ctx, P == a.P && io->rank >= 0 && io->rank < P, "decode step: tensor-parallel ranks differ from the plan");
    a.rank = io->rank;
    if (P > 1) {
        for (int s = 0; s < P; s++) {
            TB_REQUIRE(ctx, io->tp_inbox[s], "decode step: exchange arena of rank %d not mapped", s);
            a.peer_inbox[s] = io->tp_inbox[s];
        }
        TB_REQUIRE(ctx, io->xpart && io->tp_poison, "decode step: this rank's exchange arena is not set");
        a.xpart = io->xpart;
        a.my_inbox = io->tp_inbox[a.rank];
        a.poison = io->tp_poison;
    }
    void (*kern)(const StepArgs) = nullptr;
    if (a.tern) {
        switch (p->grp) {
        case 1: kern = k_decode_step<1, true>; break;
        case 2: kern = k_decode_step<2, true>; break;
        case 4: kern = k_decode_step<4, true>; break;
        default: kern = k_decode_step<8, true>; break;
        }
    } else {
        switch (p->grp) {
        case 1: kern = k_decode_step<1, false>; break;
        case 2: kern = k_decode_step<2, false>; break;
        case 4: kern = k_decode_step<4, false>; break;
        default: kern = k_decode_step<8, false>; break;
        }
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
