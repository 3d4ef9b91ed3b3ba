// tb_gemm_i8.cu -- the reference's integer prefill GEMM (gemmDP4A for int4 weights,
// gemmTern for the ternary WebGPU layout; models/qwen3.js gemmdp4Wgsl :1321-1407,
// gemmTern :1410-1420) on the 5th-generation tensor cores: tcgen05.mma kind::i8
// with the int32 group sums in TMEM.
//
// y[m][n] (epilogue) sum_g (f32(s[n][g]) * xs[m][g]) * S_g[m][n], S_g the exact
// int32 sum over the 32 k of group g of xq[m][k] * w[n][k] (w = nib - 8, or
// code - 1), folded into f32 in group order with one fma per group -- the
// reference's dot4I8Packed group sums scaled once per group, and the same values
// in the same order as the warp-level form (tb_gemm_dp4.cu), so the two are
// bit-equal.
//
// One kind::i8 MMA has K = 32: exactly one scale group.  Every MMA therefore
// writes a fresh 128 x 128 int32 tile into one of four TMEM slots (512 columns),
// and sixteen epilogue warps turn slot after slot into f32 while the tensor core
// fills the next ones.  The weights enter the MMA as raw unsigned nibbles (or
// ternary codes 0..2) widened to bytes, so the MMA sums xq * nib; the offset is
// removed in the int32 -> f32 conversion: as_float(S + kc) - 1.5 * 2^23 with
// kc = 0x4B400000 - 8 * sum_k xq (ternary: - 1 * sum), exact for |S| < 2^22.
//
// Warp roles (704 threads, one CTA an SM, persistent over 128 x 128 tiles):
//   warp 0      one thread issues the TMA copies of a k-step (128 k): the X tile
//               (128 rows x 128 int8, 128-byte swizzle, exactly the layout the
//               MMA descriptor reads) and the raw packed weight tile;
//   warps 1-4   widen the raw weights into the swizzled B tile (byte masks and
//               permutes, no arithmetic), form kc from the X tile (dp4a against
//               ones), stage xs and the f16 weight scales as f32;
//   warp 5      owns TMEM; one thread issues four MMAs a k-step, each into its
//               group slot, and commits each slot to the epilogue;
//   warps 6-21  read a slot (32 TMEM lanes = rows x 32 columns per warp, one
//               TMEM load), release it, and fold it into 32 f32 accumulators a
//               thread; after the last k-step of a tile they apply the epilogue and
//               store the rows (four of them a scheduler: 1.02x the throughput of
//               two with 64 columns each).
// The f32 folding is the bound (2.5 packed-f32 instructions an output per 32
// MACs), so the MMA and the operand staging run on other warps.
// Every wait is bounded: a wait that gives up records ERR_I8_WAIT in the context's
// error word and raises the CTA's abort flag, every role leaves its loop, the TMA
// thread waits for its copies in flight, and TMEM is freed.
#include "tb_internal.h"

namespace {

constexpr int BM = 128, BN = 128, BK = 128, NG = BK / 32;   // 4 scale groups a k-step
constexpr int NST = 4;                                        // k-step stages
constexpr int A_BYTES = BM * BK, B_BYTES = BN * BK;           // 16 KB each, 1024-aligned
constexpr int RAW_BYTES = BN * BK / 2;                        // packed int4 (ternary uses half)
constexpr int WS_BYTES = NG * BN * 4;                         // f32 weight scales [group][col]
constexpr int XK_BYTES = NG * BM * 8;                         // {xs, kc} [group][row]
constexpr int STAGE = A_BYTES + B_BYTES + RAW_BYTES + WS_BYTES + XK_BYTES;
static_assert(STAGE % 1024 == 0, "stages keep the 1024-byte swizzle alignment");
constexpr int SMEM = 1024 + NST * STAGE + 256;
static_assert(SMEM <= 227 * 1024, "shared memory");
constexpr int W_TMA = 0, W_WIDEN = 1, N_WIDEN = 4, W_MMA = 5, W_EPI = 6, N_EPI = 16;
constexpr int THREADS = (W_EPI + N_EPI) * 32;
constexpr int EPI_COLS = BN * 4 / N_EPI;                      // columns a warp folds (4 lane quarters)
static_assert(EPI_COLS % 32 == 0, "whole 32-column TMEM loads");
// registers are allocated per scheduler (16384 each): 22 warps put 6 on some of
// them, so 6 x 32 x MAX_REGS must fit
constexpr int MAX_REGS = 80;
static_assert(((THREADS / 32 + 3) / 4) * 32 * MAX_REGS <= 16384, "registers per scheduler");
constexpr int NSLOT = NG, TMEM_COLS = NSLOT * BN;             // one 128-column slot a group
static_assert(TMEM_COLS == 512, "TMEM");
constexpr int WAIT_TRIES = 1000;       // x a 1 ms suspend hint per try: at most ~1 s a wait
constexpr int ERR_I8_WAIT = 0x6b02;
constexpr uint32_t KC_MAGIC = 0x4B400000u;   // as_float = 1.5 * 2^23

// kind::i8 instruction descriptor: D s32 (bits 4-5 = 2), A signed (bit 7), B
// unsigned, both K-major, N >> 3 at bit 17, M >> 4 at bit 24
constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (0u << 10) | ((uint32_t)(BN >> 3) << 17) |
                           ((uint32_t)(BM >> 4) << 24);

struct I8Args {
    CUtensorMap ta;         // xq [M][K] int8, box 128 x 128, 128-byte swizzle
    CUtensorMap tw;         // packed weights as bytes [N][K/2] (ternary [N][K/4]), box 64 (32) x 128
    const float* xs;        // [M][K/32]
    const uint16_t* scales; // [N][K/32] f16
    float* y;               // [M][N]
    int M, N, K, epi, tiles_n, tiles;
    int* err;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* b, unsigned count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* b)
{
    asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(b)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
// true once the phase with this parity has completed; false when the CTA's abort
// flag (if given) is up or after the limit (try_wait suspends up to the 1 ms hint
// per try)
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity, volatile int* abort_flag)
{
    const uint32_t a = smem_u32(b);
    for (int it = 0; it < WAIT_TRIES; it++) {
        uint32_t done;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
                     " selp.u32 %0, 1, 0, p;\n}"
                     : "=r"(done) : "r"(a), "r"(parity), "r"(1000000u) : "memory");
        if (done) return true;
        if (abort_flag && *abort_flag) return false;
    }
    return false;
}
// the same wait by every lane of a warp, with one outcome for the whole warp (the
// lanes then run the .aligned tcgen05 loads and __syncwarp together)
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* b, uint32_t parity, volatile int* abort_flag)
{
    const bool ok = __all_sync(0xffffffffu, mbar_wait(b, parity, abort_flag));
    __syncwarp();
    return ok;
}
__device__ __forceinline__ void give_up(volatile int* abort_flag, int* err)
{
    *abort_flag = 1;
    atomicExch(err, ERR_I8_WAIT);
}

__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
                 : "memory");
}

// K-major operand, 128-byte swizzle: 8-row atoms of 128-byte rows 1024 bytes apart
__device__ __forceinline__ uint64_t kmajor_sw128_desc(uint32_t saddr)
{
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// byte offset of 16-byte chunk c (0..7) of row r in a swizzled K-major tile
__device__ __forceinline__ uint32_t sw128(int r, int c) { return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ float2 fmul2(float2 a, float2 b)
{
    float2 d;
    asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2,%3};\n mov.b64 rb, {%4,%5};\n"
        " mul.rn.f32x2 rd, ra, rb;\n mov.b64 {%0,%1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// 8 packed nibbles (k = 8i..8i+7 at bits 4(k-8i)) -> 8 unsigned bytes in k order
__device__ __forceinline__ uint2 widen_nib(uint32_t w)
{
    const uint32_t lo = w & 0x0f0f0f0fu, hi = (w >> 4) & 0x0f0f0f0fu;   // k 0 2 4 6 / 1 3 5 7
    return make_uint2(__byte_perm(lo, hi, 0x5140), __byte_perm(lo, hi, 0x7362));
}
// 16 ternary codes (k = 4s+b at bits 8b+2s) -> 16 unsigned bytes in k order
__device__ __forceinline__ uint4 widen_code(uint32_t w)
{
    constexpr uint32_t M = 0x03030303u;
    return make_uint4(w & M, (w >> 2) & M, (w >> 4) & M, (w >> 6) & M);
}

// 32 columns of TMEM (this warp's 32 lanes) into registers
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r)
{
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
                 "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                   "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
                   "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
                   "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
                   "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
}

// the k-step `it` of this CTA: its tile's first row and column, and k-step index
struct Step {
    int m0, n0, ks;
};
__device__ __forceinline__ Step step_of(const I8Args& a, int it, int nk)
{
    const int t = (int)blockIdx.x + (it / nk) * (int)gridDim.x;
    return Step{(t / a.tiles_n) * BM, (t % a.tiles_n) * BN, it % nk};
}

template <bool TERN>
__global__ void __maxnreg__(MAX_REGS) k_gemm_i8(const __grid_constant__ I8Args a)
{
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* base = smem_raw + (((raw + 1023) & ~1023u) - raw);
    uint64_t* full_tma = reinterpret_cast<uint64_t*>(base + NST * STAGE);   // X and raw weight copies landed
    uint64_t* full = full_tma + NST;                                         // B, scales and kc staged
    uint64_t* empty = full + NST;                                            // stage free (MMA + epilogue)
    uint64_t* tfull = empty + NST;                                           // TMEM slot written
    uint64_t* tempty = tfull + NSLOT;                                        // TMEM slot read
    uint64_t* done = tempty + NSLOT;                                         // every MMA completed
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(done + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nk = a.K / BK, G = a.K / 32;
    const int my_tiles = a.tiles > (int)blockIdx.x ? (a.tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int total = my_tiles * nk;   // k-steps this CTA runs, over all its tiles
    if (tid == 0) {
        for (int s = 0; s < NST; s++) {
            mbar_init(&full_tma[s], 1);
            mbar_init(&full[s], N_WIDEN);
            mbar_init(&empty[s], 1 + N_EPI);
        }
        for (int j = 0; j < NSLOT; j++) {
            mbar_init(&tfull[j], 1);
            mbar_init(&tempty[j], N_EPI);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == W_MMA) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32((const void*)tmem_slot)), "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    tb_pdl_wait();
    tb_pdl_trigger();

    if (warp == W_TMA) {
        if (lane == 0) {
            int it = 0;
            for (; it < total; it++) {
                const int s = it % NST;
                if (!mbar_wait(&empty[s], ((it / NST) & 1) ^ 1, abort_flag)) {
                    give_up(abort_flag, a.err);
                    break;
                }
                const Step st = step_of(a, it, nk);
                uint8_t* sb = base + s * STAGE;
                mbar_expect_tx(&full_tma[s], (uint32_t)(A_BYTES + (TERN ? RAW_BYTES / 2 : RAW_BYTES)));
                tma_2d(sb, &a.ta, st.ks * BK, st.m0, &full_tma[s]);
                tma_2d(sb + A_BYTES + B_BYTES, &a.tw, st.ks * (TERN ? BK / 4 : BK / 2), st.n0, &full_tma[s]);
            }
            // no copy may land after the CTA has left: wait for the last stages issued
            for (int i = it > NST ? it - NST : 0; i < it; i++) mbar_wait(&full_tma[i % NST], (i / NST) & 1, nullptr);
        }
    } else if (warp < W_WIDEN + N_WIDEN) {
        const int wt = tid - 32 * W_WIDEN;   // row of the X tile (kc, xs) and of the weight tile (scales)
        for (int it = 0; it < total; it++) {
            const int s = it % NST;
            const Step st = step_of(a, it, nk);
            const float4 xv = __ldg(reinterpret_cast<const float4*>(a.xs + (size_t)(st.m0 + wt) * G + st.ks * NG));
            const uint2 sv = __ldg(reinterpret_cast<const uint2*>(a.scales + (size_t)(st.n0 + wt) * G + st.ks * NG));
            if (!mbar_wait_warp(&full_tma[s], (it / NST) & 1, abort_flag)) {
                give_up(abort_flag, a.err);
                break;
            }
            uint8_t* A = base + s * STAGE;
            uint8_t* B = A + A_BYTES;
            const uint8_t* RW = B + B_BYTES;
            float* WS = reinterpret_cast<float*>(A + A_BYTES + B_BYTES + RAW_BYTES);
            uint2* XK = reinterpret_cast<uint2*>(A + A_BYTES + B_BYTES + RAW_BYTES + WS_BYTES);
            // B: 128 rows x 8 chunks of 16 k; chunk q of this thread: row q/8, chunk q%8
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const int q = i * 128 + wt, r = q >> 3, c = q & 7;
                uint4 o;
                if (TERN) {
                    o = widen_code(*reinterpret_cast<const uint32_t*>(RW + r * 32 + 4 * c));
                } else {
                    const uint2 w2 = *reinterpret_cast<const uint2*>(RW + r * 64 + 8 * c);
                    const uint2 p = widen_nib(w2.x), p2 = widen_nib(w2.y);
                    o = make_uint4(p.x, p.y, p2.x, p2.y);
                }
                *reinterpret_cast<uint4*>(B + sw128(r, c)) = o;
            }
            // kc of row wt: the sum of its int8 activations over each group
            int sum[NG] = {0, 0, 0, 0};
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const uint4 v = *reinterpret_cast<const uint4*>(A + sw128(wt, c));
                int t = sum[c >> 1];
                t = __dp4a((int)v.x, 0x01010101, t);
                t = __dp4a((int)v.y, 0x01010101, t);
                t = __dp4a((int)v.z, 0x01010101, t);
                t = __dp4a((int)v.w, 0x01010101, t);
                sum[c >> 1] = t;
            }
            const float xsv[NG] = {xv.x, xv.y, xv.z, xv.w};
            const uint32_t sc[NG] = {sv.x & 0xffffu, sv.x >> 16, sv.y & 0xffffu, sv.y >> 16};
#pragma unroll
            for (int g = 0; g < NG; g++) {
                XK[g * BM + wt] = make_uint2(__float_as_uint(xsv[g]), KC_MAGIC - (uint32_t)((TERN ? 1 : 8) * sum[g]));
                WS[g * BN + wt] = tb_h2f((uint16_t)sc[g]);
            }
            // generic-proxy writes of B -> visible to the tensor core (async proxy)
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[s]);
        }
    } else if (warp == W_MMA) {
        if (lane == 0) {
            for (int it = 0; it < total; it++) {
                const int s = it % NST;
                if (!mbar_wait(&full_tma[s], (it / NST) & 1, abort_flag) ||
                    !mbar_wait(&full[s], (it / NST) & 1, abort_flag)) {
                    give_up(abort_flag, a.err);
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t A = smem_u32(base + s * STAGE), Bt = A + A_BYTES;
                bool ok = true;
                for (int g = 0; g < NG; g++) {
                    if (!mbar_wait(&tempty[g], (it & 1) ^ 1, abort_flag)) {
                        give_up(abort_flag, a.err);
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint64_t da = kmajor_sw128_desc(A + 32 * g), db = kmajor_sw128_desc(Bt + 32 * g);
                    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                                 " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}"
                                 ::"r"(tmem + (uint32_t)(BN * g)), "l"(da), "l"(db), "r"(IDESC), "r"(0u), "r"(0u)
                                 : "memory");
                    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                                 ::"r"(smem_u32(&tfull[g])) : "memory");
                }
                if (!ok) break;
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                             ::"r"(smem_u32(&empty[s])) : "memory");
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         ::"r"(smem_u32(done)) : "memory");
            if (!mbar_wait(done, 0, nullptr)) give_up(abort_flag, a.err);   // no MMA in flight past here
        }
    } else {
        // ---- epilogue: TMEM lanes 32q.. (tile rows), columns EPI_COLS*h ..
        const int q = warp & 3, h = (warp - W_EPI) >> 2, rl = 32 * q + lane;
        const float2 M2 = make_float2(-12582912.f, -12582912.f);
        float2 acc[EPI_COLS / 2];
#pragma unroll
        for (int i = 0; i < EPI_COLS / 2; i++) acc[i] = make_float2(0.f, 0.f);
        for (int it = 0; it < total; it++) {
            const int s = it % NST;
            const Step st = step_of(a, it, nk);
            if (!mbar_wait_warp(&full[s], (it / NST) & 1, abort_flag)) {   // this stage's scales and kc
                give_up(abort_flag, a.err);
                break;
            }
            const uint8_t* sb = base + s * STAGE;
            const float* WS = reinterpret_cast<const float*>(sb + A_BYTES + B_BYTES + RAW_BYTES);
            const uint2* XK = reinterpret_cast<const uint2*>(sb + A_BYTES + B_BYTES + RAW_BYTES + WS_BYTES);
            bool ok = true;
#pragma unroll 1
            for (int g = 0; g < NG; g++) {
                const uint2 xk = XK[g * BM + rl];
                const float2 X2 = make_float2(__uint_as_float(xk.x), __uint_as_float(xk.x));
                const uint32_t kc = xk.y;
                if (!mbar_wait_warp(&tfull[g], it & 1, abort_flag)) {
                    give_up(abort_flag, a.err);
                    ok = false;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
#pragma unroll
                for (int j = 0; j < EPI_COLS / 32; j++) {
                    uint32_t r[32];
                    tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(BN * g + EPI_COLS * h + 32 * j), r);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    const float4* wp = reinterpret_cast<const float4*>(WS + g * BN + EPI_COLS * h + 32 * j);
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        const float4 w = wp[c];
                        // exact group sum: as_float(S + kc) - 1.5 * 2^23
                        const float2 f0 = fadd2(make_float2(__uint_as_float(r[4 * c] + kc),
                                                            __uint_as_float(r[4 * c + 1] + kc)), M2);
                        const float2 f1 = fadd2(make_float2(__uint_as_float(r[4 * c + 2] + kc),
                                                            __uint_as_float(r[4 * c + 3] + kc)), M2);
                        // f32(s) * xs per output (the shader's f32(sc) * xsc), then * the group sum
                        float2& a0 = acc[16 * j + 2 * c];
                        float2& a1 = acc[16 * j + 2 * c + 1];
                        a0 = ffma2(fmul2(make_float2(w.x, w.y), X2), f0, a0);
                        a1 = ffma2(fmul2(make_float2(w.z, w.w), X2), f1, a1);
                    }
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[g]);
            }
            if (!ok) break;
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            if (st.ks == nk - 1) {
                float4* yp = reinterpret_cast<float4*>(a.y + (size_t)(st.m0 + rl) * a.N + st.n0 + EPI_COLS * h);
#pragma unroll
                for (int c = 0; c < EPI_COLS / 4; c++) {
                    float4 v = make_float4(acc[2 * c].x, acc[2 * c].y, acc[2 * c + 1].x, acc[2 * c + 1].y);
                    if (a.epi == 1) {          // fused residual: y += X W^T
                        const float4 o = yp[c];
                        v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
                    } else if (a.epi == 2) {   // fused SwiGLU: y holds gate, y = silu(gate) * (X W_up^T)
                        const float4 gt = yp[c];
                        v.x = __fdiv_rn(gt.x, 1.0f + expf(-gt.x)) * v.x;
                        v.y = __fdiv_rn(gt.y, 1.0f + expf(-gt.y)) * v.y;
                        v.z = __fdiv_rn(gt.z, 1.0f + expf(-gt.z)) * v.z;
                        v.w = __fdiv_rn(gt.w, 1.0f + expf(-gt.w)) * v.w;
                    }
                    yp[c] = v;
                    acc[2 * c] = acc[2 * c + 1] = make_float2(0.f, 0.f);
                }
            }
        }
    }

    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == W_MMA) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
}

template <bool TERN>
int launch_i8(tb_ctx* ctx, const I8Args& a, int grid)
{
    static bool attr[64] = {};
    if (ctx->device >= 64 || !attr[ctx->device]) {
        cudaError_t e = cudaFuncSetAttribute(k_gemm_i8<TERN>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
        if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "gemm_i8 attribute: %s", cudaGetErrorString(e));
        if (ctx->device < 64) attr[ctx->device] = true;
    }
    cudaError_t e = tb_launch(ctx, k_gemm_i8<TERN>, dim3(grid), dim3(THREADS), (size_t)SMEM, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "gemm_i8 launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

}  // namespace

// gemmDP4A / gemmTern with exact group sums on tcgen05 (the product's prefill route)
int tb_gemm_dp4_impl(tb_ctx* ctx, float* y, const int8_t* xq, const float* xs, const uint32_t* pack,
                     const uint16_t* scales, int64_t M, int64_t N, int64_t K, int epilogue, bool tern)
{
    TB_REQUIRE(ctx, y && xq && xs && pack && scales, "null pointer");
    TB_REQUIRE(ctx, M > 0 && M % BM == 0 && N > 0 && N % BN == 0 && K > 0 && K % BK == 0,
               "gemm_dp4: M %% %d, N %% %d and K %% %d must be 0 (got %lld x %lld x %lld)", BM, BN, BK,
               (long long)M, (long long)N, (long long)K);
    TB_REQUIRE(ctx, (M / BM) * (N / BN) < (1LL << 31) && M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 30),
               "gemm_dp4: shape too large");
    TB_REQUIRE(ctx, epilogue >= 0 && epilogue <= 2, "gemm_dp4: bad epilogue %d", epilogue);
    TB_REQUIRE(ctx, TB_ALIGNED(xq, 16) && TB_ALIGNED(xs, 16) && TB_ALIGNED(pack, 16) && TB_ALIGNED(scales, 8) &&
                        TB_ALIGNED(y, 16),
               "gemm_dp4: xq, xs, pack, y 16-byte and scales 8-byte aligned");
    I8Args a{};
    int rc = tb_encode_2d(ctx, &a.ta, xq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, K, M, BK, BM,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc)
        rc = tb_encode_2d(ctx, &a.tw, pack, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, tern ? K / 4 : K / 2, N,
                          tern ? BK / 4 : BK / 2, BN, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    a.xs = xs;
    a.scales = scales;
    a.y = y;
    a.M = (int)M;
    a.N = (int)N;
    a.K = (int)K;
    a.epi = epilogue;
    a.tiles_n = (int)(N / BN);
    a.tiles = (int)((M / BM) * (N / BN));
    a.err = ctx->dev_error;
    const int grid = a.tiles < ctx->num_sms ? a.tiles : ctx->num_sms;
    return tern ? launch_i8<true>(ctx, a, grid) : launch_i8<false>(ctx, a, grid);
}

extern "C" TB_API int tb_gemm_dp4(tb_ctx* ctx, float* y, const int8_t* xq, const float* xs, const uint32_t* pack,
                                  const uint16_t* scales, int64_t M, int64_t N, int64_t K, int epilogue, int tern)
{
    if (!ctx) return TB_ERR_INVALID;
    return tb_gemm_dp4_impl(ctx, y, xq, xs, pack, scales, M, N, K, epilogue, tern != 0);
}
