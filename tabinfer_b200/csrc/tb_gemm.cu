// tb_gemm.cu -- prefill GEMM Y[M,N] (+)= f16(X[M,K]) . f16(deq(W[N,K]))^T on the
// 5th-generation tensor cores (tcgen05.mma kind::f16, f32 accumulators in TMEM).
//
// The math is the reference's f16 prefill GEMM (gemmqWgsl / gemmQ,
// models/qwen3.js:964-1026): every activation is rounded to f16, every weight is
// dequantized as f16((nib - 8) * f16 scale) (one rounding of the exact product),
// and the products are summed in f32.
//
// X is rounded to f16 once, by a pre-pass into context scratch (f32 or bf16 rows,
// or QUANTQ8T rows as f16(xs * q)), padded with zero rows to 256, so the A tiles
// arrive by TMA in the 128-byte swizzle the MMA descriptor reads, with no
// conversion work inside the GEMM; the pre-pass writes each 8-group in the k order
// the weight dequant produces its f16 pairs (no byte permutes in the producers).
// CTA tile 256 (M) x 256 (N) -- each dequantized weight tile (the producer work,
// fused here) feeds two 128 x 256 x 16 MMAs per k16, one per 128-row half of the X
// tile, into two 256-column f32 accumulators (all 512 TMEM columns) -- or 128 x 256
// when that costs fewer whole waves; K in steps of 64.  One thread of warp 17
// issues per k-step two tensor copies: the raw packed weight tile and the X tile.
// Warps 0-15 are producers: each thread reads its 32-weight group of the raw tile
// and writes it dequantized into the swizzled B tile; its two group scales come
// from a register ring filled 8 k-steps ahead (16-byte loads of 8 groups when
// K % 256 == 0, else a 4-byte cp.async NR-1 k-steps ahead).  Warp 16 owns TMEM
// and one of its threads issues the MMAs.  After the last stage warps 0-15 read
// the accumulators (warp w: TMEM lanes 32*(w%4).., columns 64*(w/4).. of both) and
// store f32 rows.  When the tiles leave SMs idle the K range is split across
// grid.z: each split stores its raw sums into context scratch and
// k_splitk_reduce adds them in split order and applies the epilogue.
// Ternary weights in the WebGPU layout (gemmTern, qwen3.js:1410-1420) use the
// same pipeline with the operands of that GEMM: X as QUANTQ8T int8 rows with
// per-32 f32 scales becomes f16(xs * q); a weight becomes the exact f16
// (c - 1) * s.  (The reference sums the int8 products of a group exactly and
// scales once per group; here f16(xs * q) rounds each activation to 11 bits,
// ~1e-4 of a row's scale.)  Waits are bounded: on a timeout the CTA records
// ERR_GEMM_WAIT, stops issuing, waits for its copies, and still frees its TMEM.
#include "tb_internal.h"

namespace {

constexpr int BM = 256, BN = 256, BK = 64, MMA_M = 128;   // BM: the largest tile (HM = 2 row halves)
constexpr int PROD_WARPS = 16, PROD = PROD_WARPS * 32;
constexpr int W_MMA = PROD_WARPS, W_TMA = PROD_WARPS + 1, THREADS = PROD + 64;
// per k-step stage: HM row halves of X (16 KB each) + the weight tile (32 KB)
template <int HM> constexpr int a_bytes() { return HM * MMA_M * BK * 2; }
constexpr int B_BYTES = BN * BK * 2;
template <int HM> constexpr int stage_bytes() { return a_bytes<HM>() + B_BYTES; }
constexpr int NST = 3;   // MMA operand stages
constexpr int NR = 3;    // raw weight stages, filled NR-1 k-steps ahead of the dequant
// raw staging: the packed W tile of a k-step as [256 rows][32 bytes] (ternary 16),
// copied by TMA -- thread t = 2 row + half reads bytes 16 t .. (ternary 8 t ..),
// one 32-group -- then the rows' two f16 group scales of the k-step, 4 bytes a
// thread (cp.async by the thread itself)
constexpr int RAW_W = PROD * 16, RAW_S = PROD * 4, RSTAGE = RAW_W + RAW_S;
template <int HM> constexpr int smem_bytes() { return 1024 + NST * stage_bytes<HM>() + NR * RSTAGE + 256; }
static_assert(smem_bytes<2>() <= 227 * 1024, "shared memory");
constexpr int TMEM_COLS = 512;   // two 256-column f32 accumulators
constexpr int GEMM_WAIT_TRIES = 1000;      // x a 1 ms suspend bound per try: at most ~1 s
constexpr int ERR_GEMM_WAIT = 0x6b01;
// X as given: f32 / bf16 rows (gemmQ), or QUANTQ8T int8 rows + f32 group scales
enum XMode { X_F32 = 0, X_BF16 = 1, X_Q8 = 2 };

struct GemmArgs {
    CUtensorMap tx;         // f16 X [Mpad][K] (the pre-pass output), box 64 x 128 HM, 128-byte swizzle
    CUtensorMap tw;         // packed weights as bytes [N][K/2] (ternary [N][K/4]), box 32 (16) x 256
    const uint32_t* pack;   // [N][K/8] int4, or [N][K/16] ternary codes
    const uint16_t* scales; // [N][K/32] f16
    float* y;               // [M][N]
    int M, N, K, acc;
    // split-K: CTA z of grid.z runs k-steps [z kps, (z + 1) kps) and, with part set,
    // stores its raw f32 sums into part[z][M][N] for k_splitk_reduce
    int kps;
    float* part;
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
// true once the phase with this parity has completed; false after the limit.
// try_wait suspends the thread until the phase completes (woken at once) or the
// 1 ms hint runs out, so the loop is bounded in time.
__device__ __forceinline__ bool mbar_wait(uint64_t* b, uint32_t parity)
{
    const uint32_t a = smem_u32(b);
    for (int it = 0; it < GEMM_WAIT_TRIES; it++) {
        uint32_t done;
        asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
                     " selp.u32 %0, 1, 0, p;\n}"
                     : "=r"(done) : "r"(a), "r"(parity), "r"(1000000u) : "memory");
        if (done) return true;
    }
    return false;
}

// K-major operand, 128-byte swizzle: 8-row atoms of 128-byte rows, atoms 1024
// bytes apart (stride byte offset), leading byte offset unused (16 B).
__device__ __forceinline__ uint64_t kmajor_sw128_desc(uint32_t saddr)
{
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// kind::f16 instruction descriptor: D f32, A and B f16, both K-major, N = BN, M = 128
constexpr uint32_t IDESC = (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(BN >> 3) << 17) |
                           ((uint32_t)(MMA_M >> 4) << 24);

// byte offset of 16-byte chunk c (0..7) of row r in a swizzled K-major tile
__device__ __forceinline__ uint32_t sw128(int r, int c) { return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ uint32_t f32x2_to_f16x2(float lo, float hi)
{
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

__device__ __forceinline__ void cp4(void* sdst, const void* gsrc)
{
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(sdst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// 8 weights of one packed word -> 8 f16 f16((nib - 8) * s), in the pair order the
// magic-number nibbles come out (k 0 4 1 5 2 6 3 7; 16 bytes)
__device__ __forceinline__ uint4 dequant_word(uint32_t w, uint32_t s2)
{
    const uint32_t magic = 0x64006400u;   // f16 1024 + nib in both halves
    uint32_t p0 = (w & 0x000F000Fu) | magic;           // k0, k4
    uint32_t p1 = ((w >> 4) & 0x000F000Fu) | magic;    // k1, k5
    uint32_t p2 = ((w >> 8) & 0x000F000Fu) | magic;    // k2, k6
    uint32_t p3 = ((w >> 12) & 0x000F000Fu) | magic;   // k3, k7
    const uint32_t bias = 0x64086408u;                 // 1032 = 1024 + 8
    asm("sub.rn.f16x2 %0, %0, %1;" : "+r"(p0) : "r"(bias));
    asm("sub.rn.f16x2 %0, %0, %1;" : "+r"(p1) : "r"(bias));
    asm("sub.rn.f16x2 %0, %0, %1;" : "+r"(p2) : "r"(bias));
    asm("sub.rn.f16x2 %0, %0, %1;" : "+r"(p3) : "r"(bias));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(p0) : "r"(s2));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(p1) : "r"(s2));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(p2) : "r"(s2));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(p3) : "r"(s2));
    return make_uint4(p0, p1, p2, p3);   // k 0 4 1 5 2 6 3 7 (X is written in the same order)
}

// 8 ternary codes k = 8h..8h+7 of one word (k = 4s+b at bits 8b+2s, s = 2h, 2h+1)
// -> 8 f16 (c - 1) * s in the pair order they come out (k 0 2 1 3 4 6 5 7 of the
// 8; 16 bytes); exact: c - 1 is -1, 0 or 1.
__device__ __forceinline__ uint4 dequant_tern8(uint32_t w, int h, uint32_t s2)
{
    const uint32_t magic = 0x64006400u;   // f16 1024 + c in both halves
    const uint32_t lo = w >> (4 * h), hi = w >> (4 * h + 2);
    uint32_t p0 = (lo & 0x00030003u) | magic;          // s = 2h:   b0, b2
    uint32_t p1 = ((lo >> 8) & 0x00030003u) | magic;   //           b1, b3
    uint32_t p2 = (hi & 0x00030003u) | magic;          // s = 2h+1: b0, b2
    uint32_t p3 = ((hi >> 8) & 0x00030003u) | magic;   //           b1, b3
    const uint32_t bias = 0x64016401u;                 // 1025 = 1024 + 1
    asm("sub.rn.f16x2 %0, %0, %1;" : "+r"(p0) : "r"(bias));
    asm("sub.rn.f16x2 %0, %0, %1;" : "+r"(p1) : "r"(bias));
    asm("sub.rn.f16x2 %0, %0, %1;" : "+r"(p2) : "r"(bias));
    asm("sub.rn.f16x2 %0, %0, %1;" : "+r"(p3) : "r"(bias));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(p0) : "r"(s2));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(p1) : "r"(s2));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(p2) : "r"(s2));
    asm("mul.rn.f16x2 %0, %0, %1;" : "+r"(p3) : "r"(s2));
    return make_uint4(p0, p1, p2, p3);   // k 0 2 1 3 4 6 5 7 of the 8 (X is written in the same order)
}

// 4 int8 (one word) -> 4 floats exactly (2^23 + (q ^ 0x80) - (2^23 + 128)), times xs
__device__ __forceinline__ void q8x4_scaled(uint32_t w, float xs, float2& a, float2& b)
{
    const uint32_t u = w ^ 0x80808080u;
    const float2 M2 = make_float2(-8388736.0f, -8388736.0f);   // -(2^23 + 128)
    const float2 S2 = make_float2(xs, xs);
    a = fadd2(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)),
                          __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541))), M2);
    b = fadd2(make_float2(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)),
                          __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543))), M2);
    a = make_float2(__fmul_rn(a.x, S2.x), __fmul_rn(a.y, S2.y));
    b = make_float2(__fmul_rn(b.x, S2.x), __fmul_rn(b.y, S2.y));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* b, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar)
{
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
                 : "memory");
}

// X -> f16 rows [Mpad][K], rows M.. zero: 8 elements (16 bytes out) a thread, grid-stride.
// Each 8-group is written in the k order the weight dequant produces without byte
// permutes (TERN false: k 0 4 1 5 2 6 3 7; true: 0 2 1 3 4 6 5 7), so A and B agree
// and every product of the GEMM is the same; only the summation order inside an
// MMA differs from natural k order.
template <int MODE, bool TERN>
__global__ void __launch_bounds__(256) k_x_f16(const void* __restrict__ x, const float* __restrict__ xs,
                                               uint4* __restrict__ out, long long n8, long long n8_valid)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    for (long long i = (long long)blockIdx.x * 256 + threadIdx.x; i < n8; i += (long long)gridDim.x * 256) {
        uint4 o = make_uint4(0u, 0u, 0u, 0u);
        if (i < n8_valid) {
            float f[8];
            if (MODE == X_F32) {
                const float4 u = __ldg(reinterpret_cast<const float4*>(x) + 2 * i);
                const float4 v = __ldg(reinterpret_cast<const float4*>(x) + 2 * i + 1);
                f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w; f[4] = v.x; f[5] = v.y; f[6] = v.z; f[7] = v.w;
            } else if (MODE == X_BF16) {
                const uint4 v = __ldg(reinterpret_cast<const uint4*>(x) + i);
                const uint32_t in[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    f[2 * j] = __uint_as_float(in[j] << 16);
                    f[2 * j + 1] = __uint_as_float(in[j] & 0xFFFF0000u);
                }
            } else {
                const uint2 q = __ldg(reinterpret_cast<const uint2*>(x) + i);
                const float xsc = __ldg(xs + ((8 * i) >> 5));   // [M][K/32]: element e's group is e / 32
                float2 p0, p1, p2, p3;
                q8x4_scaled(q.x, xsc, p0, p1);
                q8x4_scaled(q.y, xsc, p2, p3);
                f[0] = p0.x; f[1] = p0.y; f[2] = p1.x; f[3] = p1.y; f[4] = p2.x; f[5] = p2.y; f[6] = p3.x; f[7] = p3.y;
            }
            if (TERN)
                o = make_uint4(f32x2_to_f16x2(f[0], f[2]), f32x2_to_f16x2(f[1], f[3]), f32x2_to_f16x2(f[4], f[6]),
                               f32x2_to_f16x2(f[5], f[7]));
            else
                o = make_uint4(f32x2_to_f16x2(f[0], f[4]), f32x2_to_f16x2(f[1], f[5]), f32x2_to_f16x2(f[2], f[6]),
                               f32x2_to_f16x2(f[3], f[7]));
        }
        out[i] = o;
    }
}

template <bool TERN, int HM>
__global__ void __launch_bounds__(THREADS, 1) k_gemm_f16(const __grid_constant__ GemmArgs a)
{
    constexpr int A_BYTES = a_bytes<HM>(), STAGE = stage_bytes<HM>();
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw = smem_u32(smem_raw);
    uint8_t* base = smem_raw + (((raw + 1023) & ~1023u) - raw);
    uint8_t* rawbase = base + NST * STAGE;
    uint64_t* full = reinterpret_cast<uint64_t*>(rawbase + NR * RSTAGE);   // B dequantized + X tile landed
    uint64_t* empty = full + NST;                                          // stage consumed by the MMAs
    uint64_t* rfull = empty + NST;                                         // raw weight tile landed
    uint64_t* rempty = rfull + NR;                                         // raw weight tile read
    uint64_t* done = rempty + NR;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(done + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(done + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < NST; s++) {
            mbar_init(&full[s], PROD_WARPS + 1);   // the producer warps + the X copy's expect_tx arrival
            mbar_init(&empty[s], 1);
        }
        for (int r = 0; r < NR; r++) {
            mbar_init(&rfull[r], 1);
            mbar_init(&rempty[r], PROD_WARPS);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == W_MMA) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32((const void*)tmem_slot)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;
    tb_pdl_wait();
    tb_pdl_trigger();

    const int m0 = blockIdx.y * (MMA_M * HM), n0 = blockIdx.x * BN;
    // this CTA's k-steps: kb .. kb + nk - 1 (loops below count i from 0; data at kb + i)
    const int kb = (int)blockIdx.z * a.kps;
    const int nk = min(a.K / BK - kb, a.kps);
    if (warp < PROD_WARPS) {
        // ---- producers: W rows (2 threads a row, one 32-group each).  The raw
        // weight tile arrives by TMA (rfull); each thread copies its own two group
        // scales (cp.async, NR-1 k-steps ahead).
        const int wr = tid >> 1, wh = tid & 1;
        // scales: with 16-byte aligned scale rows (K % 256 == 0) one 16-byte load
        // brings 8 groups (4 k-steps) into a 3-deep register ring, 8 k-steps ahead;
        // otherwise a 4-byte cp.async a k-step, NR-1 k-steps ahead
        const bool svec = (a.K % 256) == 0;
        const uint16_t* srow = a.scales + (size_t)(n0 + wr) * (a.K / 32);
        auto sload = [&](int i) {   // groups 2(kb+i) .. +7 (k-steps kb+i .. +3), kb + i % 4 == 0
            return i < nk ? __ldg(reinterpret_cast<const uint4*>(srow + 2 * (kb + i))) : make_uint4(0u, 0u, 0u, 0u);
        };
        uint4 sq0 = make_uint4(0u, 0u, 0u, 0u), sq1 = sq0, sq2 = sq0;
        if (svec) {
            sq0 = sload(0);
            sq1 = sload(4);
            sq2 = sload(8);
        }
        auto fetch = [&](int i) {
            if (!svec && i < nk) {
                uint8_t* rs = rawbase + (i % NR) * RSTAGE;
                cp4(rs + RAW_W + tid * 4, srow + (kb + i) * BK / 32);
            }
            cp_commit();   // a group per k-step, empty past the end, keeps the count uniform
        };
        for (int i = 0; i < NR - 1; i++) fetch(i);
        for (int i = 0; i < nk; i++) {
            fetch(i + NR - 1);
            cp_wait<NR - 1>();        // this thread's raw bytes of k-step i have landed
            const int s = i % NST;
            if (!mbar_wait(&empty[s], ((i / NST) & 1) ^ 1)) {
                *abort_flag = 1;
                atomicExch(a.err, ERR_GEMM_WAIT);
            }
            if (*abort_flag) break;
            const int r = i % NR;
            if (!__all_sync(0xffffffffu, mbar_wait(&rfull[r], (i / NR) & 1))) {
                *abort_flag = 1;
                atomicExch(a.err, ERR_GEMM_WAIT);
                break;
            }
            uint8_t* Bt = base + s * STAGE + A_BYTES;
            const uint8_t* rs = rawbase + r * RSTAGE;
            if (svec && i > 0 && (i & 3) == 0) {
                sq0 = sq1;
                sq1 = sq2;
                sq2 = sload(i + 8);
            }
            const int iq = i & 3;
            const uint32_t sc = svec ? (iq == 0 ? sq0.x : iq == 1 ? sq0.y : iq == 2 ? sq0.z : sq0.w)
                                     : *reinterpret_cast<const uint32_t*>(rs + RAW_W + tid * 4);
            const uint32_t s2 = (wh ? (sc >> 16) : (sc & 0xFFFFu)) * 0x10001u;
            uint4 w4;
            if (TERN) {
                const uint2 w2 = *reinterpret_cast<const uint2*>(rs + tid * 8);
                w4 = make_uint4(w2.x, w2.y, 0u, 0u);
            } else {
                w4 = *reinterpret_cast<const uint4*>(rs + tid * 16);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&rempty[r]);   // this warp's raw weight bytes are in registers
            if (TERN) {
#pragma unroll
                for (int c = 0; c < 4; c++)
                    *reinterpret_cast<uint4*>(Bt + sw128(wr, 4 * wh + c)) = dequant_tern8(c < 2 ? w4.x : w4.y, c & 1, s2);
            } else {
                const uint32_t ws[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                for (int c = 0; c < 4; c++) *reinterpret_cast<uint4*>(Bt + sw128(wr, 4 * wh + c)) = dequant_word(ws[c], s2);
            }
            // generic-proxy writes -> visible to the tensor core (async proxy)
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[s]);
        }
        cp_wait<0>();   // no copy in flight when the CTA leaves
    } else if (warp == W_TMA) {
        if (lane == 0) {
            // ---- per k-step: the raw weight tile (256 rows x 32 bytes) and the X
            // tile (128 HM rows x 64 f16), one tensor copy each
            constexpr uint32_t WBYTES = TERN ? BN * BK / 4 : BN * BK / 2;
            int issued_w = 0, issued_x = 0;
            for (int i = 0; i < nk; i++) {
                const int s = i % NST, r = i % NR;
                if (!mbar_wait(&rempty[r], ((i / NR) & 1) ^ 1)) {
                    *abort_flag = 1;
                    atomicExch(a.err, ERR_GEMM_WAIT);
                }
                if (*abort_flag) break;
                mbar_expect_tx(&rfull[r], WBYTES);
                tma_2d(rawbase + r * RSTAGE, &a.tw, (kb + i) * (TERN ? BK / 4 : BK / 2), n0, &rfull[r]);
                issued_w = i + 1;
                if (!mbar_wait(&empty[s], ((i / NST) & 1) ^ 1)) {
                    *abort_flag = 1;
                    atomicExch(a.err, ERR_GEMM_WAIT);
                }
                if (*abort_flag) break;
                mbar_expect_tx(&full[s], (uint32_t)A_BYTES);
                tma_2d(base + s * STAGE, &a.tx, (kb + i) * BK, m0, &full[s]);
                issued_x = i + 1;
            }
            // no copy may land after the CTA has left: wait for the last copies issued
            // (their barriers complete when the bytes land; full also needs the
            // producers, so on an abort that wait runs to its bound)
            for (int i = issued_w > NR ? issued_w - NR : 0; i < issued_w; i++) mbar_wait(&rfull[i % NR], (i / NR) & 1);
            for (int i = issued_x > NST ? issued_x - NST : 0; i < issued_x; i++) mbar_wait(&full[i % NST], (i / NST) & 1);
        }
    } else if (lane == 0) {
        // ---- MMA issuer: per k16, rows 0-127 into columns 0-255, rows 128-255 into 256-511
        for (int i = 0; i < nk; i++) {
            const int s = i % NST;
            if (!mbar_wait(&full[s], (i / NST) & 1)) {
                *abort_flag = 1;
                atomicExch(a.err, ERR_GEMM_WAIT);
            }
            if (*abort_flag) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t A = smem_u32(base + s * STAGE), Bt = A + A_BYTES;
#pragma unroll
            for (int kk = 0; kk < BK / 16; kk++) {
                const uint64_t db = kmajor_sw128_desc(Bt + kk * 32);
                const uint32_t accum = (i > 0 || kk > 0) ? 1u : 0u;
#pragma unroll
                for (int hm = 0; hm < HM; hm++) {
                    const uint64_t da = kmajor_sw128_desc(A + hm * (MMA_M * 128) + kk * 32);
                    asm volatile("{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
                                 " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n}"
                                 ::"r"(tmem + (uint32_t)(hm * BN)), "l"(da), "l"(db), "r"(IDESC), "r"(accum), "r"(0u)
                                 : "memory");
                }
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         ::"r"(smem_u32(&empty[s])) : "memory");
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     ::"r"(smem_u32(done)) : "memory");
    }

    if (warp == W_MMA && lane == 0) mbar_wait(done, 0);   // every MMA completed before TMEM is freed
    if (warp < PROD_WARPS) {
        // ---- epilogue: this warp's 32 TMEM lanes x 64 columns of both accumulators
        const bool ok = __all_sync(0xffffffffu, mbar_wait(done, 0) && !*abort_flag);
        __syncwarp();
        if (!ok && lane == 0) atomicExch(a.err, ERR_GEMM_WAIT);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        if (ok) {
            const int q = warp & 3, h = warp >> 2;      // TMEM lanes 32q.., columns 64h..
#pragma unroll 1
            for (int hm = 0; hm < HM; hm++) {
                const int row = m0 + hm * MMA_M + 32 * q + lane;
                float* yrow = (a.part ? a.part + (size_t)blockIdx.z * a.M * a.N : a.y) + (size_t)row * a.N + n0 + 64 * h;
#pragma unroll 1
                for (int j = 0; j < 2; j++) {
                    uint32_t r[32];
                    const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(hm * BN + 64 * h + 32 * j);
                    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
                                 "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
                                   "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
                                   "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
                                   "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
                                   "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                                 : "r"(taddr));
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                    if (row >= a.M) continue;   // zero padding rows of the last tile
                    float4* yp = reinterpret_cast<float4*>(yrow + 32 * j);
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        float4 v = make_float4(__uint_as_float(r[4 * c]), __uint_as_float(r[4 * c + 1]),
                                               __uint_as_float(r[4 * c + 2]), __uint_as_float(r[4 * c + 3]));
                        if (a.part) {
                        } else if (a.acc == 1) {   // fused residual: y += X W^T
                            const float4 o = yp[c];
                            v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
                        } else if (a.acc == 2) {   // fused SwiGLU: y holds gate, y = silu(gate) * (X W_up^T)
                            const float4 gt = yp[c];
                            v.x = __fdiv_rn(gt.x, 1.0f + expf(-gt.x)) * v.x;
                            v.y = __fdiv_rn(gt.y, 1.0f + expf(-gt.y)) * v.y;
                            v.z = __fdiv_rn(gt.z, 1.0f + expf(-gt.z)) * v.z;
                            v.w = __fdiv_rn(gt.w, 1.0f + expf(-gt.w)) * v.w;
                        }
                        yp[c] = v;
                    }
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

// y (epilogue)= the sum of the split-K partials in split order: part [nsplit][M][N]
__global__ void __launch_bounds__(256) k_splitk_reduce(const float4* __restrict__ part, int nsplit, long long n4,
                                                       float4* __restrict__ y, int acc)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    for (long long i = (long long)blockIdx.x * 256 + threadIdx.x; i < n4; i += (long long)gridDim.x * 256) {
        float4 v = part[i];
        for (int z = 1; z < nsplit; z++) {
            const float4 p = part[(long long)z * n4 + i];
            v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
        }
        if (acc == 1) {
            const float4 o = y[i];
            v.x += o.x; v.y += o.y; v.z += o.z; v.w += o.w;
        } else if (acc == 2) {
            const float4 gt = y[i];
            v.x = __fdiv_rn(gt.x, 1.0f + expf(-gt.x)) * v.x;
            v.y = __fdiv_rn(gt.y, 1.0f + expf(-gt.y)) * v.y;
            v.z = __fdiv_rn(gt.z, 1.0f + expf(-gt.z)) * v.z;
            v.w = __fdiv_rn(gt.w, 1.0f + expf(-gt.w)) * v.w;
        }
        y[i] = v;
    }
}

template <bool TERN, int HM>
int launch_gemm(tb_ctx* ctx, const GemmArgs& a, int64_t M)
{
    static bool attr_set[64] = {};
    if (ctx->device >= 64 || !attr_set[ctx->device]) {
        cudaError_t e = cudaFuncSetAttribute(k_gemm_f16<TERN, HM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             smem_bytes<HM>());
        if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "gemm attribute: %s", cudaGetErrorString(e));
        if (ctx->device < 64) attr_set[ctx->device] = true;
    }
    const unsigned rows = (unsigned)((M + MMA_M * HM - 1) / (MMA_M * HM));
    const unsigned splits = (unsigned)((a.K / BK + a.kps - 1) / a.kps);
    cudaError_t e = tb_launch(ctx, k_gemm_f16<TERN, HM>, dim3(a.N / BN, rows, splits), dim3(THREADS),
                              (size_t)smem_bytes<HM>(), a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "gemm launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

// X rounded to f16 into context scratch ([Mpad][K], zero rows past M), then the GEMM
int run_gemm(tb_ctx* ctx, float* y, const void* x, int mode, const float* xs, const uint32_t* pack,
             const uint16_t* scales, int64_t M, int64_t N, int64_t K, int acc, bool tern)
{
    const int64_t Mpad = (M + BM - 1) / BM * BM;
    // two 128-row halves a CTA (each weight tile dequantized once per 256 rows), or
    // one when that costs fewer whole waves (a 128-row tile taking ~0.6 of the time)
    const int64_t t2 = ((M + BM - 1) / BM) * (N / BN), t1 = (M / MMA_M) * (N / BN);
    const int64_t w2 = (t2 + ctx->num_sms - 1) / ctx->num_sms, w1 = (t1 + ctx->num_sms - 1) / ctx->num_sms;
    const int hm = 10 * w2 <= 6 * w1 ? 2 : 1;
    // split-K when the tiles leave SMs idle: at most 8 splits of at least 4 k-steps,
    // split boundaries on 4 k-steps (the scale loads' 8-group alignment)
    const int64_t tiles = hm == 2 ? t2 : t1, nk = K / BK;
    int64_t sk = ctx->num_sms / tiles;
    if (sk > 8) sk = 8;
    if (sk > nk / 4) sk = nk / 4;
    if (sk < 1) sk = 1;
    const int64_t kps = ((nk + sk - 1) / sk + 3) / 4 * 4;
    sk = (nk + kps - 1) / kps;
    const size_t xbytes = ((size_t)(Mpad * K * 2) + 255) & ~(size_t)255;
    const size_t pbytes = sk > 1 ? (size_t)(sk * M * N * 4) : 0;
    unsigned char* scr = static_cast<unsigned char*>(tb_ctx_scratch(ctx, xbytes + pbytes));
    if (!scr) return TB_ERR_NOMEM;
    uint4* xf = reinterpret_cast<uint4*>(scr);
    float* part = sk > 1 ? reinterpret_cast<float*>(scr + xbytes) : nullptr;
    const long long n8 = Mpad * K / 8, n8v = M * K / 8;
    const long long want = (n8 + 255) / 256, cap = (long long)ctx->num_sms * 16;
    const dim3 grid((unsigned)(want < cap ? want : cap));
    cudaError_t e;
    if (tern) e = tb_launch(ctx, k_x_f16<X_Q8, true>, grid, dim3(256), 0, x, xs, xf, n8, n8v);
    else if (mode == X_F32) e = tb_launch(ctx, k_x_f16<X_F32, false>, grid, dim3(256), 0, x, xs, xf, n8, n8v);
    else if (mode == X_BF16) e = tb_launch(ctx, k_x_f16<X_BF16, false>, grid, dim3(256), 0, x, xs, xf, n8, n8v);
    else e = tb_launch(ctx, k_x_f16<X_Q8, false>, grid, dim3(256), 0, x, xs, xf, n8, n8v);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "gemm x pass launch: %s", cudaGetErrorString(e));
    GemmArgs a{};
    int rc = tb_encode_2d(ctx, &a.tx, xf, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K, Mpad, BK, MMA_M * hm,
                          CU_TENSOR_MAP_SWIZZLE_128B);
    if (!rc)
        rc = tb_encode_2d(ctx, &a.tw, pack, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, tern ? K / 4 : K / 2, N,
                          tern ? BK / 4 : BK / 2, BN, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    a.pack = pack;
    a.scales = scales;
    a.y = y;
    a.M = (int)M;
    a.N = (int)N;
    a.K = (int)K;
    a.acc = acc;
    a.kps = (int)kps;
    a.part = part;
    a.err = ctx->dev_error;
    if (hm == 2) rc = tern ? launch_gemm<true, 2>(ctx, a, M) : launch_gemm<false, 2>(ctx, a, M);
    else rc = tern ? launch_gemm<true, 1>(ctx, a, M) : launch_gemm<false, 1>(ctx, a, M);
    if (rc || sk == 1) return rc;
    const long long n4 = M * N / 4, rw = (n4 + 255) / 256;
    e = tb_launch(ctx, k_splitk_reduce, dim3((unsigned)(rw < cap ? rw : cap)), dim3(256), 0,
                  reinterpret_cast<const float4*>(part), (int)sk, n4, reinterpret_cast<float4*>(y), acc);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "gemm split-K reduce launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

}  // namespace

int tb_gemm_int4_impl(tb_ctx* ctx, float* y, const void* x, int x_bf16, const uint32_t* pack, const uint16_t* scales,
                      int64_t M, int64_t N, int64_t K, int acc)
{
    TB_REQUIRE(ctx, y && x && pack && scales, "null pointer");
    TB_REQUIRE(ctx, M > 0 && M % 128 == 0 && N > 0 && N % BN == 0 && K > 0 && K % BK == 0,
               "gemm_int4: M %% 128, N %% %d and K %% %d must be 0 (got %lld x %lld x %lld)", BN, BK,
               (long long)M, (long long)N, (long long)K);
    TB_REQUIRE(ctx, (M + BM - 1) / BM <= 65535 && K < (1LL << 30) && N * K < (1LL << 40), "gemm_int4: shape too large");
    TB_REQUIRE(ctx, TB_ALIGNED(x, 16) && TB_ALIGNED(pack, 16) && TB_ALIGNED(scales, 4) && TB_ALIGNED(y, 16),
               "gemm_int4: x, pack, y 16-byte and scales 4-byte aligned");
    return run_gemm(ctx, y, x, x_bf16 ? X_BF16 : X_F32, nullptr, pack, scales, M, N, K, acc ? 1 : 0, false);
}

// gemmDP4A (qwen3.js:1232-1400, linearQ's default prefill route) on the tensor
// cores: QUANTQ8T rows become f16(xs * q), int4 weights f16((nib - 8) * s).
// epilogue: 0 store, 1 y += (fused residual), 2 y = silu(y) * (fused SwiGLU).
int tb_gemm_q8_int4_impl(tb_ctx* ctx, float* y, const int8_t* xq, const float* xs, const uint32_t* pack,
                         const uint16_t* scales, int64_t M, int64_t N, int64_t K, int epilogue)
{
    TB_REQUIRE(ctx, y && xq && xs && pack && scales, "null pointer");
    TB_REQUIRE(ctx, M > 0 && M % 128 == 0 && N > 0 && N % BN == 0 && K > 0 && K % BK == 0,
               "gemm_q8: M %% 128, N %% %d and K %% %d must be 0 (got %lld x %lld x %lld)", BN, BK,
               (long long)M, (long long)N, (long long)K);
    TB_REQUIRE(ctx, (M + BM - 1) / BM <= 65535 && K < (1LL << 30) && N * K < (1LL << 40), "gemm_q8: shape too large");
    TB_REQUIRE(ctx, epilogue >= 0 && epilogue <= 2, "gemm_q8: bad epilogue %d", epilogue);
    TB_REQUIRE(ctx, TB_ALIGNED(xq, 16) && TB_ALIGNED(xs, 4) && TB_ALIGNED(pack, 16) && TB_ALIGNED(scales, 4) &&
                        TB_ALIGNED(y, 16),
               "gemm_q8: xq, pack, y 16-byte and xs, scales 4-byte aligned");
    return run_gemm(ctx, y, xq, X_Q8, xs, pack, scales, M, N, K, epilogue, false);
}

int tb_gemm_tern_wgsl_impl(tb_ctx* ctx, float* y, const int8_t* xq, const float* xs, const uint32_t* pack,
                           const uint16_t* scales, int64_t M, int64_t N, int64_t K, int acc)
{
    TB_REQUIRE(ctx, y && xq && xs && pack && scales, "null pointer");
    TB_REQUIRE(ctx, M > 0 && M % 128 == 0 && N > 0 && N % BN == 0 && K > 0 && K % BK == 0,
               "gemm_tern: M %% 128, N %% %d and K %% %d must be 0 (got %lld x %lld x %lld)", BN, BK,
               (long long)M, (long long)N, (long long)K);
    TB_REQUIRE(ctx, (M + BM - 1) / BM <= 65535 && K < (1LL << 30) && N * K < (1LL << 40), "gemm_tern: shape too large");
    TB_REQUIRE(ctx, TB_ALIGNED(xq, 16) && TB_ALIGNED(xs, 4) && TB_ALIGNED(pack, 16) && TB_ALIGNED(scales, 4) &&
                        TB_ALIGNED(y, 16),
               "gemm_tern: xq, pack, y 16-byte and xs, scales 4-byte aligned");
    TB_REQUIRE(ctx, acc >= 0 && acc <= 2, "gemm_tern: bad epilogue %d", acc);
    return run_gemm(ctx, y, xq, X_Q8, xs, pack, scales, M, N, K, acc, true);
}

extern "C" TB_API int tb_gemm_int4_q8(tb_ctx* ctx, float* y, const int8_t* xq, const float* xs, const uint32_t* pack,
                                      const uint16_t* scales, int64_t M, int64_t N, int64_t K, int epilogue)
{
    if (!ctx) return TB_ERR_INVALID;
    return tb_gemm_q8_int4_impl(ctx, y, xq, xs, pack, scales, M, N, K, epilogue);
}

extern "C" TB_API int tb_gemm_tern_wgsl(tb_ctx* ctx, float* y, const int8_t* xq, const float* xs, const uint32_t* pack,
                                        const uint16_t* scales, int64_t M, int64_t N, int64_t K, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    return tb_gemm_tern_wgsl_impl(ctx, y, xq, xs, pack, scales, M, N, K, acc);
}

extern "C" TB_API int tb_gemm_int4_g32(tb_ctx* ctx, float* y, const void* x, int x_bf16, const uint32_t* pack,
                                       const uint16_t* scales, int64_t M, int64_t N, int64_t K, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    return tb_gemm_int4_impl(ctx, y, x, x_bf16, pack, scales, M, N, K, acc);
}
