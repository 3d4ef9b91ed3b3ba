// tb_tern.cu -- ternary Q2_0_g64 path of the Bonsai engine
// (native/crates/n2-kernels/src/tern.rs, cpu/kernel/src/lib.rs).
//
// Format (native/docs/FORMAT.md:49-112): per row, K/64 groups; group = 16
// bytes of codes (code c in byte c%16 at bit 2*(c/16), value code-1) and one
// f32 scale.  out[n] = sum_b s*dot_b - sum_b s*xsum_b, two f32 chains summed
// in block order and subtracted once (tern.rs:79-119).
//
// GEMV design: a warp tile is TR consecutive rows, i.e. one contiguous run of
// TR*K/4 code bytes and TR*K/64 scales, loaded with perfectly coalesced 16-byte
// lane loads (phase A).  Each (row, group) item gives an exact int32 dot via
// 16 dp4a, and the rounded product s*dot is parked in shared memory.  Phase B
// gives one lane per (row, activation column) and sums the products serially
// in block order with separately rounded f32 adds, which reproduces
// gemv_tern_scalar bit for bit while the HBM stream stays fully parallel.
#include "tb_common.cuh"
#include "tb_gemv_dev.cuh"

namespace {

constexpr int TERN_THREADS = 128;
constexpr int TERN_WARPS = TERN_THREADS / 32;
constexpr int TERN_UNROLL = 4;

// ---- pack_ternary (tern.rs:131-160): one warp per (row, 64-group) ----------
__global__ void __launch_bounds__(256) k_pack_ternary(const float* __restrict__ w, uint8_t* __restrict__ codes,
                                                      float* __restrict__ scales, long long ngroups)
{
    // no early launch_dependents: a GEMV after it requests these codes before
    // its own wait, so it may start only once they are all written
    tb_pdl_wait();
    const int lane = threadIdx.x & 31;
    for (long long g = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; g < ngroups;
         g += ((long long)gridDim.x * blockDim.x) >> 5) {
        const float a = w[g * 64 + lane], b = w[g * 64 + 32 + lane];
        float s = fmaxf(fabsf(a), fabsf(b));
        s = warp_max(s);
        const float thr = s * 0.5f;
        const uint32_t ca = fabsf(a) < thr ? 1u : (a < 0.0f ? 0u : 2u);   // element lane
        const uint32_t cb = fabsf(b) < thr ? 1u : (b < 0.0f ? 0u : 2u);   // element 32+lane
        const uint32_t pa = __shfl_down_sync(0xffffffffu, ca, 16);          // element 16+lane
        const uint32_t pb = __shfl_down_sync(0xffffffffu, cb, 16);          // element 48+lane
        if (lane < 16) codes[g * 16 + lane] = (uint8_t)(ca | (pa << 2) | (cb << 4) | (pb << 6));
        if (lane == 0) scales[g] = s;
    }
}

// ---- quantize_act_into (tern.rs:206-222): one CTA per activation row -------
// WASM: the CPU engine's quantize (cpu/kernel/src/lib.rs:566-606) instead:
// asc = amax/127 (1e-9 for a zero row), x*(1/asc) rounded to nearest-even,
// and asc stored where tern.rs stores 127/amax.
template <bool WASM>
__global__ void __launch_bounds__(256) k_quant_act(const float* __restrict__ x, int8_t* __restrict__ act,
                                                   int32_t* __restrict__ xsum, float* __restrict__ scale_out, int K)
{
    __shared__ float red[32];
    tb_pdl_wait();
    tb_pdl_trigger();
    const int row = blockIdx.x, lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const float* xr = x + (long long)row * K;
    float m = 0.0f;
    for (int i = threadIdx.x; i < K; i += blockDim.x) m = fmaxf(m, fabsf(xr[i]));
    m = warp_max(m);
    if (lane == 0) red[wid] = m;
    __syncthreads();
    if (wid == 0) {
        float t = lane < nw ? red[lane] : 0.0f;
        t = warp_max(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    const float amax = red[0];
    float scale;
    if (WASM) {
        const float asc = amax > 0.0f ? __fdiv_rn(amax, 127.0f) : 1e-9f;
        if (threadIdx.x == 0) scale_out[row] = asc;
        scale = __fdiv_rn(1.0f, asc);
    } else {
        scale = amax > 0.0f ? __fdiv_rn(127.0f, amax) : 1.0f;
        if (threadIdx.x == 0) scale_out[row] = scale;
    }
    for (int g = wid; g < K / 64; g += nw) {
        int s = 0;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            int i = g * 64 + h * 32 + lane;
            // tern.rs: half away from zero (f32::round); WASM: f32x4_nearest, ties to even
            float v = WASM ? rintf(__fmul_rn(xr[i], scale)) : roundf(__fmul_rn(xr[i], scale));
            v = fminf(127.0f, fmaxf(-127.0f, v));
            int q = (int)v;
            act[(long long)row * K + i] = (int8_t)q;
            s += q;
        }
        s = (int)warp_sum((float)s);   // |s| <= 64*127: exact in f32
        if (lane == 0) xsum[(long long)row * (K / 64) + g] = s;
    }
}

// ---- ternary GEMV --------------------------------------------------------
struct TernArgs {
    float* out;
    const uint8_t* codes;
    const float* scales;
    const int8_t* act;
    const int32_t* xsum;
    const float* act_scale;   // optional [B]: out *= 1/act_scale (Model::linear, model.rs:334-337)
    int N, K, tiles;
};

// act chunk j (16 bytes = 4 words) of group b lives at slot j ^ ((b>>1)&3),
// which spreads 8 consecutive groups over 8 bank quads.
__device__ __forceinline__ int act_slot(int b, int j) { return b * 4 + (j ^ ((b >> 1) & 3)); }

template <int B>
__global__ void __launch_bounds__(TERN_THREADS) k_gemv_tern(const TernArgs a)
{
    constexpr int TR = B <= 4 ? 8 : 32 / B;   // rows per warp tile
    extern __shared__ __align__(128) unsigned char smem[];
    const int nb = a.K >> 6;
    const int ld = nb + 1;                      // padded row stride of the parking area
    uint4* act_s = reinterpret_cast<uint4*>(smem);                       // [B][nb*4]
    int* xsum_s = reinterpret_cast<int*>(act_s + B * nb * 4);            // [B][nb]
    float* park = reinterpret_cast<float*>(xsum_s + B * nb);             // per warp: S[TR][ld], P[B][TR][ld]
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    float* S = park + wid * (B + 1) * TR * ld;
    float* P = S + TR * ld;

    const int items = TR * nb;                 // (row, group) items per tile
    const int gw = blockIdx.x * TERN_WARPS + wid, nwarps = gridDim.x * TERN_WARPS;

    // prologue: first items of the first tile, before waiting on the producer
    uint4 cv[TERN_UNROLL];
    float sv[TERN_UNROLL];
    auto load_items = [&](int tile, int i0) {
        const long long base = (long long)tile * items;   // tile rows are contiguous
#pragma unroll
        for (int u = 0; u < TERN_UNROLL; u++) {
            int i = i0 + u * 32;
            long long gi = base + i;
            bool ok = i < items && gi < (long long)a.N * nb;
            cv[u] = ok ? ldg_stream_v4(a.codes + gi * 16) : make_uint4(0, 0, 0, 0);
            sv[u] = ok ? __ldg(a.scales + gi) : 0.0f;
        }
    };
    if (gw < a.tiles) load_items(gw, lane);

    tb_pdl_wait();
    tb_pdl_trigger();
    for (int i = threadIdx.x; i < B * nb * 4; i += blockDim.x) {
        int b = i / (nb * 4), r = i - b * nb * 4, g = r >> 2, j = r & 3;
        act_s[b * nb * 4 + act_slot(g, j)] = reinterpret_cast<const uint4*>(a.act + (long long)b * a.K)[g * 4 + j];
    }
    for (int i = threadIdx.x; i < B * nb; i += blockDim.x) xsum_s[i] = a.xsum[i];
    __syncthreads();

    for (int tile = gw; tile < a.tiles; tile += nwarps) {
        for (int i0 = lane;; i0 += TERN_UNROLL * 32) {
            if (tile != gw || i0 != lane) load_items(tile, i0);
#pragma unroll
            for (int u = 0; u < TERN_UNROLL; u++) {
                int i = i0 + u * 32;
                if (i >= items) break;
                const int r = i / nb, g = i - r * nb;
                const uint32_t cw[4] = {cv[u].x, cv[u].y, cv[u].z, cv[u].w};
#pragma unroll
                for (int b = 0; b < B; b++) {
                    const uint4* ab = act_s + b * nb * 4;
                    int d = 0;
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const uint4 av = ab[act_slot(g, j)];
                        const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
                        for (int w = 0; w < 4; w++)
                            d = __dp4a((int)((cw[w] >> (2 * j)) & 0x03030303u), (int)aw[w], d);
                    }
                    P[(b * TR + r) * ld + g] = __fmul_rn(sv[u], (float)d);
                }
                S[r * ld + g] = sv[u];
            }
            if (i0 + TERN_UNROLL * 32 >= items) break;
        }
        __syncwarp();
        if (lane < TR * B) {
            const int r = lane % TR, b = lane / TR;
            const int row = tile * TR + r;
            if (row < a.N) {
                const float* pr = P + (b * TR + r) * ld;
                const float* sr = S + r * ld;
                const int* xb = xsum_s + b * nb;
                float acc = 0.0f, sxs = 0.0f;
                for (int g = 0; g < nb; g++) {
                    acc = __fadd_rn(acc, pr[g]);
                    sxs = __fadd_rn(sxs, __fmul_rn(sr[g], (float)xb[g]));
                }
                float v = __fsub_rn(acc, sxs);
                if (a.act_scale) v = __fmul_rn(v, __fdiv_rn(1.0f, a.act_scale[b]));
                a.out[(long long)b * a.N + row] = v;
            }
        }
        __syncwarp();
    }
}

// ---- ternary GEMV, streaming form ------------------------------------------------
// The row tiles of a CTA (TR consecutive rows: one contiguous run of codes and
// one of scales) are staged in shared memory by cp.async.bulk in a ring of NST
// stages, the first NST requested before the grid waits on its producer (the
// weights do not depend on it).  Lane l of every warp owns the 64-groups
// l, l + 32, ... of the row: their int8 activations stay in registers for the
// whole CTA.  Warp w owns rows w*RW .. w*RW+RW-1 of a tile.  A (row, group) item
// is the exact i32 dot of the group's unsigned codes with the activations: each
// code word is split by masks into its four planes, scaled by 1, 4, 16, 64
// (dp4a.u32.s32 on the masked bytes), and the four sums are shifted back
// exactly.  The rounded pair (s*dot, s*xsum) of every item is parked in a
// CTA-wide buffer (two of them, alternating by tile), and one warp per tile --
// warp k % 8 for the CTA's k-th tile, so the chains rotate over the warps --
// gives each lane one (activation row, row) and adds the pairs serially in
// block order with one packed f32x2 add (two IEEE round-to-nearest lanes), as
// gemv_tern_scalar adds its two chains, so the result is bit for bit the
// scalar one.
constexpr int T2_THREADS = 256;
constexpr int T2_WARPS = T2_THREADS / 32;
constexpr int T2_ERR_WAIT = 0x6d02;

struct Tern2Args {
    float* out;
    const uint8_t* codes;
    const float* scales;
    const int8_t* act;
    const int32_t* xsum;
    const float* act_scale;   // optional [B]: out *= 1/act_scale
    int N, K, TR, NST, tiles;
    int stage_bytes;          // TR * (K/4 + nb*4) rounded up to 128
    int park_ld;              // float2 pairs per parked row
    int* err;
};

__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c)
{
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ float2 fmul2(float2 a, float2 b)
{
    float2 d;
    asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2,%3};\n mov.b64 rb, {%4,%5};\n"
        " mul.rn.f32x2 rd, ra, rb;\n mov.b64 {%0,%1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// CTAs an SM the streaming form is planned for: three at batch 1 with at most
// two 64-groups a lane (85 registers), else two
__host__ __device__ constexpr int t2_ctas(int B, int NBL) { return (B == 1 && NBL <= 2) ? 3 : 2; }

template <int B, int NBL>
__global__ void __launch_bounds__(T2_THREADS, t2_ctas(B, NBL)) k_gemv_tern2(const Tern2Args a)
{
    extern __shared__ __align__(128) unsigned char smem[];
    const int nb = a.K >> 6, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int TR = a.TR, RW = TR / T2_WARPS, ld = a.park_ld;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);                          // [NST]
    float2* park = reinterpret_cast<float2*>(smem + 128);                        // [2][B][TR][ld]
    const size_t park_pairs = (size_t)B * TR * ld;
    unsigned char* stages = smem + 128 + 2 * park_pairs * sizeof(float2);
    stages = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(stages) + 127) & ~uintptr_t(127));
    const int cb = a.K >> 2;                                     // code bytes a row
    const int my_tiles = a.tiles > (int)blockIdx.x ? (a.tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    auto issue = [&](int k) {                                    // thread 0: tile k of this CTA -> stage k % NST
        const int t = blockIdx.x + k * gridDim.x;
        const int row0 = t * TR, rows = min(TR, a.N - row0);
        unsigned char* st = stages + (size_t)(k % a.NST) * a.stage_bytes;
        uint64_t* bar = bars + (k % a.NST);
        const uint32_t c_bytes = (uint32_t)rows * cb, s_bytes = (uint32_t)rows * nb * 4;
        const bool sbulk = (s_bytes & 15u) == 0;
        mbar_expect_tx(bar, c_bytes + (sbulk ? s_bytes : 0u));
        bulk_g2s(st, a.codes + (size_t)row0 * cb, c_bytes, bar);
        if (sbulk) bulk_g2s(st + (size_t)TR * cb, a.scales + (size_t)row0 * nb, s_bytes, bar);
    };
    if (tid == 0) {
        for (int s = 0; s < a.NST; s++) mbar_init(&bars[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int k = 0; k < min(a.NST, my_tiles); k++) issue(k);
    }
    __syncthreads();
    tb_pdl_wait();
    tb_pdl_trigger();

    // this lane's activations: group g = lane + 32 i, plane j, word w
    uint32_t A[B][NBL][4][4];
    float xs[B][NBL];
#pragma unroll
    for (int b = 0; b < B; b++)
#pragma unroll
        for (int i = 0; i < NBL; i++) {
            const int g = lane + 32 * i;
            const bool ok = g < nb;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint4 v = ok ? __ldg(reinterpret_cast<const uint4*>(a.act + (size_t)b * a.K + g * 64) + j)
                                   : make_uint4(0, 0, 0, 0);
                A[b][i][j][0] = v.x; A[b][i][j][1] = v.y; A[b][i][j][2] = v.z; A[b][i][j][3] = v.w;
            }
            xs[b][i] = ok ? (float)__ldg(a.xsum + (size_t)b * nb + g) : 0.0f;
        }

    for (int k = 0; k < my_tiles; k++) {
        const int t = blockIdx.x + k * gridDim.x;
        const int row0 = t * TR, rows = min(TR, a.N - row0);
        const unsigned char* st = stages + (size_t)(k % a.NST) * a.stage_bytes;
        float2* pk = park + (size_t)(k & 1) * park_pairs;
        const bool ok = mbar_wait(bars + (k % a.NST), (uint32_t)((k / a.NST) & 1));
        if (__syncthreads_or(!ok)) {
            // the copies did not land within the bound: record it, then give the
            // tiles still requested (k + 1 .. k + NST - 1) a bounded wait each so no
            // copy is in flight when the CTA's shared memory is released
            if (tid == 0) {
                atomicExch(a.err, T2_ERR_WAIT);
                for (int kk = k + 1; kk < min(my_tiles, k + a.NST); kk++)
                    mbar_wait(bars + (kk % a.NST), (uint32_t)((kk / a.NST) & 1));
            }
            break;
        }
        const float* sc = reinterpret_cast<const float*>(st + (size_t)TR * cb);
        const bool sbulk = (((uint32_t)rows * nb * 4) & 15u) == 0;
        // items: rows of this warp x groups of this lane
        for (int q = 0; q < RW; q++) {
            const int r = wid * RW + q;
            if (r >= rows) break;
#pragma unroll
            for (int i = 0; i < NBL; i++) {
                const int g = lane + 32 * i;
                if (g >= nb) break;
                const uint4 cw = *reinterpret_cast<const uint4*>(st + (size_t)r * cb + g * 16);
                const float s = sbulk ? sc[r * nb + g] : __ldg(a.scales + (size_t)(row0 + r) * nb + g);
                const uint32_t c[4] = {cw.x, cw.y, cw.z, cw.w};
#pragma unroll
                for (int b = 0; b < B; b++) {
                    int d0 = 0, d1 = 0, d2 = 0, d3 = 0;
#pragma unroll
                    for (int w = 0; w < 4; w++) {
                        d0 = dp4a_us(c[w] & 0x03030303u, A[b][i][0][w], d0);
                        d1 = dp4a_us(c[w] & 0x0C0C0C0Cu, A[b][i][1][w], d1);
                        d2 = dp4a_us(c[w] & 0x30303030u, A[b][i][2][w], d2);
                        d3 = dp4a_us(c[w] & 0xC0C0C0C0u, A[b][i][3][w], d3);
                    }
                    const int dot = d0 + (d1 >> 2) + (d2 >> 4) + (d3 >> 6);   // exact: d_j is a multiple of 4^j
                    pk[((size_t)b * TR + r) * ld + g] = fmul2(make_float2(s, s), make_float2((float)dot, xs[b][i]));
                }
            }
        }
        __syncthreads();                       // the stage is consumed; this tile's pairs are parked
        if (tid == 0 && k + a.NST < my_tiles) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(k + a.NST);
        }
        // this tile's serial chains: warp k % 8, one lane per (activation row, row)
        if (wid == (k & (T2_WARPS - 1)) && lane < B * TR) {
            const int b = lane / TR, r = lane - b * TR;
            if (r < rows) {
                const float2* pr = pk + ((size_t)b * TR + r) * ld;
                float2 acc = make_float2(0.0f, 0.0f);        // (sum s*dot, sum s*xsum)
                int g = 0;
                for (; g + 2 <= nb; g += 2) {
                    const float4 v = *reinterpret_cast<const float4*>(pr + g);
                    acc = fadd2(acc, make_float2(v.x, v.y));
                    acc = fadd2(acc, make_float2(v.z, v.w));
                }
                if (g < nb) acc = fadd2(acc, pr[g]);
                float v = __fsub_rn(acc.x, acc.y);
                if (a.act_scale) v = __fmul_rn(v, __fdiv_rn(1.0f, a.act_scale[b]));
                a.out[(size_t)b * a.N + row0 + r] = v;
            }
        }
    }
}

// Tile rows, stages and shared memory of the streaming form for this shape, or
// false when it does not apply (the activations would not fit in registers).
struct T2Plan {
    int TR, NST, NBL, park_ld, stage_bytes;
    size_t smem;
};
bool tern2_plan(int B, int64_t N, int64_t K, int num_sms, T2Plan* p)
{
    const int nb = (int)(K / 64);
    const int NBL = (nb + 31) / 32;
    if (NBL > 4 || B * NBL > 4) return false;              // <= 64 activation registers a lane
    const int rowb = (int)(K / 4) + nb * 4;                // code + scale bytes a row
    // one chain lane per (activation row, row); enough tiles to give every SM two
    // CTAs' worth when the matrix allows it; large K keeps the stages small
    int TR = 32 / B >= 32 ? 32 : (32 / B >= 16 ? 16 : 8);
    while (TR > 8 && ((N + TR - 1) / TR < 2LL * num_sms || TR * rowb > 32 * 1024)) TR /= 2;
    p->TR = TR;
    p->NBL = NBL;
    p->park_ld = ((nb + 15) & ~15) + 2;                    // float4 rows, 4-bank shift between rows
    p->stage_bytes = (TR * rowb + 127) & ~127;
    const size_t park = 2 * (size_t)B * TR * p->park_ld * 8;
    // shared memory for t2_ctas CTAs an SM (~200 KB), at least 2 and at most 6 stages
    const long long budget = 200LL * 1024 / t2_ctas(B, NBL) - 1024;
    int nst = (int)((budget - 256 - (long long)park) / p->stage_bytes);
    nst = std::max(2, std::min(6, nst));
    p->NST = nst;
    p->smem = 128 + park + 128 + (size_t)nst * p->stage_bytes;
    return p->smem <= 227 * 1024;
}

template <int B, int NBL>
int launch_tern2(tb_ctx* ctx, const Tern2Args& a, const T2Plan& p)
{
    auto kern = k_gemv_tern2<B, NBL>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    int occ = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, T2_THREADS, p.smem);
    if (occ < 1) occ = 1;
    const int grid = std::min(a.tiles, ctx->num_sms * occ);
    e = tb_launch(ctx, kern, dim3(grid), dim3(T2_THREADS), p.smem, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "gemv_tern launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

int tern2_dispatch(tb_ctx* ctx, Tern2Args& a, const T2Plan& p, int B)
{
#define T2_CASE(BB, NN) \
    if (B == BB && p.NBL == NN) return launch_tern2<BB, NN>(ctx, a, p);
    T2_CASE(1, 1) T2_CASE(1, 2) T2_CASE(1, 3) T2_CASE(1, 4)
    T2_CASE(2, 1) T2_CASE(2, 2) T2_CASE(3, 1) T2_CASE(4, 1)
#undef T2_CASE
    return TB_ERR_UNSUPPORTED;
}

size_t tern_smem(int B, int nb)
{
    const int TR = B <= 4 ? 8 : 32 / B;
    return (size_t)B * nb * 64 + (size_t)B * nb * 4 + (size_t)TERN_WARPS * (B + 1) * TR * (nb + 1) * 4;
}

template <int B>
int launch_tern_B(tb_ctx* ctx, const TernArgs& a)
{
    const int nb = a.K >> 6;
    size_t sm = tern_smem(B, nb);
    if (sm > 227 * 1024) return tb_fail(ctx, TB_ERR_UNSUPPORTED, "K=%d batch=%d needs %zu bytes of shared memory", a.K, B, sm);
    if (sm > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_gemv_tern<B>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
        if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    }
    int occ = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k_gemv_tern<B>, TERN_THREADS, sm);
    if (occ < 1) occ = 1;
    int grid = std::min(tb_cdiv(a.tiles, TERN_WARPS), ctx->num_sms * occ);
    cudaError_t e = tb_launch(ctx, k_gemv_tern<B>, dim3(grid), dim3(TERN_THREADS), sm, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "gemv_tern launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

}  // namespace

int tb_gemv_tern_impl(tb_ctx* ctx, float* out, const uint8_t* codes, const float* scales, const int8_t* act,
                      const int32_t* xsum, int64_t N, int64_t K, int batch, const float* act_scale)
{
    TB_REQUIRE(ctx, out && codes && scales && act && xsum, "null pointer");
    TB_REQUIRE(ctx, N > 0 && N < (1LL << 31) && K > 0 && K % 64 == 0 && K <= (1 << 18),
               "bad shape N=%lld K=%lld (K%%64 must be 0)", (long long)N, (long long)K);
    TB_REQUIRE(ctx, TB_ALIGNED(codes, 16) && TB_ALIGNED(act, 16) && TB_ALIGNED(scales, 4) && TB_ALIGNED(xsum, 4),
               "codes/act must be 16-byte aligned");
    T2Plan p2;
    if (batch >= 1 && batch <= 4 && TB_ALIGNED(scales, 16) && tern2_plan(batch, N, K, ctx->num_sms, &p2)) {
        Tern2Args t{out, codes, scales, act, xsum, act_scale, (int)N, (int)K, p2.TR, p2.NST, tb_cdiv(N, p2.TR),
                    p2.stage_bytes, p2.park_ld, ctx->dev_error};
        const int rc = tern2_dispatch(ctx, t, p2, batch);
        if (rc != TB_ERR_UNSUPPORTED) return rc;
    }
    TernArgs a{out, codes, scales, act, xsum, act_scale, (int)N, (int)K, 0};
    const int TR = batch <= 4 ? 8 : 32 / batch;
    a.tiles = tb_cdiv(N, TR);
    switch (batch) {
    case 1: return launch_tern_B<1>(ctx, a);
    case 2: return launch_tern_B<2>(ctx, a);
    case 3: return launch_tern_B<3>(ctx, a);
    case 4: return launch_tern_B<4>(ctx, a);
    case 5: return launch_tern_B<5>(ctx, a);
    case 6: return launch_tern_B<6>(ctx, a);
    case 7: return launch_tern_B<7>(ctx, a);
    case 8: return launch_tern_B<8>(ctx, a);
    }
    return tb_fail(ctx, TB_ERR_INVALID, "batch must be 1..8 (got %d)", batch);
}

int tb_quant_act_impl(tb_ctx* ctx, const float* x, int8_t* act, int32_t* xsum, float* scale, int64_t T, int64_t K,
                      bool wasm)
{
    TB_REQUIRE(ctx, x && act && xsum && scale, "null pointer");
    TB_REQUIRE(ctx, T > 0 && T <= 65535 && K > 0 && K % 64 == 0, "bad shape T=%lld K=%lld", (long long)T, (long long)K);
    cudaError_t e = wasm ? tb_launch(ctx, k_quant_act<true>, dim3((unsigned)T), dim3(256), 0, x, act, xsum, scale, (int)K)
                         : tb_launch(ctx, k_quant_act<false>, dim3((unsigned)T), dim3(256), 0, x, act, xsum, scale,
                                     (int)K);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "quant_act launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

extern "C" {

TB_API int tb_pack_tern_q2g64(tb_ctx* ctx, const float* w, uint8_t* codes, float* scales, int64_t N, int64_t K)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, w && codes && scales, "null pointer");
    TB_REQUIRE(ctx, N > 0 && K > 0 && K % 64 == 0, "bad shape N=%lld K=%lld (K%%64 must be 0)", (long long)N, (long long)K);
    long long ng = N * (K / 64);
    int grid = (int)std::min<long long>((ng * 32 + 255) / 256, (long long)ctx->num_sms * 8);
    cudaError_t e = tb_launch(ctx, k_pack_ternary, dim3(grid), dim3(256), 0, w, codes, scales, ng);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "pack_ternary launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_quant_act_q8(tb_ctx* ctx, const float* x, int8_t* act, int32_t* xsum, float* scale, int64_t T, int64_t K)
{
    if (!ctx) return TB_ERR_INVALID;
    return tb_quant_act_impl(ctx, x, act, xsum, scale, T, K, false);
}

TB_API int tb_quantize_wasm(tb_ctx* ctx, int8_t* dst, int32_t* xsum, const float* x, int64_t k, float* asc,
                            int64_t rows)
{
    if (!ctx) return TB_ERR_INVALID;
    return tb_quant_act_impl(ctx, x, dst, xsum, asc, rows, k, true);
}

TB_API int tb_gemv_tern_q2g64(tb_ctx* ctx, float* out, const uint8_t* codes, const float* scales, const int8_t* act,
                              const int32_t* xsum, int64_t N, int64_t K, int batch)
{
    if (!ctx) return TB_ERR_INVALID;
    return tb_gemv_tern_impl(ctx, out, codes, scales, act, xsum, N, K, batch, nullptr);
}

}  // extern "C"
