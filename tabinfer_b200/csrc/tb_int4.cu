// tb_int4.cu -- int4 G=32 weight path: quant-on-arrival, per-32 int8 activation
// quantizers, and the HBM-bound decode GEMVs (int8-activation DP4A and
// f32-activation forms, 1..8 activation rows, fused gate+up+SiLU, and several
// matrices sharing one activation in a single launch).
//
// Layout (identical to models/qwen3.js:263-270, so packs made by the reference's
// loader or its quant cache are read unchanged): pack u32 [N][K/8], weight k of
// row n in word k/8 at bits 4*(k%8) as q+8; scales f16 [N][K/32].
//
// GEMV design (B200): a scale group is 32 nibbles = 16 bytes = exactly one
// 128-bit load, so each lane owns whole groups.  Eight lanes share a row and
// walk its groups with stride 8 (a warp touches 4 rows x 128 contiguous bytes
// per load), each lane keeping up to 8 independent 16-byte loads in flight.
// Weights do not depend on earlier kernels, so the first chunk is loaded
// BEFORE griddepcontrol.wait: under programmatic dependent launch this
// kernel's weight stream overlaps the tail of the kernel that produces its
// activation.  The activation (a few KB) is staged in shared memory after the
// wait, pre-permuted so that the nibble lanes of a word line up with dp4a
// byte lanes (even k in one word, odd k in the other) and with the per-group
// activation sum folded in: sum (nib-8)*x = dp4a(lo,x_even)+dp4a(hi,x_odd)-8*sum(x).
#include "tb_common.cuh"

namespace {

constexpr int LPR = 8;            // lanes per row
constexpr int RSETS = 32 / LPR;   // row sets per warp
constexpr int CH = 4;             // groups per lane per chunk
constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;

// ---------------------------------------------------------------------------
// quant-on-arrival (bit-exact with quantizeInt4Bf16, models/qwen3.js:3405-3426)
// ---------------------------------------------------------------------------

// models/qwen3.js:3357-3374: f16 bits of an f32, mantissa rounded half-up.
__device__ __forceinline__ uint32_t js_f32_to_f16(float val)
{
    uint32_t x = __float_as_uint(val);
    uint32_t sign = (x >> 16) & 0x8000u, ex = (x >> 23) & 0xffu, mant = x & 0x7fffffu;
    if (ex == 0xffu) return sign | (mant ? 0x7e00u : 0x7c00u);
    int e = (int)ex - 127 + 15;
    if (e >= 31) return sign | 0x7c00u;
    if (e <= 0) {
        if (e < -10) return sign;
        uint32_t m = mant | 0x800000u;
        int shift = 14 - e;
        uint32_t half = (m >> shift) + ((m >> (shift - 1)) & 1u);
        return sign | half;
    }
    return sign | ((((uint32_t)e << 10) | (mant >> 13)) + ((mant >> 12) & 1u));
}

// JavaScript Math.round on a double (ties toward +inf; NaN/Inf unchanged).
__device__ __forceinline__ double js_round(double v)
{
    if (isnan(v) || isinf(v)) return v;
    double f = floor(v);
    return __dsub_rn(v, f) >= 0.5 ? __dadd_rn(f, 1.0) : f;
}

// One thread per (row, 32-group).  The JS runs in doubles, so does this.
__global__ void __launch_bounds__(256) k_quant_int4_g32(const uint16_t* __restrict__ w, uint32_t* __restrict__ pack,
                                                        uint16_t* __restrict__ scales, long long ngroups)
{
    tb_pdl_wait();
    for (long long gi = blockIdx.x * (long long)blockDim.x + threadIdx.x; gi < ngroups;
         gi += (long long)gridDim.x * blockDim.x) {
        const uint4* src = reinterpret_cast<const uint4*>(w + gi * 32);
        uint32_t u[16];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            uint4 v = src[i];
            u[4 * i + 0] = v.x; u[4 * i + 1] = v.y; u[4 * i + 2] = v.z; u[4 * i + 3] = v.w;
        }
        double maxabs = 0.0;
#pragma unroll
        for (int j = 0; j < 32; j++) {
            uint32_t b = (j & 1) ? (u[j >> 1] >> 16) : (u[j >> 1] & 0xffffu);
            double a = fabs((double)__uint_as_float(b << 16));
            if (a > maxabs) maxabs = a;
        }
        double scale = maxabs > 0.0 ? __ddiv_rn(maxabs, 7.0) : 1e-8;
        uint32_t sb = js_f32_to_f16(__double2float_rn(scale));
        double sval = (double)__half2float(__ushort_as_half((unsigned short)sb));
        double inv = __ddiv_rn(1.0, sval);
        uint32_t words[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int j = 0; j < 32; j++) {
            uint32_t b = (j & 1) ? (u[j >> 1] >> 16) : (u[j >> 1] & 0xffffu);
            double q = js_round(__dmul_rn((double)__uint_as_float(b << 16), inv));
            if (q < -8.0) q = -8.0; else if (q > 7.0) q = 7.0;
            uint32_t nib = isnan(q) ? 0u : (uint32_t)((int)q + 8) & 0xfu;
            words[j >> 3] |= nib << (4 * (j & 7));
        }
        reinterpret_cast<uint4*>(pack)[gi] = make_uint4(words[0], words[1], words[2], words[3]);
        scales[gi] = (uint16_t)sb;
    }
}

// ---------------------------------------------------------------------------
// per-32 int8 activation quantization (QUANTQ8 / QUANTQ8T / RMSNORMQ)
// ---------------------------------------------------------------------------

// One warp per (row, 32-group); lane j owns element j.  WGSL f32 semantics:
// scale = maxabs/127, q = clamp(round_half_even(x * (1/scale)), -127, 127).
__device__ __forceinline__ void q8_group_store(float v, int lane, int8_t* xq, float* xs, int32_t* xsum16)
{
    float m = warp_max(fabsf(v));
    float scale = __fdiv_rn(m, 127.0f);
    float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
    int q = __float2int_rn(__fmul_rn(v, inv));
    q = max(-127, min(127, q));
    xq[lane] = (int8_t)q;
    int s = q;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);   // sums within each half-warp
    if (lane == 0) *xs = scale;
    if (xsum16 && (lane & 15) == 0) xsum16[lane >> 4] = s;
}

__global__ void __launch_bounds__(256) k_quant_q8(const float* __restrict__ x, int8_t* __restrict__ xq,
                                                  float* __restrict__ xs, int32_t* __restrict__ xsum16,
                                                  long long ngroups)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    const int lane = threadIdx.x & 31;
    for (long long g = (blockIdx.x * (long long)blockDim.x + threadIdx.x) >> 5; g < ngroups;
         g += ((long long)gridDim.x * blockDim.x) >> 5) {
        float v = x[g * 32 + lane];
        q8_group_store(v, lane, xq + g * 32, xs + g, xsum16 ? xsum16 + 2 * g : nullptr);
    }
}

// RMSNORMQ (qwen3.js:569-612): one CTA per row.  inv = 1/sqrt(mean(x^2)+eps),
// normalized = (x*inv)*w, then the per-32 quantization above.
__global__ void __launch_bounds__(256) k_rmsnorm_q8(const float* __restrict__ x, const uint16_t* __restrict__ w16,
                                                    float eps, int H, int8_t* __restrict__ xq,
                                                    float* __restrict__ xs, int32_t* __restrict__ xsum16)
{
    __shared__ float red[32];
    tb_pdl_wait();
    tb_pdl_trigger();
    const int row = blockIdx.x, lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const float* xr = x + (long long)row * H;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < H; i += blockDim.x) { float v = xr[i]; ss = fmaf(v, v, ss); }
    ss = warp_sum(ss);
    if (lane == 0) red[wid] = ss;
    __syncthreads();
    if (wid == 0) {
        float t = lane < (int)(blockDim.x >> 5) ? red[lane] : 0.0f;
        t = warp_sum(t);
        if (lane == 0) red[0] = t;
    }
    __syncthreads();
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(red[0], (float)H), eps)));
    const int ng = H / 32;
    for (int g = wid; g < ng; g += blockDim.x >> 5) {
        int i = g * 32 + lane;
        float v = __fmul_rn(__fmul_rn(xr[i], inv), tb_h2f(w16[i]));
        q8_group_store(v, lane, xq + (long long)row * H + g * 32, xs + (long long)row * ng + g,
                       xsum16 ? xsum16 + (long long)row * (H / 16) + 2 * g : nullptr);
    }
}

// ---------------------------------------------------------------------------
// decode GEMVs
// ---------------------------------------------------------------------------

struct GemvMat {
    const uint32_t* pack;
    const uint16_t* scales;
    float* y;
    int N;
    int tile_begin;   // first warp tile of this matrix
};
struct GemvArgs {
    GemvMat m[4];
    int count;
    int tiles;        // total warp tiles over all matrices
    int K;
    int acc;
    const void* x;    // int8 [B][K] (Q8) or f32 [B][K] (F32)
    const float* xs;  // [B][K/32] (Q8 only)
};

// Staged int8 activation, per (b, g): lo = (even0,odd0,even1,odd1), hi = (even2,odd2,even3,odd3),
// xs8 = 8*sum(x) over the group, xsf = activation scale.
template <int B>
__device__ __forceinline__ void stage_q8(const GemvArgs& a, int G, uint4* xlo, uint4* xhi, int* xs8, float* xsf)
{
    const int8_t* xq = static_cast<const int8_t*>(a.x);
    for (int i = threadIdx.x; i < B * G; i += blockDim.x) {
        int b = i / G, g = i - b * G;
        const uint4* src = reinterpret_cast<const uint4*>(xq + (long long)b * a.K + g * 32);
        uint4 p = src[0], q = src[1];
        uint32_t w[8] = {p.x, p.y, p.z, p.w, q.x, q.y, q.z, q.w};
        uint32_t e[4], o[4];
        int s = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            e[j] = __byte_perm(w[2 * j], w[2 * j + 1], 0x6420);
            o[j] = __byte_perm(w[2 * j], w[2 * j + 1], 0x7531);
            s = __dp4a((int)w[2 * j], 0x01010101, s);
            s = __dp4a((int)w[2 * j + 1], 0x01010101, s);
        }
        xlo[i] = make_uint4(e[0], o[0], e[1], o[1]);
        xhi[i] = make_uint4(e[2], o[2], e[3], o[3]);
        xs8[i] = 8 * s;
        xsf[i] = a.xs[(long long)b * G + g];
    }
}

// Locate the matrix and first row of a warp tile (rows_per_tile rows each).
__device__ __forceinline__ int tile_matrix(const GemvArgs& a, int tile)
{
    int m = 0;
#pragma unroll
    for (int i = 1; i < 4; i++) if (i < a.count && tile >= a.m[i].tile_begin) m = i;
    return m;
}

// int8-activation GEMV.  GATEUP: matrices 0 (gate) and 1 (up) are walked in
// lock step; the second row slot of a tile is the up row of the same index and
// the output is silu(g)*u into m[0].y.
template <int B, bool GATEUP>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv_int4_q8(const GemvArgs a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int G = a.K >> 5;
    uint4* xlo = reinterpret_cast<uint4*>(smem);
    uint4* xhi = xlo + B * G;
    int* xs8 = reinterpret_cast<int*>(xhi + B * G);
    float* xsf = reinterpret_cast<float*>(xs8 + B * G);

    const int lane = threadIdx.x & 31, rs = lane >> 3, sl = lane & (LPR - 1);
    const int gw = blockIdx.x * GEMV_WARPS + (threadIdx.x >> 5);
    const int nw = gridDim.x * GEMV_WARPS;
    constexpr int RU = 2;                                   // row slots per lane
    constexpr int ROWS_PER_TILE = GATEUP ? RSETS : RSETS * RU;

    // ---- prologue: first chunk of weights for this warp's first tile (before the wait)
    uint4 wv[RU][CH];
    uint16_t sv[RU][CH];
    const uint32_t* rowp[RU];
    const uint16_t* rows_s[RU];
    bool rvalid[RU];
    int row_idx = 0, mi = 0;
    auto setup_tile = [&](int tile) {
        mi = GATEUP ? 0 : tile_matrix(a, tile);
        const GemvMat& M = a.m[mi];
        int local = tile - M.tile_begin;
#pragma unroll
        for (int u = 0; u < RU; u++) {
            const GemvMat& MU = GATEUP ? a.m[u] : M;
            int r = GATEUP ? local * ROWS_PER_TILE + rs : local * ROWS_PER_TILE + u * RSETS + rs;
            if (u == 0) row_idx = r;
            rvalid[u] = r < MU.N;
            int rc = rvalid[u] ? r : 0;
            rowp[u] = MU.pack + (long long)rc * (a.K >> 3);
            rows_s[u] = MU.scales + (long long)rc * G;
        }
    };
    auto load_chunk = [&](int g0) {
#pragma unroll
        for (int c = 0; c < CH; c++) {
            int g = g0 + c * LPR;
#pragma unroll
            for (int u = 0; u < RU; u++) {
                bool ok = rvalid[u] && g < G;
                wv[u][c] = ok ? ldg_stream_v4(rowp[u] + g * 4) : make_uint4(0, 0, 0, 0);
                sv[u][c] = ok ? ldg_u16(rows_s[u] + g) : (uint16_t)0;
            }
        }
    };

    int tile = gw;
    if (tile < a.tiles) { setup_tile(tile); load_chunk(sl); }

    tb_pdl_wait();
    tb_pdl_trigger();
    stage_q8<B>(a, G, xlo, xhi, xs8, xsf);
    __syncthreads();

    for (; tile < a.tiles; tile += nw) {
        if (tile != gw) { setup_tile(tile); load_chunk(sl); }
        float acc[RU][B];
#pragma unroll
        for (int u = 0; u < RU; u++)
#pragma unroll
            for (int b = 0; b < B; b++) acc[u][b] = 0.0f;

        for (int g0 = sl;; g0 += CH * LPR) {
#pragma unroll
            for (int c = 0; c < CH; c++) {
                int g = g0 + c * LPR;
                if (g >= G) break;
#pragma unroll
                for (int b = 0; b < B; b++) {
                    const uint4 xl = xlo[b * G + g], xh = xhi[b * G + g];
                    const int s8 = xs8[b * G + g];
                    const float xsc = xsf[b * G + g];
#pragma unroll
                    for (int u = 0; u < RU; u++) {
                        const uint4 w = wv[u][c];
                        int d = 0;
                        d = __dp4a((int)(w.x & 0x0f0f0f0fu), (int)xl.x, d);
                        d = __dp4a((int)((w.x >> 4) & 0x0f0f0f0fu), (int)xl.y, d);
                        d = __dp4a((int)(w.y & 0x0f0f0f0fu), (int)xl.z, d);
                        d = __dp4a((int)((w.y >> 4) & 0x0f0f0f0fu), (int)xl.w, d);
                        d = __dp4a((int)(w.z & 0x0f0f0f0fu), (int)xh.x, d);
                        d = __dp4a((int)((w.z >> 4) & 0x0f0f0f0fu), (int)xh.y, d);
                        d = __dp4a((int)(w.w & 0x0f0f0f0fu), (int)xh.z, d);
                        d = __dp4a((int)((w.w >> 4) & 0x0f0f0f0fu), (int)xh.w, d);
                        d -= s8;
                        acc[u][b] = fmaf(tb_h2f(sv[u][c]) * xsc, (float)d, acc[u][b]);
                    }
                }
            }
            if (g0 + CH * LPR >= G) break;
            load_chunk(g0 + CH * LPR);
        }
        // reduce the LPR lanes of each row
#pragma unroll
        for (int u = 0; u < RU; u++)
#pragma unroll
            for (int b = 0; b < B; b++) {
                float v = acc[u][b];
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                v += __shfl_xor_sync(0xffffffffu, v, 4);
                acc[u][b] = v;
            }
        if (sl == 0) {
            if (GATEUP) {
                if (rvalid[0]) {
                    const int N = a.m[0].N;
#pragma unroll
                    for (int b = 0; b < B; b++) {
                        float g = acc[0][b], uu = acc[1][b];
                        float silu = __fdiv_rn(g, 1.0f + expf(-g));
                        a.m[0].y[(long long)b * N + row_idx] = silu * uu;
                    }
                }
            } else {
                const GemvMat& M = a.m[mi];
#pragma unroll
                for (int u = 0; u < RU; u++) {
                    if (!rvalid[u]) continue;
                    int r = row_idx + u * RSETS;
#pragma unroll
                    for (int b = 0; b < B; b++) {
                        float* yp = M.y + (long long)b * M.N + r;
                        *yp = (a.acc ? *yp : 0.0f) + acc[u][b];
                    }
                }
            }
        }
    }
}

// f32-activation GEMV (gemvQ math).  x staged per (b, g) as 8 float4, the
// float4 index XOR-swizzled by (g & 7) so the 8 lanes of a row (8 different
// groups) hit 8 different bank quads.
template <int B>
__global__ void __launch_bounds__(GEMV_THREADS) k_gemv_int4_f32(const GemvArgs a)
{
    extern __shared__ __align__(16) unsigned char smem[];
    const int G = a.K >> 5;
    float4* xsm = reinterpret_cast<float4*>(smem);   // [B][G][8]

    const int lane = threadIdx.x & 31, rs = lane >> 3, sl = lane & (LPR - 1);
    const int gw = blockIdx.x * GEMV_WARPS + (threadIdx.x >> 5);
    const int nw = gridDim.x * GEMV_WARPS;
    constexpr int RU = 2;
    constexpr int ROWS_PER_TILE = RSETS * RU;

    uint4 wv[RU][CH];
    uint16_t sv[RU][CH];
    const uint32_t* rowp[RU];
    const uint16_t* rows_s[RU];
    bool rvalid[RU];
    int row_idx = 0, mi = 0;
    auto setup_tile = [&](int tile) {
        mi = tile_matrix(a, tile);
        const GemvMat& M = a.m[mi];
        int local = tile - M.tile_begin;
#pragma unroll
        for (int u = 0; u < RU; u++) {
            int r = local * ROWS_PER_TILE + u * RSETS + rs;
            if (u == 0) row_idx = r;
            rvalid[u] = r < M.N;
            int rc = rvalid[u] ? r : 0;
            rowp[u] = M.pack + (long long)rc * (a.K >> 3);
            rows_s[u] = M.scales + (long long)rc * G;
        }
    };
    auto load_chunk = [&](int g0) {
#pragma unroll
        for (int c = 0; c < CH; c++) {
            int g = g0 + c * LPR;
#pragma unroll
            for (int u = 0; u < RU; u++) {
                bool ok = rvalid[u] && g < G;
                wv[u][c] = ok ? ldg_stream_v4(rowp[u] + g * 4) : make_uint4(0, 0, 0, 0);
                sv[u][c] = ok ? ldg_u16(rows_s[u] + g) : (uint16_t)0;
            }
        }
    };

    int tile = gw;
    if (tile < a.tiles) { setup_tile(tile); load_chunk(sl); }

    tb_pdl_wait();
    tb_pdl_trigger();
    {
        const float4* xg = static_cast<const float4*>(a.x);
        const int per_row = a.K >> 2;
        for (int i = threadIdx.x; i < B * per_row; i += blockDim.x) {
            int b = i / per_row, f = i - b * per_row, g = f >> 3, j = f & 7;
            xsm[(b * G + g) * 8 + (j ^ (g & 7))] = xg[(long long)b * per_row + f];
        }
    }
    __syncthreads();

    for (; tile < a.tiles; tile += nw) {
        if (tile != gw) { setup_tile(tile); load_chunk(sl); }
        float acc[RU][B];
#pragma unroll
        for (int u = 0; u < RU; u++)
#pragma unroll
            for (int b = 0; b < B; b++) acc[u][b] = 0.0f;

        for (int g0 = sl;; g0 += CH * LPR) {
#pragma unroll
            for (int c = 0; c < CH; c++) {
                int g = g0 + c * LPR;
                if (g >= G) break;
                const int sw = g & 7;
#pragma unroll
                for (int b = 0; b < B; b++) {
                    const float4* xr = xsm + (b * G + g) * 8;
                    float d[RU];
#pragma unroll
                    for (int u = 0; u < RU; u++) d[u] = 0.0f;
#pragma unroll
                    for (int wi = 0; wi < 4; wi++) {
                        const float4 xa = xr[(2 * wi) ^ sw], xb = xr[(2 * wi + 1) ^ sw];
#pragma unroll
                        for (int u = 0; u < RU; u++) {
                            const uint32_t w = wi == 0 ? wv[u][c].x : wi == 1 ? wv[u][c].y : wi == 2 ? wv[u][c].z : wv[u][c].w;
                            const uint32_t lo = w & 0x0f0f0f0fu, hi = (w >> 4) & 0x0f0f0f0fu;
                            // 0x4B0000nn is 2^23 + nn exactly; subtracting 2^23 + 8 gives nn - 8.
                            float n0 = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7540)) - 8388616.0f;
                            float n1 = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7540)) - 8388616.0f;
                            float n2 = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7541)) - 8388616.0f;
                            float n3 = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7541)) - 8388616.0f;
                            float n4 = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7542)) - 8388616.0f;
                            float n5 = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7542)) - 8388616.0f;
                            float n6 = __uint_as_float(__byte_perm(lo, 0x4B000000u, 0x7543)) - 8388616.0f;
                            float n7 = __uint_as_float(__byte_perm(hi, 0x4B000000u, 0x7543)) - 8388616.0f;
                            float t = d[u];
                            t = fmaf(n0, xa.x, t); t = fmaf(n1, xa.y, t);
                            t = fmaf(n2, xa.z, t); t = fmaf(n3, xa.w, t);
                            t = fmaf(n4, xb.x, t); t = fmaf(n5, xb.y, t);
                            t = fmaf(n6, xb.z, t); t = fmaf(n7, xb.w, t);
                            d[u] = t;
                        }
                    }
#pragma unroll
                    for (int u = 0; u < RU; u++) acc[u][b] = fmaf(tb_h2f(sv[u][c]), d[u], acc[u][b]);
                }
            }
            if (g0 + CH * LPR >= G) break;
            load_chunk(g0 + CH * LPR);
        }
#pragma unroll
        for (int u = 0; u < RU; u++)
#pragma unroll
            for (int b = 0; b < B; b++) {
                float v = acc[u][b];
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                v += __shfl_xor_sync(0xffffffffu, v, 4);
                acc[u][b] = v;
            }
        if (sl == 0) {
            const GemvMat& M = a.m[mi];
#pragma unroll
            for (int u = 0; u < RU; u++) {
                if (!rvalid[u]) continue;
                int r = row_idx + u * RSETS;
#pragma unroll
                for (int b = 0; b < B; b++) {
                    float* yp = M.y + (long long)b * M.N + r;
                    *yp = (a.acc ? *yp : 0.0f) + acc[u][b];
                }
            }
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

size_t q8_smem(int B, int G) { return (size_t)B * G * (16 + 16 + 4 + 4); }
size_t f32_smem(int B, int G) { return (size_t)B * G * 128; }

template <typename KernT>
int set_smem(tb_ctx* ctx, KernT kern, size_t bytes)
{
    if (bytes > 48 * 1024) {
        if (bytes > 227 * 1024) return tb_fail(ctx, TB_ERR_UNSUPPORTED, "activation staging needs %zu bytes of shared memory", bytes);
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
        if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    }
    return TB_OK;
}

int gemv_grid(tb_ctx* ctx, int tiles)
{
    // two resident CTAs per SM at most, so the next kernel in the stream can
    // start its weight prefetch alongside this one
    int want = tb_cdiv(tiles, GEMV_WARPS);
    int cap = ctx->num_sms * 2;
    return want < cap ? want : cap;
}

template <int B, bool GATEUP>
int launch_q8_B(tb_ctx* ctx, const GemvArgs& a)
{
    const int G = a.K >> 5;
    size_t sm = q8_smem(B, G);
    int rc = set_smem(ctx, k_gemv_int4_q8<B, GATEUP>, sm);
    if (rc) return rc;
    cudaError_t e = tb_launch(ctx, k_gemv_int4_q8<B, GATEUP>, dim3(gemv_grid(ctx, a.tiles)), dim3(GEMV_THREADS), sm, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "gemv_int4_q8 launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

template <bool GATEUP>
int launch_q8(tb_ctx* ctx, const GemvArgs& a, int B)
{
    switch (B) {
    case 1: return launch_q8_B<1, GATEUP>(ctx, a);
    case 2: return launch_q8_B<2, GATEUP>(ctx, a);
    case 3: return launch_q8_B<3, GATEUP>(ctx, a);
    case 4: return launch_q8_B<4, GATEUP>(ctx, a);
    case 5: return launch_q8_B<5, GATEUP>(ctx, a);
    case 6: return launch_q8_B<6, GATEUP>(ctx, a);
    case 7: return launch_q8_B<7, GATEUP>(ctx, a);
    case 8: return launch_q8_B<8, GATEUP>(ctx, a);
    }
    return tb_fail(ctx, TB_ERR_INVALID, "batch must be 1..8 (got %d)", B);
}

template <int B>
int launch_f32_B(tb_ctx* ctx, const GemvArgs& a)
{
    const int G = a.K >> 5;
    size_t sm = f32_smem(B, G);
    int rc = set_smem(ctx, k_gemv_int4_f32<B>, sm);
    if (rc) return rc;
    cudaError_t e = tb_launch(ctx, k_gemv_int4_f32<B>, dim3(gemv_grid(ctx, a.tiles)), dim3(GEMV_THREADS), sm, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "gemv_int4_f32 launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

int launch_f32(tb_ctx* ctx, const GemvArgs& a, int B)
{
    switch (B) {
    case 1: return launch_f32_B<1>(ctx, a);
    case 2: return launch_f32_B<2>(ctx, a);
    case 3: return launch_f32_B<3>(ctx, a);
    case 4: return launch_f32_B<4>(ctx, a);
    case 5: return launch_f32_B<5>(ctx, a);
    case 6: return launch_f32_B<6>(ctx, a);
    case 7: return launch_f32_B<7>(ctx, a);
    case 8: return launch_f32_B<8>(ctx, a);
    }
    return tb_fail(ctx, TB_ERR_INVALID, "batch must be 1..8 (got %d)", B);
}

int check_int4_mat(tb_ctx* ctx, const uint32_t* pack, const uint16_t* scales, int64_t N, int64_t K)
{
    TB_REQUIRE(ctx, pack && scales, "null weight pointer");
    TB_REQUIRE(ctx, N > 0 && N < (1LL << 31), "N out of range (%lld)", (long long)N);
    TB_REQUIRE(ctx, K > 0 && K % 32 == 0 && K <= (1 << 20), "K must be a positive multiple of 32 (got %lld)", (long long)K);
    TB_REQUIRE(ctx, TB_ALIGNED(pack, 16), "pack must be 16-byte aligned");
    TB_REQUIRE(ctx, TB_ALIGNED(scales, 2), "scales must be 2-byte aligned");
    return TB_OK;
}

int fill_mats(tb_ctx* ctx, GemvArgs& a, int count, float* const* ys, const uint32_t* const* packs,
              const uint16_t* const* scales, const int64_t* Ns, int rows_per_tile)
{
    TB_REQUIRE(ctx, count >= 1 && count <= 4, "count must be 1..4");
    int t = 0;
    for (int i = 0; i < count; i++) {
        int rc = check_int4_mat(ctx, packs[i], scales[i], Ns[i], a.K);
        if (rc) return rc;
        TB_REQUIRE(ctx, ys[i] != nullptr, "null output pointer");
        a.m[i] = GemvMat{packs[i], scales[i], ys[i], (int)Ns[i], t};
        t += tb_cdiv(Ns[i], rows_per_tile);
    }
    for (int i = count; i < 4; i++) a.m[i] = GemvMat{nullptr, nullptr, nullptr, 0, 1 << 30};
    a.count = count;
    a.tiles = t;
    return TB_OK;
}

}  // namespace

// Shared with tb_linear.cu
int tb_gemv_q8_impl(tb_ctx* ctx, int count, float* const* ys, const uint32_t* const* packs,
                    const uint16_t* const* scales, const int64_t* Ns, const int8_t* xq, const float* xs,
                    int64_t K, int batch, int acc)
{
    GemvArgs a{};
    a.K = (int)K;
    a.acc = acc ? 1 : 0;
    a.x = xq;
    a.xs = xs;
    TB_REQUIRE(ctx, xq && xs, "null activation pointer");
    TB_REQUIRE(ctx, TB_ALIGNED(xq, 16), "xq must be 16-byte aligned");
    int rc = fill_mats(ctx, a, count, ys, packs, scales, Ns, RSETS * 2);
    if (rc) return rc;
    return launch_q8<false>(ctx, a, batch);
}

int tb_gemv_f32_impl(tb_ctx* ctx, float* y, const float* x, const uint32_t* pack, const uint16_t* scales,
                     int64_t N, int64_t K, int batch, int acc)
{
    GemvArgs a{};
    a.K = (int)K;
    a.acc = acc ? 1 : 0;
    a.x = x;
    a.xs = nullptr;
    TB_REQUIRE(ctx, x && TB_ALIGNED(x, 16), "x must be non-null and 16-byte aligned");
    int rc = fill_mats(ctx, a, 1, &y, &pack, &scales, &N, RSETS * 2);
    if (rc) return rc;
    return launch_f32(ctx, a, batch);
}

int tb_quant_q8_impl(tb_ctx* ctx, const float* x, int8_t* xq, float* xs, int32_t* xsum16, int64_t T, int64_t K)
{
    TB_REQUIRE(ctx, x && xq && xs, "null pointer");
    TB_REQUIRE(ctx, T > 0 && K > 0 && K % 32 == 0, "bad shape T=%lld K=%lld", (long long)T, (long long)K);
    long long ng = T * (K / 32);
    int grid = (int)std::min<long long>((ng * 32 + 255) / 256, (long long)ctx->num_sms * 8);
    cudaError_t e = tb_launch(ctx, k_quant_q8, dim3(grid), dim3(256), 0, x, xq, xs, xsum16, ng);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "quant_q8 launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

extern "C" {

TB_API int tb_quant_int4_g32(tb_ctx* ctx, const uint16_t* w, uint32_t* pack, uint16_t* scales, int64_t N, int64_t K)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, w && pack && scales, "null pointer");
    TB_REQUIRE(ctx, N > 0 && K > 0 && K % 32 == 0, "bad shape N=%lld K=%lld (K%%32 must be 0)", (long long)N, (long long)K);
    TB_REQUIRE(ctx, TB_ALIGNED(w, 16) && TB_ALIGNED(pack, 16) && TB_ALIGNED(scales, 2), "misaligned pointer");
    long long ng = N * (K / 32);
    int grid = (int)std::min<long long>((ng + 255) / 256, (long long)ctx->num_sms * 16);
    cudaError_t e = tb_launch(ctx, k_quant_int4_g32, dim3(grid), dim3(256), 0, w, pack, scales, ng);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "quant_int4 launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_quant_q8(tb_ctx* ctx, const float* x, int8_t* xq, float* xs, int32_t* xsum16, int64_t T, int64_t K)
{
    if (!ctx) return TB_ERR_INVALID;
    return tb_quant_q8_impl(ctx, x, xq, xs, xsum16, T, K);
}

TB_API int tb_rmsnorm_q8(tb_ctx* ctx, const float* x, const uint16_t* w16, float eps, int8_t* xq, float* xs,
                         int32_t* xsum16, int64_t T, int64_t H)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, x && w16 && xq && xs, "null pointer");
    TB_REQUIRE(ctx, T > 0 && T <= 65535 && H > 0 && H % 32 == 0, "bad shape T=%lld H=%lld", (long long)T, (long long)H);
    cudaError_t e = tb_launch(ctx, k_rmsnorm_q8, dim3((unsigned)T), dim3(256), 0, x, w16, eps, (int)H, xq, xs, xsum16);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "rmsnorm_q8 launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_gemv_int4_q8(tb_ctx* ctx, float* y, const int8_t* xq, const float* xs, const uint32_t* pack,
                           const uint16_t* scales, int64_t N, int64_t K, int batch, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    return tb_gemv_q8_impl(ctx, 1, &y, &pack, &scales, &N, xq, xs, K, batch, acc);
}

TB_API int tb_gemv_int4_q8_multi(tb_ctx* ctx, int count, float* const* ys, const uint32_t* const* packs,
                                 const uint16_t* const* scales, const int64_t* Ns, const int8_t* xq,
                                 const float* xs, int64_t K, int batch, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, ys && packs && scales && Ns, "null array");
    return tb_gemv_q8_impl(ctx, count, ys, packs, scales, Ns, xq, xs, K, batch, acc);
}

TB_API int tb_gemv_int4_f32(tb_ctx* ctx, float* y, const float* x, const uint32_t* pack, const uint16_t* scales,
                            int64_t N, int64_t K, int batch, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    return tb_gemv_f32_impl(ctx, y, x, pack, scales, N, K, batch, acc);
}

TB_API int tb_gateup_silu_int4_q8(tb_ctx* ctx, float* swi, const int8_t* xq, const float* xs,
                                  const uint32_t* gpack, const uint16_t* gscales, const uint32_t* upack,
                                  const uint16_t* uscales, int64_t I, int64_t H, int batch)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, xq && xs && swi, "null pointer");
    TB_REQUIRE(ctx, TB_ALIGNED(xq, 16), "xq must be 16-byte aligned");
    GemvArgs a{};
    a.K = (int)H;
    a.acc = 0;
    a.x = xq;
    a.xs = xs;
    float* ys[2] = {swi, swi};
    const uint32_t* packs[2] = {gpack, upack};
    const uint16_t* scs[2] = {gscales, uscales};
    int64_t Ns[2] = {I, I};
    int rc = fill_mats(ctx, a, 2, ys, packs, scs, Ns, RSETS);
    if (rc) return rc;
    a.tiles = a.m[1].tile_begin;   // gate and up are walked together
    return launch_q8<true>(ctx, a, batch);
}

}  // extern "C"
