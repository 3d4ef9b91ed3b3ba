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
#include "tb_common.cuh"

namespace {

constexpr int ATT_WARPS = 4;
constexpr int ATT_THREADS = ATT_WARPS * 32;
constexpr int ATT_MAXG = 8;       // q heads per kv head handled by one CTA
constexpr float NEG_BIG = -3.0e38f;

__device__ __forceinline__ int8_t snorm8(float v)
{
    float c = fminf(1.0f, fmaxf(-1.0f, v));
    return (int8_t)floorf(__fadd_rn(0.5f, __fmul_rn(127.0f, c)));
}

// signed byte i of w as an exact float
__device__ __forceinline__ float sbyte_f(uint32_t w, int i)
{
    uint32_t u = __byte_perm(w ^ 0x80808080u, 0x4B000000u, 0x7540 + i);   // 2^23 + (c+128)
    return __uint_as_float(u) - 8388736.0f;
}

// ---- fused prep: q rope, k rope + quant-write, v quant-write ---------------
// grid = nHq + 2*nKv CTAs, block = hd threads (hd % 32 == 0, hd <= 256).
__global__ void __launch_bounds__(256) k_attn_prep(const float* __restrict__ q, const float* __restrict__ k,
                                                   const float* __restrict__ v, const uint16_t* __restrict__ qw,
                                                   const uint16_t* __restrict__ kw, float* __restrict__ qr,
                                                   int8_t* __restrict__ Kq, float* __restrict__ Ks,
                                                   int8_t* __restrict__ Vq, float* __restrict__ Vs,
                                                   int nHq, int nKv, int hd, long long pos, float theta, float eps)
{
    __shared__ float rk[256];
    __shared__ float red[8];
    tb_pdl_wait();
    tb_pdl_trigger();
    const int j = threadIdx.x, lane = j & 31, wid = j >> 5, nw = hd >> 5;
    const int role = blockIdx.x;
    const bool isQ = role < nHq, isK = !isQ && role < nHq + nKv;
    const int head = isQ ? role : (isK ? role - nHq : role - nHq - nKv);
    const float* src = isQ ? q : (isK ? k : v);
    float x = src[(long long)head * hd + j];
    if (isQ || isK) {
        float ss = warp_sum(x * x);
        if (lane == 0) red[wid] = ss;
        __syncthreads();
        float t = 0.0f;
        for (int i = 0; i < nw; i++) t += red[i];
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)hd), eps)));
        rk[j] = __fmul_rn(__fmul_rn(x, inv), tb_h2f((isQ ? qw : kw)[j]));
        __syncthreads();
        const int half = hd >> 1;
        const int fi = j < half ? j : j - half;
        // angle in double: pos * theta^(-2 fi / hd)
        double ang = (double)pos * pow((double)theta, -2.0 * (double)fi / (double)hd);
        double sd, cd;
        sincos(ang, &sd, &cd);
        const float partner = j < half ? rk[j + half] : rk[j - half];
        const float rot = j < half ? -partner : partner;
        x = fmaf(rk[j], (float)cd, rot * (float)sd);
        if (isQ) { qr[(long long)head * hd + j] = x; return; }
    }
    // quantize one 32-group per warp straight into the cache row `pos`
    const float m = fmaxf(1e-12f, warp_max(fabsf(x)));
    const long long row = pos * nKv * hd + (long long)head * hd;
    int8_t* dq = isK ? Kq : Vq;
    float* ds = isK ? Ks : Vs;
    dq[row + j] = snorm8(__fdiv_rn(x, m));
    if (lane == 0) ds[row / 32 + wid] = m;
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
    int S, nHq, nKv, nsplit, per;
};

// hd fixed at compile time (128 for Qwen3); GRP = q heads per kv head.
template <int HD, int GRP>
__global__ void __launch_bounds__(ATT_THREADS) k_attn_decode(const AttnArgs a)
{
    constexpr int NG = HD / 32;          // scale groups per head row
    constexpr int DPL = HD / 32;         // dims per lane in P.V
    __shared__ __align__(16) float qs[GRP][HD];
    __shared__ float wm[ATT_WARPS][GRP], wl[ATT_WARPS][GRP];
    __shared__ __align__(16) float wo[ATT_WARPS][GRP][HD];

    tb_pdl_wait();
    tb_pdl_trigger();
    const int hk = blockIdx.x, split = blockIdx.y;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int row_elems = a.nKv * HD, row_groups = row_elems / 32;
    const float qscale = rsqrtf((float)HD) * (1.0f / 127.0f);
    for (int i = threadIdx.x; i < GRP * HD; i += ATT_THREADS) {
        int h = i / HD, d = i - h * HD;
        qs[h][d] = a.qr[(long long)(hk * GRP + h) * HD + d];
    }
    __syncthreads();

    const int c0 = split * a.per, c1 = min(a.S, c0 + a.per);
    float m[GRP], l[GRP], o[GRP][DPL];
#pragma unroll
    for (int h = 0; h < GRP; h++) {
        m[h] = NEG_BIG; l[h] = 0.0f;
#pragma unroll
        for (int i = 0; i < DPL; i++) o[h][i] = 0.0f;
    }

    for (int t0 = c0 + wid * 32; t0 < c1; t0 += ATT_WARPS * 32) {
        const int t = t0 + lane;
        const bool valid = t < c1;
        // ---- scores: lane per key
        float s[GRP];
#pragma unroll
        for (int h = 0; h < GRP; h++) s[h] = 0.0f;
        if (valid) {
            const uint4* kr = reinterpret_cast<const uint4*>(a.Kq + (long long)t * row_elems + hk * HD);
            const float* ksr = a.Ks + (long long)t * row_groups + hk * NG;
            uint4 kv[HD / 16];
#pragma unroll
            for (int i = 0; i < HD / 16; i++) kv[i] = __ldg(kr + i);
            float kscale[NG];
#pragma unroll
            for (int g = 0; g < NG; g++) kscale[g] = __ldg(ksr + g);
#pragma unroll
            for (int g = 0; g < NG; g++) {
                float p[GRP];
#pragma unroll
                for (int h = 0; h < GRP; h++) p[h] = 0.0f;
#pragma unroll
                for (int i = 0; i < 2; i++) {
                    const uint4 w4 = kv[g * 2 + i];
                    const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                    for (int wq = 0; wq < 4; wq++)
#pragma unroll
                        for (int bb = 0; bb < 4; bb++) {
                            const float kf = sbyte_f(ww[wq], bb);
                            const int d = g * 32 + i * 16 + wq * 4 + bb;
#pragma unroll
                            for (int h = 0; h < GRP; h++) p[h] = fmaf(qs[h][d], kf, p[h]);
                        }
                }
#pragma unroll
                for (int h = 0; h < GRP; h++) s[h] = fmaf(p[h], kscale[g], s[h]);
            }
        }
        // ---- online softmax update, per q head
        float pr[GRP];
#pragma unroll
        for (int h = 0; h < GRP; h++) {
            const float sc = valid ? s[h] * qscale : NEG_BIG;
            const float mt = warp_max(sc);
            const float mn = fmaxf(m[h], mt);
            const float corr = __expf(m[h] - mn);
            pr[h] = valid ? __expf(sc - mn) : 0.0f;
            l[h] = l[h] * corr + warp_sum(pr[h]);
            m[h] = mn;
#pragma unroll
            for (int i = 0; i < DPL; i++) o[h][i] *= corr;
        }
        // ---- P.V: lane owns dims [lane*DPL, lane*DPL+DPL)
        const int nk = min(32, c1 - t0);
        for (int kk = 0; kk < nk; kk++) {
            const long long tr = (long long)(t0 + kk);
            const int8_t* vrow = a.Vq + tr * row_elems + hk * HD;
            const uint32_t vw = DPL == 4 ? __ldg(reinterpret_cast<const uint32_t*>(vrow) + lane)
                                         : (uint32_t)__ldg(reinterpret_cast<const uint16_t*>(vrow) + lane);
            const float vs = __ldg(a.Vs + tr * row_groups + hk * NG + (lane * DPL) / 32) * (1.0f / 127.0f);
#pragma unroll
            for (int h = 0; h < GRP; h++) {
                const float pw = __shfl_sync(0xffffffffu, pr[h], kk) * vs;
#pragma unroll
                for (int i = 0; i < DPL; i++) o[h][i] = fmaf(pw, sbyte_f(vw, i), o[h][i]);
            }
        }
    }
    // ---- merge warps
#pragma unroll
    for (int h = 0; h < GRP; h++) {
        if (lane == 0) { wm[wid][h] = m[h]; wl[wid][h] = l[h]; }
#pragma unroll
        for (int i = 0; i < DPL; i++) wo[wid][h][lane * DPL + i] = o[h][i];
    }
    __syncthreads();
    for (int i = threadIdx.x; i < GRP * HD; i += ATT_THREADS) {
        const int h = i / HD, d = i - h * HD;
        float M = NEG_BIG;
#pragma unroll
        for (int w = 0; w < ATT_WARPS; w++) M = fmaxf(M, wm[w][h]);
        float L = 0.0f, O = 0.0f;
#pragma unroll
        for (int w = 0; w < ATT_WARPS; w++) {
            const float e = __expf(wm[w][h] - M);
            L = fmaf(wl[w][h], e, L);
            O = fmaf(wo[w][h][d], e, O);
        }
        const long long pidx = (long long)(hk * GRP + h) * a.nsplit + split;
        a.PO[pidx * HD + d] = O;
        if (d == 0) { a.PML[pidx * 2] = M; a.PML[pidx * 2 + 1] = L; }
    }
}

// combine: one CTA per q head, one thread per dim
__global__ void __launch_bounds__(256) k_attn_combine(const float* __restrict__ PO, const float* __restrict__ PML,
                                                      float* __restrict__ out, int nsplit, int hd)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    const int hq = blockIdx.x, d = threadIdx.x;
    const float* pml = PML + (long long)hq * nsplit * 2;
    float M = NEG_BIG;
    for (int i = 0; i < nsplit; i++) M = fmaxf(M, pml[2 * i]);
    float L = 0.0f, O = 0.0f;
    for (int i = 0; i < nsplit; i++) {
        const float e = __expf(pml[2 * i] - M);
        L = fmaf(pml[2 * i + 1], e, L);
        O = fmaf(PO[((long long)hq * nsplit + i) * hd + d], e, O);
    }
    out[(long long)hq * hd + d] = L > 0.0f ? O / L : 0.0f;
}

template <int HD, int GRP>
int launch_decode(tb_ctx* ctx, const AttnArgs& a)
{
    cudaError_t e = tb_launch(ctx, k_attn_decode<HD, GRP>, dim3(a.nKv, a.nsplit), dim3(ATT_THREADS), 0, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "attn_decode launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

}  // namespace

// Split count used when the caller passes nsplit = 0: at least 128 keys per
// CTA, and enough CTAs (nKv * nsplit) for ~4 per SM at long context.
int tb_attn_auto_nsplit(tb_ctx* ctx, int64_t S, int64_t nKv)
{
    long long by_keys = (S + 127) / 128;
    long long by_fill = (4LL * ctx->num_sms + nKv - 1) / nKv;
    long long n = std::min(by_keys, by_fill);
    return (int)std::max(1LL, std::min(n, 1024LL));
}

int tb_attn_decode_impl(tb_ctx* ctx, float* out, const float* qr, const int8_t* Kq, const float* Ks,
                        const int8_t* Vq, const float* Vs, int64_t S, int64_t nHq, int64_t nKv, int64_t hd,
                        int nsplit, float* PO, float* PML)
{
    AttnArgs a{qr, Kq, Ks, Vq, Vs, PO, PML, (int)S, (int)nHq, (int)nKv, nsplit, 0};
    a.per = (int)((S + nsplit - 1) / nsplit);
    const int grp = (int)(nHq / nKv);
    int rc = TB_OK;
    if (hd == 128) {
        switch (grp) {
        case 1: rc = launch_decode<128, 1>(ctx, a); break;
        case 2: rc = launch_decode<128, 2>(ctx, a); break;
        case 4: rc = launch_decode<128, 4>(ctx, a); break;
        case 8: rc = launch_decode<128, 8>(ctx, a); break;
        default: return tb_fail(ctx, TB_ERR_UNSUPPORTED, "nHq/nKv = %d not built (1, 2, 4, 8)", grp);
        }
    } else if (hd == 64) {
        switch (grp) {
        case 1: rc = launch_decode<64, 1>(ctx, a); break;
        case 2: rc = launch_decode<64, 2>(ctx, a); break;
        case 4: rc = launch_decode<64, 4>(ctx, a); break;
        case 8: rc = launch_decode<64, 8>(ctx, a); break;
        default: return tb_fail(ctx, TB_ERR_UNSUPPORTED, "nHq/nKv = %d not built (1, 2, 4, 8)", grp);
        }
    } else {
        return tb_fail(ctx, TB_ERR_UNSUPPORTED, "head_dim %lld not built (64, 128)", (long long)hd);
    }
    if (rc) return rc;
    cudaError_t e = tb_launch(ctx, k_attn_combine, dim3((unsigned)nHq), dim3((unsigned)hd), 0,
                              (const float*)PO, (const float*)PML, out, nsplit, (int)hd);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "attn_combine launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

int tb_attn_check(tb_ctx* ctx, const float* qr, const int8_t* Kq, const float* Ks, const int8_t* Vq, const float* Vs,
                  int64_t S, int64_t nHq, int64_t nKv, int64_t hd, int nsplit)
{
    TB_REQUIRE(ctx, qr && Kq && Ks && Vq && Vs, "null pointer");
    TB_REQUIRE(ctx, S >= 0 && S < (1LL << 31), "bad S");
    TB_REQUIRE(ctx, nKv > 0 && nHq > 0 && nHq % nKv == 0 && nHq / nKv <= ATT_MAXG, "bad head counts nHq=%lld nKv=%lld",
               (long long)nHq, (long long)nKv);
    TB_REQUIRE(ctx, hd == 64 || hd == 128, "head_dim must be 64 or 128 (got %lld)", (long long)hd);
    TB_REQUIRE(ctx, TB_ALIGNED(Kq, 16) && TB_ALIGNED(Vq, 16) && TB_ALIGNED(Ks, 16), "KV cache must be 16-byte aligned");
    TB_REQUIRE(ctx, nsplit >= 0 && nsplit <= 1024, "nsplit must be 0..1024");
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
                              kw16, qr, Kq, Ks, Vq, Vs, (int)nHq, (int)nKv, (int)hd, (long long)pos, theta, eps);
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
    TB_REQUIRE(ctx, out != nullptr, "null output");
    if (nsplit == 0) nsplit = tb_attn_auto_nsplit(ctx, S, nKv);
    size_t po = (size_t)nHq * nsplit * hd * sizeof(float), pml = (size_t)nHq * nsplit * 2 * sizeof(float);
    float* scr = static_cast<float*>(tb_ctx_scratch(ctx, po + pml));
    if (!scr) return TB_ERR_NOMEM;
    return tb_attn_decode_impl(ctx, out, qr, Kq, Ks, Vq, Vs, S, nHq, nKv, hd, nsplit, scr, scr + po / sizeof(float));
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
//    reads it), but calls that overlap on the GPU (other streams, other contexts
//    on the same device) race on it: order them.
constexpr size_t NOALLOC_SCRATCH_FLOATS = size_t(1) << 18;
static __device__ __align__(256) float g_attn_noalloc_scratch[NOALLOC_SCRATCH_FLOATS];

#include <mutex>

namespace {
constexpr int NOALLOC_MAX_DEVICES = 64;
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[NOALLOC_MAX_DEVICES] = {};

// Device address of the array on ctx's device (host code may not use the
// symbol itself as an address).
int noalloc_scratch(tb_ctx* ctx, float** out)
{
    TB_REQUIRE(ctx, ctx->device >= 0 && ctx->device < NOALLOC_MAX_DEVICES, "device index out of range");
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[ctx->device]) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaError_t e = cudaSetDevice(ctx->device);
        void* p = nullptr;
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&p, g_attn_noalloc_scratch);
        cudaSetDevice(prev);
        if (e != cudaSuccess || !p)
            return tb_fail(ctx, TB_ERR_CUDA, "cudaGetSymbolAddress(attention scratch): %s", cudaGetErrorString(e));
        g_noalloc_ptr[ctx->device] = static_cast<float*>(p);
    }
    *out = g_noalloc_ptr[ctx->device];
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
    TB_REQUIRE(ctx, out != nullptr, "null output");
    if (nsplit == 0) nsplit = tb_attn_auto_nsplit(ctx, S, nKv);
    const size_t need = (size_t)nHq * nsplit * (hd + 2);
    if (need > NOALLOC_SCRATCH_FLOATS)
        return tb_fail(ctx, TB_ERR_INVALID,
                       "attn_decode_q8_noalloc: nHq*nsplit*(hd+2) = %zu floats exceeds the fixed scratch of %zu floats "
                       "(use fewer splits or tb_attn_decode_q8)", need, NOALLOC_SCRATCH_FLOATS);
    float* scr = nullptr;
    rc = noalloc_scratch(ctx, &scr);
    if (rc) return rc;
    return tb_attn_decode_impl(ctx, out, qr, Kq, Ks, Vq, Vs, S, nHq, nKv, hd, nsplit, scr,
                               scr + (size_t)nHq * nsplit * hd);
}
