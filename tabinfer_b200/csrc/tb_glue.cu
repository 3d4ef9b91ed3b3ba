// tb_glue.cu -- decode-step glue: argmax, RMSNorm, embedding gather, and the
// sampling transforms that precede argmax: the grammar logit mask and
// Gumbel-max temperature noise (models/qwen3.js:2692-2737), standalone and
// fused into argmax's first pass (so a sampled step reads the logits once and
// leaves them unmodified).
#include "tb_act.cuh"
#include "tb_internal.h"

namespace {

constexpr int AMAX_THREADS = 256;

// Orderable key: larger value wins, then the LOWER index (ties), NaN never wins
// (the reference's `if (v > bv)` skips NaN).
__device__ __forceinline__ unsigned long long amax_key(float v, unsigned idx)
{
    if (isnan(v)) v = -INFINITY;
    uint32_t f = __float_as_uint(v);
    uint32_t o = (f & 0x80000000u) ? ~f : (f | 0x80000000u);
    return ((unsigned long long)o << 32) | (0xffffffffu - idx);
}

__device__ __forceinline__ unsigned long long block_max_key(unsigned long long k)
{
    __shared__ unsigned long long sk[32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        unsigned long long p = __shfl_xor_sync(0xffffffffu, k, o);
        k = p > k ? p : k;
    }
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (lane == 0) sk[wid] = k;
    __syncthreads();
    if (wid == 0) {
        k = lane < (int)(blockDim.x >> 5) ? sk[lane] : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            unsigned long long p = __shfl_xor_sync(0xffffffffu, k, o);
            k = p > k ? p : k;
        }
    }
    return k;   // valid in thread 0
}

// GUMBEL_WGSL's hash (qwen3.js:2724): a PCG output permutation of one word
__device__ __forceinline__ uint32_t pcg_hash(uint32_t v0)
{
    const uint32_t v = v0 * 747796405u + 2891336453u;
    const uint32_t w = ((v >> ((v >> 28u) + 4u)) ^ v) * 277803737u;
    return (w >> 22u) ^ w;
}
// T * Gumbel(0,1) noise of flat logit index i under `seed` (qwen3.js:2726-2730):
// u = (h >> 8 + 0.5) / 2^24 lies in (0, 1) and is exact in f32
__device__ __forceinline__ float gumbel_noise(uint32_t i, uint32_t seed, float temp)
{
    const uint32_t h = pcg_hash(i ^ (seed * 2654435761u));
    const float u = ((float)(h >> 8) + 0.5f) / 16777216.0f;
    return temp * (-logf(-logf(u)));
}
// LOGITMASK_WGSL (qwen3.js:2696-2704): a token whose bit is clear gets -3e38
constexpr float MASKED = -3.0e38f;

struct SampleXf {
    const uint32_t* mask;   // [rows][ceil(n/32)] bit per token, or nullptr
    uint32_t seed;
    float temp;             // 0: no noise
};

// stage 1: blocks (bx, row) reduce an interleaved slice of row `row`; with XF the
// logit is first masked and given its Gumbel noise (the transforms above, on the
// flat index row * n + i)
template <bool XF>
__global__ void __launch_bounds__(AMAX_THREADS) k_argmax_p1(const float* __restrict__ x, long long n,
                                                            unsigned long long* __restrict__ part, SampleXf xf)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    const int row = blockIdx.y;
    const float* xr = x + (long long)row * n;
    const long long mw = (n + 31) >> 5;
    unsigned long long best = 0ull;
    for (long long i = blockIdx.x * (long long)AMAX_THREADS + threadIdx.x; i < n;
         i += (long long)gridDim.x * AMAX_THREADS) {
        float v = xr[i];
        if (XF) {
            if (xf.mask && ((xf.mask[row * mw + (i >> 5)] >> (i & 31)) & 1u) == 0u) v = MASKED;
            if (xf.temp != 0.0f) v = v + gumbel_noise((uint32_t)(row * n + i), xf.seed, xf.temp);
        }
        unsigned long long k = amax_key(v, (unsigned)i);
        best = k > best ? k : best;
    }
    best = block_max_key(best);
    if (threadIdx.x == 0) part[(long long)row * gridDim.x + blockIdx.x] = best;
}

__global__ void __launch_bounds__(256) k_logit_mask(float* __restrict__ logits, const uint32_t* __restrict__ mask,
                                                    long long n, long long total)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    const long long mw = (n + 31) >> 5;
    for (long long f = blockIdx.x * 256ll + threadIdx.x; f < total; f += (long long)gridDim.x * 256) {
        const long long row = f / n, i = f - row * n;
        if (((mask[row * mw + (i >> 5)] >> (i & 31)) & 1u) == 0u) logits[f] = MASKED;
    }
}

__global__ void __launch_bounds__(256) k_gumbel(float* __restrict__ logits, long long total, uint32_t seed, float temp)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    for (long long f = blockIdx.x * 256ll + threadIdx.x; f < total; f += (long long)gridDim.x * 256)
        logits[f] = logits[f] + gumbel_noise((uint32_t)f, seed, temp);
}

// stage 2: one block per row.  Writes the row's index (out, + idx_base: the
// first global row of this vocab shard) and/or its ordered key (out_key, for a
// cross-shard merge), and advances the row's position (pos_inc) when given.
__global__ void __launch_bounds__(AMAX_THREADS) k_argmax_p2(const unsigned long long* __restrict__ part, int nparts,
                                                            uint32_t* __restrict__ out, unsigned long long* out_key,
                                                            unsigned idx_base, int* pos_inc)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    const int row = blockIdx.x;
    unsigned long long best = 0ull;
    for (int i = threadIdx.x; i < nparts; i += AMAX_THREADS) {
        unsigned long long k = part[(long long)row * nparts + i];
        best = k > best ? k : best;
    }
    best = block_max_key(best);
    if (threadIdx.x == 0) {
        const uint32_t idx = 0xffffffffu - (uint32_t)(best & 0xffffffffu) + idx_base;
        if (out) out[row] = idx;
        if (out_key) out_key[row] = (best & 0xffffffff00000000ull) | (0xffffffffu - idx);
        if (pos_inc) pos_inc[row] += 1;
    }
}

// merge of per-shard keys [nshard][rows]: the largest key wins (value, then the
// lower global index), as a single argmax over the whole vocabulary would.
__global__ void k_argmax_merge(const unsigned long long* __restrict__ keys, int nshard, int rows,
                               uint32_t* __restrict__ out, int* pos_inc)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= rows) return;
    unsigned long long best = 0ull;
    for (int s = 0; s < nshard; s++) {
        const unsigned long long k = keys[(long long)s * rows + row];
        best = k > best ? k : best;
    }
    out[row] = 0xffffffffu - (uint32_t)(best & 0xffffffffu);
    if (pos_inc) pos_inc[row] += 1;
}

// RMSNorm, qwen3.js:60-88: one 256-thread CTA per row (the reduction the
// fused lm_head prologue uses too, tb_act.cuh).
__global__ void __launch_bounds__(256) k_rmsnorm(const float* __restrict__ x, const uint16_t* __restrict__ w16,
                                                 float* __restrict__ y, int H, float eps)
{
    __shared__ float red[80];
    tb_pdl_wait();
    tb_pdl_trigger();
    const int row = blockIdx.x;
    const float* xr = x + (long long)row * H;
    const float inv = rms_inv(block256_sumsq(xr, H, red), H, eps);
    for (int i = threadIdx.x; i < H; i += blockDim.x)
        y[(long long)row * H + i] = __fmul_rn(__fmul_rn(xr[i], inv), tb_h2f(w16[i]));
}

// embedGather, qwen3.js:1621-1675: y[t,h] = f32(embed[ids[idoff+t], h])
__global__ void __launch_bounds__(256) k_embed(const uint32_t* __restrict__ ids, long long idoff,
                                               const uint16_t* __restrict__ emb, float* __restrict__ y, int T, int H)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)T * H;
         i += (long long)gridDim.x * blockDim.x) {
        const int t = (int)(i / H), h = (int)(i - (long long)t * H);
        y[i] = tb_h2f(emb[(long long)ids[idoff + t] * H + h]);
    }
}

}  // namespace

int tb_argmax_impl(tb_ctx* ctx, const float* x, int64_t n, int64_t rows, uint32_t* out, unsigned long long* part,
                   int nparts, unsigned long long* out_key, uint32_t idx_base, int32_t* pos_inc)
{
    cudaError_t e = tb_launch(ctx, k_argmax_p1<false>, dim3(nparts, (unsigned)rows), dim3(AMAX_THREADS), 0, x,
                              (long long)n, part, SampleXf{nullptr, 0u, 0.0f});
    if (e == cudaSuccess)
        e = tb_launch(ctx, k_argmax_p2, dim3((unsigned)rows), dim3(AMAX_THREADS), 0,
                      (const unsigned long long*)part, nparts, out, out_key, (unsigned)idx_base, (int*)pos_inc);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "argmax launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

int tb_argmax_merge_impl(tb_ctx* ctx, const unsigned long long* keys, int nshard, int rows, uint32_t* out,
                         int32_t* pos_inc)
{
    cudaError_t e = tb_launch(ctx, k_argmax_merge, dim3((unsigned)((rows + 127) / 128)), dim3(128), 0, keys, nshard,
                              rows, out, (int*)pos_inc);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "argmax merge launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

int tb_argmax_parts(tb_ctx* ctx, int64_t n)
{
    long long want = (n + AMAX_THREADS * 8 - 1) / (AMAX_THREADS * 8);
    return (int)std::max(1LL, std::min(want, (long long)ctx->num_sms));
}

extern "C" {

TB_API int tb_argmax(tb_ctx* ctx, const float* x, int64_t n, int64_t rows, uint32_t* out_idx, int64_t out_offset)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, x && out_idx, "null pointer");
    TB_REQUIRE(ctx, n > 0 && n < (1LL << 32) - 1 && rows > 0 && rows <= 65535 && out_offset >= 0, "bad shape");
    int nparts = tb_argmax_parts(ctx, n);
    auto* part = static_cast<unsigned long long*>(tb_ctx_scratch(ctx, (size_t)rows * nparts * 8));
    if (!part) return TB_ERR_NOMEM;
    return tb_argmax_impl(ctx, x, n, rows, out_idx + out_offset, part, nparts, nullptr, 0, nullptr);
}

TB_API int tb_logit_mask(tb_ctx* ctx, float* logits, const uint32_t* mask, int64_t n, int64_t rows)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, logits && mask, "null pointer");
    TB_REQUIRE(ctx, n > 0 && rows > 0 && n * rows < (1LL << 40), "bad shape");
    const long long tot = n * rows;
    int grid = (int)std::min<long long>((tot + 255) / 256, (long long)ctx->num_sms * 8);
    cudaError_t e = tb_launch(ctx, k_logit_mask, dim3(grid), dim3(256), 0, logits, mask, (long long)n, tot);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "logit_mask launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_gumbel_noise(tb_ctx* ctx, float* logits, int64_t n, int64_t rows, uint32_t seed, float temp)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, logits != nullptr, "null pointer");
    TB_REQUIRE(ctx, n > 0 && rows > 0 && n * rows <= (1LL << 32), "bad shape (flat indices are 32-bit)");
    const long long tot = n * rows;
    int grid = (int)std::min<long long>((tot + 255) / 256, (long long)ctx->num_sms * 8);
    cudaError_t e = tb_launch(ctx, k_gumbel, dim3(grid), dim3(256), 0, logits, tot, seed, temp);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "gumbel launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_sample_argmax(tb_ctx* ctx, const float* logits, int64_t n, int64_t rows, const uint32_t* mask,
                            uint32_t seed, float temp, uint32_t* out_idx)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, logits && out_idx, "null pointer");
    TB_REQUIRE(ctx, n > 0 && n < (1LL << 32) - 1 && rows > 0 && rows <= 65535 && n * rows <= (1LL << 32),
               "bad shape");
    TB_REQUIRE(ctx, temp >= 0.0f, "temperature must be >= 0");
    const int nparts = tb_argmax_parts(ctx, n);
    auto* part = static_cast<unsigned long long*>(tb_ctx_scratch(ctx, (size_t)rows * nparts * 8));
    if (!part) return TB_ERR_NOMEM;
    cudaError_t e = tb_launch(ctx, k_argmax_p1<true>, dim3(nparts, (unsigned)rows), dim3(AMAX_THREADS), 0, logits,
                              (long long)n, part, SampleXf{mask, seed, temp});
    if (e == cudaSuccess)
        e = tb_launch(ctx, k_argmax_p2, dim3((unsigned)rows), dim3(AMAX_THREADS), 0, (const unsigned long long*)part,
                      nparts, out_idx, (unsigned long long*)nullptr, 0u, (int*)nullptr);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "sample_argmax launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_rmsnorm(tb_ctx* ctx, const float* x, const uint16_t* w16, float* y, int64_t T, int64_t H, float eps)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, x && w16 && y, "null pointer");
    TB_REQUIRE(ctx, T > 0 && T <= 65535 && H > 0 && H % 4 == 0, "bad shape (H %% 4 must be 0)");
    TB_REQUIRE(ctx, TB_ALIGNED(x, 16), "x must be 16-byte aligned");
    cudaError_t e = tb_launch(ctx, k_rmsnorm, dim3((unsigned)T), dim3(256), 0, x, w16, y, (int)H, eps);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "rmsnorm launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_embed_gather(tb_ctx* ctx, const uint32_t* ids, int64_t idoff, const uint16_t* emb, float* y, int64_t T,
                           int64_t H)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, ids && emb && y, "null pointer");
    TB_REQUIRE(ctx, T > 0 && H > 0 && idoff >= 0, "bad shape");
    long long tot = T * H;
    int grid = (int)std::min<long long>((tot + 255) / 256, (long long)ctx->num_sms * 8);
    cudaError_t e = tb_launch(ctx, k_embed, dim3(grid), dim3(256), 0, ids, (long long)idoff, emb, y, (int)T, (int)H);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "embed launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

}  // extern "C"
