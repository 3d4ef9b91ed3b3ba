// tb_gemv.cu -- HBM-bound int4 G=32 decode GEMVs for 1..8 activation rows.
//
// Weight layout is the reference's (models/qwen3.js:263-270): pack u32 [N][K/8],
// weight k of row n at bits 4*(k%8) of word k/8 as q+8; f16 scales [N][K/32].
//
// B200 design
//  * Work unit = a row block of RB consecutive rows.  Its packed weights
//    (RB*K/2 bytes) and scales (RB*K/16 bytes) are each ONE contiguous range,
//    moved into shared memory by a TMA bulk copy (cp.async.bulk, completion on
//    an mbarrier).  Small matrices get one row block per CTA and ~1-2 CTAs per
//    SM, so every SM streams; large ones (lm_head) pipeline NST stages per CTA.
//  * The first stages are requested BEFORE griddepcontrol.wait: with
//    programmatic dependent launch the weight stream of this kernel overlaps
//    the tail of the kernel producing its activation.
//  * The activation (a few KB) is prepared after the wait, per CTA, straight
//    from the producer's f32 output: optional RMSNorm, then the per-32 int8
//    quantization of QUANTQ8, with code shared with the standalone kernels so
//    the int8 values are bit-identical.  It is stored pre-permuted so the
//    nibble lanes of a weight word meet dp4a byte lanes directly:
//       sum (nib-8)*x = dp4a(w & 0x0f0f0f0f, x_even) + dp4a((w>>4) & 0x0f0f0f0f, x_odd) - 8*sum(x).
//  * f32-activation rows (gemvQ) convert nibbles with a byte permute into the
//    float 2^23+nib and use Blackwell's packed fma.rn.f32x2.
//  * A warp owns a row of the staged block, its lanes the row's 16-byte groups
//    (conflict-free shared-memory reads), reduced with a shuffle tree; lane 0
//    writes (optionally += y, the fused residual; or silu(g)*u for gate/up).
//  * Ternary weights in the WebGPU layout (models/qwen3.js:3427-3469: 16 2-bit
//    codes w+1 per u32, weight k = 16w+4s+b at bits 8b+2s, f16 scales [N][K/32])
//    stream through the same row blocks at 8 bytes per 32-group.  Their int8
//    activation is staged in natural k order, so (word >> 2s) & 0x03030303 meets
//    x[16w+4s .. 16w+4s+3] in dp4a byte lanes, and (c-1)*x = c*x - x turns the
//    sign decode into one subtraction of the group's sum of x (gemvTern2Wgsl,
//    qwen3.js:449-503; gateupTern2Wgsl, qwen3.js:747-810).
#include "tb_gemv_dev.cuh"

namespace {

// ---- the kernel -----------------------------------------------------------------
// Consumer mapping: warp w takes rows w, w+8, ... of the staged row block; lane l
// takes groups l, l+32, ... of the row (consecutive 16-byte items: conflict-free
// shared-memory reads); the 32 partial sums of a row meet in a shuffle tree.
template <int B, int KIND>
__global__ void __launch_bounds__(THREADS, 2) k_gemv(const Args a)
{
    extern __shared__ __align__(128) unsigned char smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    float* red = reinterpret_cast<float*>(smem + 64);
    __shared__ int abort_flag;
    unsigned char* act = smem + SMEM_HDR;
    float* xbuf = reinterpret_cast<float*>(act + a.act_bytes);
    uint16_t* nws = reinterpret_cast<uint16_t*>(act + a.act_bytes + a.xbuf_bytes);
    unsigned char* stages = act + a.act_bytes + a.xbuf_bytes + a.nw_bytes;
    constexpr bool gateup = kind_gateup(KIND);
    constexpr bool TERN = kind_tern(KIND);
    constexpr int NM = gateup ? 2 : 1;
    const int stage_bytes = NM * a.slot_bytes;
    const int G = a.K >> 5;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;

    // ---- prologue (independent of earlier kernels): norm weights, barriers and
    // the first weight stages
    if (a.act_src == ACT_RMSNORM) {
        for (int i = tid; i < (a.K >> 3); i += THREADS)
            reinterpret_cast<uint4*>(nws)[i] = __ldg(reinterpret_cast<const uint4*>(a.normw) + i);
    }
    if (tid == 0) {
        abort_flag = 0;
        for (int s = 0; s < a.nst; s++) mbar_init(&bars[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        for (int j = 0; j < a.nst; j++) {
            const int rb = blockIdx.x + j * gridDim.x;
            if (rb >= a.nrb) break;
            issue_block(a, rb, stages + j * stage_bytes, &bars[j], gateup);
        }
    }
    __syncthreads();

    // ---- wait for the producer of the activation, then prepare it
    tb_pdl_wait();
    tb_pdl_trigger();
    if (KIND == KIND_F32) stage_f32<B>(a, act, red, nws);
    else if (KIND == KIND_F32D) stage_f32d(a, act, xbuf, red, nws);
    else stage_q8<B, TERN>(a, act, xbuf, a.xbuf_bytes >> 2, red, nws);
    __syncthreads();

    constexpr bool DREG = KIND == KIND_F32D;   // the digit form of one f32 row

    // f32 activation of a single row kept in registers (groups lane, lane+32),
    // un-swizzled on the way in so every register index is static
    constexpr bool XREG = KIND == KIND_F32 && B == 1;
    const bool xreg = XREG && G <= 64;
    float4 xr0[8], xr1[8];
    if (XREG && xreg) {
        const float4* xsm = reinterpret_cast<const float4*>(act);
        if (lane < G) {
#pragma unroll
            for (int j = 0; j < 8; j++) xr0[j] = xsm[lane * 8 + (j ^ (lane & 7))];
        }
        if (lane + 32 < G) {
#pragma unroll
            for (int j = 0; j < 8; j++) xr1[j] = xsm[(lane + 32) * 8 + (j ^ (lane & 7))];
        }
    }

    for (int j = 0;; j++) {
        const int rb = blockIdx.x + j * gridDim.x;
        if (rb >= a.nrb) break;
        const int st = j % a.nst;
        const Block bl = block_of(a, rb, gateup);
        if (!mbar_wait(&bars[st], (uint32_t)((j / a.nst) & 1))) {
            abort_flag = 1;
            if (a.err) atomicExch(a.err, ERR_WAIT_TIMEOUT);
        }
        const unsigned char* stg = stages + st * stage_bytes;
        if (!scales_bulk(bl.nrows, G) && !abort_flag) {
            // a tail block whose scales are not a whole number of 16-byte chunks:
            // copy them into the slot with plain loads, so every scale read below
            // is a shared-memory read
            for (int s = 0; s < NM; s++) {
                uint16_t* dst = reinterpret_cast<uint16_t*>(stages + st * stage_bytes + s * a.slot_bytes +
                                                            (size_t)a.RB * a.wrow_bytes);
                const uint16_t* src = a.m[gateup ? s : bl.mi].scales + (size_t)bl.row0 * G;
                for (int i = tid; i < bl.nrows * G; i += THREADS) dst[i] = src[i];
            }
            // these generic-proxy writes precede a later bulk copy into the same slot
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncthreads();
        }
        if (!abort_flag) {
            // a warp carries RPW rows at once (rows r0, r0 + 8, ...): independent dp4a /
            // FMA chains and shuffle trees that overlap, and one activation load per
            // group for all of them, instead of one row's latency chain
            constexpr int RPW = B == 1 ? 4 : (B == 2 ? 2 : 1);
            constexpr int NW = THREADS / 32;
            for (int r0 = wid; r0 < bl.nrows; r0 += NW * RPW) {
                float acc[RPW][NM][B];
#pragma unroll
                for (int q = 0; q < RPW; q++)
#pragma unroll
                    for (int s = 0; s < NM; s++)
#pragma unroll
                        for (int b = 0; b < B; b++) acc[q][s][b] = 0.0f;
#pragma unroll
                for (int s = 0; s < NM; s++) {
                    const unsigned char* slot = stg + s * a.slot_bytes;
                    const uint16_t* sbase = reinterpret_cast<const uint16_t*>(slot + (size_t)a.RB * a.wrow_bytes);
                    if (TERN) {
                        const uint2* tw = reinterpret_cast<const uint2*>(slot);
                        for (int g = lane; g < G; g += 32) {
                            if constexpr (RPW > 1) {
                                XQ<B> xg;
                                load_xq<B>(xg, act, G, g);
#pragma unroll
                                for (int q = 0; q < RPW; q++) {
                                    const int r = r0 + q * NW;
                                    if (r < bl.nrows) item_ternx<B>(tw[r * G + g], tb_h2f(sbase[r * G + g]), xg, acc[q][s]);
                                }
                            } else {
                                item_tern<B>(tw[r0 * G + g], tb_h2f(sbase[r0 * G + g]), act, G, g, acc[0][s]);
                            }
                        }
                    } else if (DREG) {
                        const uint4* wq = reinterpret_cast<const uint4*>(slot);
                        // a group's digits are read once for the warp's RPW rows
                        for (int g = lane; g < G; g += 32) {
                            XD xg;
                            load_xd(xg, act, G, g);
#pragma unroll
                            for (int q = 0; q < RPW; q++) {
                                const int r = r0 + q * NW;
                                if (r < bl.nrows)
                                    item_f32d(wq[r * G + g], tb_h2f(sbase[r * G + g]), xg, &acc[q][s][0]);
                            }
                        }
                    } else if (XREG && xreg) {
#pragma unroll
                        for (int q = 0; q < RPW; q++) {
                            const int r = r0 + q * NW;
                            if (r >= bl.nrows) continue;
                            const uint4* wrow = reinterpret_cast<const uint4*>(slot) + (size_t)r * G;
                            const uint16_t* srow = sbase + (size_t)r * G;
                            if (lane < G) {
                                const uint4 w = wrow[lane];
                                float2 d = make_float2(0.0f, 0.0f);
                                d = word_f32(w.x, xr0[0], xr0[1], d);
                                d = word_f32(w.y, xr0[2], xr0[3], d);
                                d = word_f32(w.z, xr0[4], xr0[5], d);
                                d = word_f32(w.w, xr0[6], xr0[7], d);
                                acc[q][s][0] = fmaf(tb_h2f(srow[lane]), d.x + d.y, acc[q][s][0]);
                            }
                            if (lane + 32 < G) {
                                const uint4 w = wrow[lane + 32];
                                float2 d = make_float2(0.0f, 0.0f);
                                d = word_f32(w.x, xr1[0], xr1[1], d);
                                d = word_f32(w.y, xr1[2], xr1[3], d);
                                d = word_f32(w.z, xr1[4], xr1[5], d);
                                d = word_f32(w.w, xr1[6], xr1[7], d);
                                acc[q][s][0] = fmaf(tb_h2f(srow[lane + 32]), d.x + d.y, acc[q][s][0]);
                            }
                        }
                    } else {
                        const uint4* wq = reinterpret_cast<const uint4*>(slot);
                        for (int g = lane; g < G; g += 32) {
                            if constexpr (RPW > 1 && KIND != KIND_F32) {
                                XQ<B> xg;
                                load_xq<B>(xg, act, G, g);
#pragma unroll
                                for (int q = 0; q < RPW; q++) {
                                    const int r = r0 + q * NW;
                                    if (r < bl.nrows) item_q8x<B>(wq[r * G + g], tb_h2f(sbase[r * G + g]), xg, acc[q][s]);
                                }
                            } else {
#pragma unroll
                                for (int q = 0; q < RPW; q++) {
                                    const int r = r0 + q * NW;
                                    if (r >= bl.nrows) continue;
                                    const uint4 w = wq[r * G + g];
                                    const float sc = tb_h2f(sbase[r * G + g]);
                                    if (KIND == KIND_F32) item_f32<B>(w, sc, act, G, g, acc[q][s]);
                                    else item_q8<B>(w, sc, act, G, g, acc[q][s]);
                                }
                            }
                        }
                    }
                }
#pragma unroll
                for (int q = 0; q < RPW; q++)
#pragma unroll
                    for (int s = 0; s < NM; s++)
#pragma unroll
                        for (int b = 0; b < B; b++) acc[q][s][b] = warp_sum(acc[q][s][b]);
                if (lane == 0) {
#pragma unroll
                    for (int q = 0; q < RPW; q++) {
                        const int r = r0 + q * NW;
                        if (r >= bl.nrows) continue;
                        const int row = bl.row0 + r;
                        if (gateup) {
                            const int N = a.m[0].N;
#pragma unroll
                            for (int b = 0; b < B; b++) {
                                const float g = acc[q][0][b], u = acc[q][NM - 1][b];
                                a.m[0].y[(size_t)b * N + row] = __fdiv_rn(g, 1.0f + expf(-g)) * u;
                            }
                        } else {
                            const Mat& M = a.m[bl.mi];
#pragma unroll
                            for (int b = 0; b < B; b++) {
                                float* yp = M.y + (size_t)b * M.N + row;
                                *yp = (a.acc ? *yp : 0.0f) + acc[q][0][b];
                            }
                        }
                    }
                }
            }
        }
        __syncthreads();   // stage st fully consumed
        if (abort_flag) break;
        if (tid == 0) {
            const int nrb2 = blockIdx.x + (j + a.nst) * gridDim.x;
            if (nrb2 < a.nrb) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue_block(a, nrb2, stages + st * stage_bytes, &bars[st], gateup);
            }
        }
    }
    if (abort_flag && tid == 0) {
        // let copies still in flight land before the CTA's shared memory is released
        for (int s = 0; s < a.nst; s++) { mbar_wait(&bars[s], 0); mbar_wait(&bars[s], 1); }
    }
}

// ---- host side ------------------------------------------------------------------
struct Plan {
    int RB, nst, slot_bytes, act_bytes, xbuf_bytes, nw_bytes, smem, grid, nrb;
};

int act_bytes_for(int kind, int B, int G)
{
    return kind == KIND_F32 ? B * G * 128 : (kind == KIND_F32D ? G * F32D_BYTES_PER_GROUP : B * G * 40);
}

int make_plan(tb_ctx* ctx, int kind, int B, int K, const int64_t* Ns, int count, bool norm, Plan& p)
{
    const int G = K / 32;
    const int nm = kind_gateup(kind) ? 2 : 1;
    const int mats = kind_gateup(kind) ? 1 : count;
    const int wrow = kind_tern(kind) ? K / 4 : K / 2;
    long long rows = 0;
    for (int i = 0; i < mats; i++) rows += Ns[i];
    p.act_bytes = (act_bytes_for(kind, B, G) + 127) & ~127;
    // f32 staging buffer for the Q8 prologue (whole rows, up to 48 KB)
    p.xbuf_bytes = kind == KIND_F32 ? 0 : std::min(B * K * 4, std::max(48 * 1024, K * 4));
    p.xbuf_bytes = (p.xbuf_bytes + 127) & ~127;
    p.nw_bytes = norm ? ((K * 2 + 127) & ~127) : 0;
    const int target = 2 * ctx->num_sms;
    const int budget = 112 * 1024;   // leave room for the next kernel's CTA under PDL
    int RB = 8;
    while (RB < 64 && rows / (2 * RB) >= target) RB *= 2;
    for (;; RB /= 2) {
        const int wb = RB * wrow, sb = RB * G * 2;
        p.slot_bytes = (wb + sb + 127) & ~127;
        const int per_stage = nm * p.slot_bytes;
        int nrb = 0;
        for (int i = 0; i < mats; i++) nrb += tb_cdiv(Ns[i], RB);
        const int blocks_per_cta = tb_cdiv(nrb, target);
        int nst = std::min(MAX_NST, std::max(1, blocks_per_cta));
        const int fixed = SMEM_HDR + p.act_bytes + p.xbuf_bytes + p.nw_bytes;
        while (nst > 1 && fixed + nst * per_stage > budget) nst--;
        p.smem = fixed + nst * per_stage;
        // a CTA that streams several row blocks keeps at least two stages, so a
        // copy is in flight while it computes (smaller blocks rather than one stage)
        const bool deep_enough = nst >= 2 || blocks_per_cta < 2;
        if ((p.smem <= 200 * 1024 && deep_enough) || RB == 8) {
            p.RB = RB;
            p.nst = nst;
            p.nrb = nrb;
            break;
        }
    }
    if (p.smem > 220 * 1024)
        return tb_fail(ctx, TB_ERR_UNSUPPORTED, "K=%d batch=%d needs %d bytes of shared memory", K, B, p.smem);
    int occ = p.smem <= 100 * 1024 ? 2 : 1;
    p.grid = std::min(p.nrb, ctx->num_sms * occ);
    return TB_OK;
}

template <int B, int KIND>
int launch_B(tb_ctx* ctx, Args& a, const Plan& p)
{
    auto kern = k_gemv<B, KIND>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    e = tb_launch(ctx, kern, dim3(p.grid), dim3(THREADS), (size_t)p.smem, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "gemv launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

template <int KIND>
int launch_kind(tb_ctx* ctx, Args& a, const Plan& p, int B)
{
    switch (B) {
    case 1: return launch_B<1, KIND>(ctx, a, p);
    case 2: return launch_B<2, KIND>(ctx, a, p);
    case 3: return launch_B<3, KIND>(ctx, a, p);
    case 4: return launch_B<4, KIND>(ctx, a, p);
    case 5: return launch_B<5, KIND>(ctx, a, p);
    case 6: return launch_B<6, KIND>(ctx, a, p);
    case 7: return launch_B<7, KIND>(ctx, a, p);
    case 8: return launch_B<8, KIND>(ctx, a, p);
    }
    return tb_fail(ctx, TB_ERR_INVALID, "batch must be 1..8 (got %d)", B);
}

int check_mat(tb_ctx* ctx, const uint32_t* pack, const uint16_t* scales, const float* y, int64_t N, int64_t K)
{
    TB_REQUIRE(ctx, pack && scales && y, "null weight or output pointer");
    TB_REQUIRE(ctx, N > 0 && N < (1LL << 30), "N out of range (%lld)", (long long)N);
    TB_REQUIRE(ctx, TB_ALIGNED(pack, 16) && TB_ALIGNED(scales, 16), "pack and scales must be 16-byte aligned");
    return TB_OK;
}

struct ActIn {
    int src;
    const float* x;
    const int8_t* xq;
    const float* xs;
    const uint16_t* normw;
    float eps;
};

int run(tb_ctx* ctx, int kind, int count, float* const* ys, const uint32_t* const* packs,
        const uint16_t* const* scales, const int64_t* Ns, const ActIn& in, int64_t K, int batch, int acc)
{
    TB_REQUIRE(ctx, K > 0 && K % 32 == 0 && K <= 16384, "K must be a multiple of 32 in [32, 16384] (got %lld)", (long long)K);
    TB_REQUIRE(ctx, batch >= 1 && batch <= 8, "batch must be 1..8 (got %d)", batch);
    TB_REQUIRE(ctx, count >= 1 && count <= 4, "count must be 1..4");
    if (in.src == ACT_PREQ) {
        TB_REQUIRE(ctx, in.xq && in.xs && TB_ALIGNED(in.xq, 16), "xq (16-byte aligned) and xs required");
    } else {
        TB_REQUIRE(ctx, in.x && TB_ALIGNED(in.x, 16), "x must be non-null and 16-byte aligned");
        TB_REQUIRE(ctx, in.src != ACT_RMSNORM || (in.normw && TB_ALIGNED(in.normw, 16)),
                   "norm weight required (16-byte aligned)");
    }
    Args a{};
    a.count = count;
    a.K = (int)K;
    a.acc = acc ? 1 : 0;
    a.act_src = in.src;
    a.x = in.x;
    a.xq = in.xq;
    a.xs = in.xs;
    a.normw = in.normw;
    a.eps = in.eps;
    a.err = ctx->dev_error;
    for (int i = 0; i < count; i++) {
        int rc = check_mat(ctx, packs[i], scales[i], ys[i], Ns[i], K);
        if (rc) return rc;
    }
    if (kind_gateup(kind)) TB_REQUIRE(ctx, Ns[0] == Ns[1], "gate and up must have the same rows");
    if (kind_tern(kind)) TB_REQUIRE(ctx, K % 64 == 0, "ternary weights need K %% 64 == 0 (got %lld)", (long long)K);
    // f32 rows take 4 bytes per element of shared memory: split big batches
    // into launches of rows that fit (each launch covers its own rows of y).
    const int bmax = kind == KIND_F32 ? std::max(1, (int)((96 * 1024) / (K * 4))) : 8;
    if (batch > bmax) {
        for (int b0 = 0; b0 < batch; b0 += bmax) {
            const int nb = std::min(bmax, batch - b0);
            float* ys2[4];
            for (int i = 0; i < count; i++) ys2[i] = ys[i] + (size_t)b0 * Ns[i];
            ActIn in2 = in;
            if (in2.x) in2.x += (size_t)b0 * K;
            int rc = run(ctx, kind, count, ys2, packs, scales, Ns, in2, K, nb, acc);
            if (rc) return rc;
        }
        return TB_OK;
    }
    // one f32 row (gemvQ's decode route): the two-digit int8 form on dp4a
    if (kind == KIND_F32 && batch == 1) kind = KIND_F32D;
    Plan p{};
    int rc = make_plan(ctx, kind, batch, (int)K, Ns, count, in.src == ACT_RMSNORM, p);
    if (rc) return rc;
    int rb = 0;
    for (int i = 0; i < 4; i++) {
        if (i < count) {
            a.m[i] = Mat{packs[i], scales[i], ys[i], (int)Ns[i], rb};
            if (!kind_gateup(kind)) rb += tb_cdiv(Ns[i], p.RB);
        } else {
            a.m[i] = Mat{nullptr, nullptr, nullptr, 0, 1 << 30};
        }
    }
    if (kind_gateup(kind)) a.m[1].rb_begin = 0;
    a.wrow_bytes = kind_tern(kind) ? (int)(K / 4) : (int)(K / 2);
    a.nrb = p.nrb;
    a.RB = p.RB;
    a.nst = p.nst;
    a.slot_bytes = p.slot_bytes;
    a.act_bytes = p.act_bytes;
    a.xbuf_bytes = p.xbuf_bytes;
    a.nw_bytes = p.nw_bytes;
    switch (kind) {
    case KIND_F32D: return launch_B<1, KIND_F32D>(ctx, a, p);
    case KIND_Q8: return launch_kind<KIND_Q8>(ctx, a, p, batch);
    case KIND_GATEUP: return launch_kind<KIND_GATEUP>(ctx, a, p, batch);
    case KIND_TERN: return launch_kind<KIND_TERN>(ctx, a, p, batch);
    case KIND_GATEUP_TERN: return launch_kind<KIND_GATEUP_TERN>(ctx, a, p, batch);
    default: return launch_kind<KIND_F32>(ctx, a, p, batch);
    }
}

ActIn act_f32(const float* x, const uint16_t* normw, float eps)
{
    return ActIn{normw ? ACT_RMSNORM : ACT_F32, x, nullptr, nullptr, normw, eps};
}
ActIn act_preq(const int8_t* xq, const float* xs) { return ActIn{ACT_PREQ, nullptr, xq, xs, nullptr, 0.0f}; }

}  // namespace

// shared with tb_linear.cu
int tb_gemv_q8_impl(tb_ctx* ctx, int count, float* const* ys, const uint32_t* const* packs,
                    const uint16_t* const* scales, const int64_t* Ns, const int8_t* xq, const float* xs,
                    int64_t K, int batch, int acc)
{
    return run(ctx, KIND_Q8, count, ys, packs, scales, Ns, act_preq(xq, xs), K, batch, acc);
}
int tb_gemv_dp4a_impl(tb_ctx* ctx, int count, float* const* ys, const uint32_t* const* packs,
                      const uint16_t* const* scales, const int64_t* Ns, const float* x, const uint16_t* normw,
                      float eps, int64_t K, int batch, int acc)
{
    return run(ctx, KIND_Q8, count, ys, packs, scales, Ns, act_f32(x, normw, eps), K, batch, acc);
}
int tb_gemv_f32_impl(tb_ctx* ctx, float* y, const float* x, const uint32_t* pack, const uint16_t* scales,
                     int64_t N, int64_t K, int batch, int acc)
{
    return run(ctx, KIND_F32, 1, &y, &pack, &scales, &N, act_f32(x, nullptr, 0.0f), K, batch, acc);
}
int tb_gemv_tern_wgsl_impl(tb_ctx* ctx, int count, float* const* ys, const uint32_t* const* packs,
                           const uint16_t* const* scales, const int64_t* Ns, const float* x, const uint16_t* normw,
                           float eps, int64_t K, int batch, int acc)
{
    return run(ctx, KIND_TERN, count, ys, packs, scales, Ns, act_f32(x, normw, eps), K, batch, acc);
}

extern "C" {

TB_API int tb_gemv_int4_q8(tb_ctx* ctx, float* y, const int8_t* xq, const float* xs, const uint32_t* pack,
                           const uint16_t* scales, int64_t N, int64_t K, int batch, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    return run(ctx, KIND_Q8, 1, &y, &pack, &scales, &N, act_preq(xq, xs), K, batch, acc);
}

TB_API int tb_gemv_int4_q8_multi(tb_ctx* ctx, int count, float* const* ys, const uint32_t* const* packs,
                                 const uint16_t* const* scales, const int64_t* Ns, const int8_t* xq,
                                 const float* xs, int64_t K, int batch, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, ys && packs && scales && Ns, "null array");
    return run(ctx, KIND_Q8, count, ys, packs, scales, Ns, act_preq(xq, xs), K, batch, acc);
}

TB_API int tb_gemv_int4_f32(tb_ctx* ctx, float* y, const float* x, const uint32_t* pack, const uint16_t* scales,
                            int64_t N, int64_t K, int batch, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    return run(ctx, KIND_F32, 1, &y, &pack, &scales, &N, act_f32(x, nullptr, 0.0f), K, batch, acc);
}

TB_API int tb_gemv_int4_f32_norm(tb_ctx* ctx, float* y, const float* x, const uint16_t* norm_w16, float eps,
                                 const uint32_t* pack, const uint16_t* scales, int64_t N, int64_t K, int batch,
                                 int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    return run(ctx, KIND_F32, 1, &y, &pack, &scales, &N, act_f32(x, norm_w16, eps), K, batch, acc);
}

TB_API int tb_gateup_silu_int4_q8(tb_ctx* ctx, float* swi, const int8_t* xq, const float* xs, const uint32_t* gpack,
                                  const uint16_t* gscales, const uint32_t* upack, const uint16_t* uscales, int64_t I,
                                  int64_t H, int batch)
{
    if (!ctx) return TB_ERR_INVALID;
    float* ys[2] = {swi, swi};
    const uint32_t* packs[2] = {gpack, upack};
    const uint16_t* scs[2] = {gscales, uscales};
    int64_t Ns[2] = {I, I};
    return run(ctx, KIND_GATEUP, 2, ys, packs, scs, Ns, act_preq(xq, xs), H, batch, 0);
}

TB_API int tb_gemv_int4_dp4a(tb_ctx* ctx, float* y, const float* x, const uint16_t* norm_w16, float eps,
                             const uint32_t* pack, const uint16_t* scales, int64_t N, int64_t K, int batch, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    return run(ctx, KIND_Q8, 1, &y, &pack, &scales, &N, act_f32(x, norm_w16, eps), K, batch, acc);
}

TB_API int tb_gemv_int4_dp4a_multi(tb_ctx* ctx, int count, float* const* ys, const uint32_t* const* packs,
                                   const uint16_t* const* scales, const int64_t* Ns, const float* x,
                                   const uint16_t* norm_w16, float eps, int64_t K, int batch, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, ys && packs && scales && Ns, "null array");
    return run(ctx, KIND_Q8, count, ys, packs, scales, Ns, act_f32(x, norm_w16, eps), K, batch, acc);
}

TB_API int tb_gateup_silu_int4_dp4a(tb_ctx* ctx, float* swi, const float* x, const uint16_t* norm_w16, float eps,
                                    const uint32_t* gpack, const uint16_t* gscales, const uint32_t* upack,
                                    const uint16_t* uscales, int64_t I, int64_t H, int batch)
{
    if (!ctx) return TB_ERR_INVALID;
    float* ys[2] = {swi, swi};
    const uint32_t* packs[2] = {gpack, upack};
    const uint16_t* scs[2] = {gscales, uscales};
    int64_t Ns[2] = {I, I};
    return run(ctx, KIND_GATEUP, 2, ys, packs, scs, Ns, act_f32(x, norm_w16, eps), H, batch, 0);
}

// ---- ternary weights, WebGPU layout ----------------------------------------------
// gemvTern_only (models/qwen3.js:548-556) against a pre-quantized QUANTQ8 row;
// the per-group sum of x is recomputed from xq in the prologue (the same exact
// integer as the reference's xsum buffer, so no xsum argument).
TB_API int tb_gemv_tern_wgsl_q8(tb_ctx* ctx, float* y, const int8_t* xq, const float* xs, const uint32_t* pack,
                                const uint16_t* scales, int64_t N, int64_t K, int batch, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    return run(ctx, KIND_TERN, 1, &y, &pack, &scales, &N, act_preq(xq, xs), K, batch, acc);
}

// quantQ8 + gemvTern_only for up to four matrices sharing one activation
// (projGemv at the q/k/v call sites, qwen3.js:558-561, 3982-3984), with the
// optional fused RMSNorm of RMSNORMQ.
TB_API int tb_gemv_tern_wgsl_dp4a_multi(tb_ctx* ctx, int count, float* const* ys, const uint32_t* const* packs,
                                        const uint16_t* const* scales, const int64_t* Ns, const float* x,
                                        const uint16_t* norm_w16, float eps, int64_t K, int batch, int acc)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, ys && packs && scales && Ns, "null array");
    return run(ctx, KIND_TERN, count, ys, packs, scales, Ns, act_f32(x, norm_w16, eps), K, batch, acc);
}

// gate+up+SiLU of ternary weights (gateupTern2Wgsl, qwen3.js:747-810, routed by
// gateUpSiluDP4_only, qwen3.js:861-870).
TB_API int tb_gateup_silu_tern_wgsl_q8(tb_ctx* ctx, float* swi, const int8_t* xq, const float* xs,
                                       const uint32_t* gpack, const uint16_t* gscales, const uint32_t* upack,
                                       const uint16_t* uscales, int64_t I, int64_t H, int batch)
{
    if (!ctx) return TB_ERR_INVALID;
    float* ys[2] = {swi, swi};
    const uint32_t* packs[2] = {gpack, upack};
    const uint16_t* scs[2] = {gscales, uscales};
    int64_t Ns[2] = {I, I};
    return run(ctx, KIND_GATEUP_TERN, 2, ys, packs, scs, Ns, act_preq(xq, xs), H, batch, 0);
}

TB_API int tb_gateup_silu_tern_wgsl_dp4a(tb_ctx* ctx, float* swi, const float* x, const uint16_t* norm_w16,
                                         float eps, const uint32_t* gpack, const uint16_t* gscales,
                                         const uint32_t* upack, const uint16_t* uscales, int64_t I, int64_t H,
                                         int batch)
{
    if (!ctx) return TB_ERR_INVALID;
    float* ys[2] = {swi, swi};
    const uint32_t* packs[2] = {gpack, upack};
    const uint16_t* scs[2] = {gscales, uscales};
    int64_t Ns[2] = {I, I};
    return run(ctx, KIND_GATEUP_TERN, 2, ys, packs, scs, Ns, act_f32(x, norm_w16, eps), H, batch, 0);
}

}  // extern "C"
