// tb_qwen3.cu -- the Qwen3 decode step (models/qwen3.js forward, 3938-4069, the
// T = 1 / int8-KV branch) as one CUDA graph per step, tensor-parallel across
// the GPUs of one box.
//
// Per step and sequence (batch B, positions pos_b held on the device):
//   x = f32(embed_f16[ids_b])                                   embedGather :3959
//   per layer:
//     q,k,v = W_{q,k,v} . int8(rmsnorm(x) * ln1)                rmsnormQ + projGemv :3981-3984
//     qr, K/V cache row pos_b = attnPrepQ8(q, k, v)             :4003
//     attn = attentionQ8(qr, cache, S_b = pos_b + 1)            :4004
//     x += W_o . int8(attn)                                     linearQ acc :4015
//     swi = silu(W_g . a) * (W_u . a), a = int8(rmsnorm(x)*ln2) rmsnormQ + gateUpSiluDP4_only :4023-4024
//     x += W_down . int8(swi)                                   linearQ acc :4033
//   logits = W_lm . (rmsnorm(x) * final_norm)                   :4037-4049 (gemvQ at B = 1)
//   ids_b = argmax(logits_b); pos_b += 1                        argmaxKernel :4058
//
// Tensor parallelism over P ranks (one context per GPU, one process per GPU):
// q/k/v and gate/up keep their row blocks (rank r: q heads [r*nHq/P, ...),
// kv heads [r*nKv/P, ...), the matching gate/up rows), o and down keep their
// column blocks (the matching attn / swi slice), and after each of them the
// partial products are summed with an NCCL allreduce of the B x hidden f32
// residual.  The lm_head keeps vocab rows [r*V/P, ...); each rank's argmax key
// (value, global index) is all-gathered and every rank takes the same winner.
// KV heads are never exchanged: each rank caches only its own heads.
#include "tb_internal.h"

#include <dlfcn.h>
#include <nccl.h>

#include <mutex>
#include <vector>

namespace {

constexpr int GEMV_MAX_B = 8;      // rows per fused-GEMV launch (dp4a GEMV)
constexpr int MMA_MIN_B = 2;       // rows from which the tensor-core GEMV reads each weight once
constexpr int MMA_MAX_B = 16;      // rows per tensor-core GEMV launch

// NCCL entry points, resolved from the process's libnccl.so.2 (the one the
// framework that created the ranks already loaded, when there is one).
struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
    std::string why;
};

NcclApi& nccl()
{
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) { api.why = std::string("cannot load libnccl.so.2: ") + dlerror(); return; }
        api.GetUniqueId = (decltype(api.GetUniqueId))dlsym(h, "ncclGetUniqueId");
        api.CommInitRank = (decltype(api.CommInitRank))dlsym(h, "ncclCommInitRank");
        api.CommDestroy = (decltype(api.CommDestroy))dlsym(h, "ncclCommDestroy");
        api.AllReduce = (decltype(api.AllReduce))dlsym(h, "ncclAllReduce");
        api.AllGather = (decltype(api.AllGather))dlsym(h, "ncclAllGather");
        api.GetErrorString = (decltype(api.GetErrorString))dlsym(h, "ncclGetErrorString");
        api.ok = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.AllReduce && api.AllGather &&
                 api.GetErrorString;
        if (!api.ok) api.why = "libnccl.so.2 lacks an expected symbol";
    });
    return api;
}

// a quantized weight record: int4 G32 (pack [N][K/8]) or ternary in the WebGPU
// layout (pack [N][K/16]), f16 scales [N][K/32] either way (the reference's
// wrec {pack, scales, int4 | tern}); storage is sized for int4
struct Mat {
    uint32_t* pack = nullptr;
    uint16_t* scales = nullptr;
    int64_t N = 0, K = 0;
    bool set = false;
    bool tern = false;
};

struct Layer {
    Mat q, k, v, o, gate, up, down;
    uint16_t *ln1 = nullptr, *ln2 = nullptr, *qn = nullptr, *kn = nullptr;
    int8_t *Kq = nullptr, *Vq = nullptr;
    float *Ks = nullptr, *Vs = nullptr;
};

}  // namespace

struct tb_qwen3 {
    tb_ctx* ctx = nullptr;
    tb_qwen3_config c{};
    int P = 1, r = 0;
    int64_t nHq = 0, nKv = 0, I = 0, V = 0;      // this rank's heads, intermediate rows, vocab rows
    std::vector<Layer> L;
    uint16_t* embed = nullptr;                   // f16 [vocab][H] (whole table on every rank)
    uint16_t* fnorm = nullptr;
    Mat lm;
    // activations
    float* x[2] = {nullptr, nullptr};            // residual (ping-pong under TP)
    float *q = nullptr, *k = nullptr, *v = nullptr, *qr = nullptr, *attn = nullptr, *swi = nullptr;
    float *logits = nullptr, *PO = nullptr, *PML = nullptr;
    unsigned* counters = nullptr;
    uint32_t* ids = nullptr;
    int32_t* pos = nullptr;
    unsigned long long *amax_part = nullptr, *amax_key = nullptr, *amax_all = nullptr;
    int nsplit = 1, amax_nparts = 1;
    // graph
    cudaStream_t cap_stream = nullptr;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    // tensor parallel: NCCL, or the exchange kernels over IPC-mapped peer arenas
    ncclComm_t comm = nullptr;
    char* arena = nullptr;                       // this rank's exchange arena (tb_tp.cu)
    char* peer_arena[8] = {};                    // every rank's arena, mapped here (own at [r])
    bool p2p = false;
    int ncoll = 0;                               // NCCL calls in the recorded step
    std::vector<void*> allocs;
    // prefill (forward at T > 1): buffers of `pf_cap` rows, grown on demand
    int64_t pf_cap = 0;
    float *pf_x = nullptr, *pf_q = nullptr, *pf_k = nullptr, *pf_v = nullptr, *pf_qr = nullptr,
          *pf_attn = nullptr, *pf_gate = nullptr, *pf_xs = nullptr;
    int8_t* pf_xq = nullptr;
    uint32_t* pf_ids = nullptr;
    int32_t* pf_pos = nullptr;
    // the decode step as one persistent kernel (tb_step.cu) when it applies
    int step_mode = TB_QW_STEP_AUTO;             // requested
    int step_kind = 0;                           // recorded: TB_QW_STEP_KERNELS or TB_QW_STEP_PERSISTENT
    tb_step_plan* step = nullptr;
    unsigned char* step_layers = nullptr;        // device per-layer records
    int step_tern = -1;                          // weight format the plan was made for (1 ternary)
    unsigned* step_ctrl = nullptr;               // [256] block arrivals, grid barrier, abort word
    unsigned* step_heads = nullptr;              // [layers][kv heads] phase-A arrivals of the persistent step
    unsigned long long* step_pk = nullptr;       // [hidden] phase-boundary packets of x after o
    unsigned char* step_attnq = nullptr;         // quantized attention output of the persistent step
    unsigned char* mma_act = nullptr;            // fragment-ordered int8 rows of the tensor-core GEMVs
    unsigned char* mma_act2 = nullptr;           // ... of the down GEMV, written by the gate/up epilogue
    bool step_direct = false;                    // persistent step launched per call (not capturable)
    void* step_trace = nullptr;                  // optional phase trace of the persistent kernel
};

namespace {

template <typename T>
int alloc(tb_qwen3* m, T** p, size_t count)
{
    void* q = nullptr;
    size_t bytes = (count * sizeof(T) + 255) & ~size_t(255);
    if (cudaMalloc(&q, bytes ? bytes : 256) != cudaSuccess) {
        cudaGetLastError();
        return tb_fail(m->ctx, TB_ERR_NOMEM, "qwen3: cudaMalloc of %zu bytes failed", bytes);
    }
    m->allocs.push_back(q);
    *p = static_cast<T*>(q);
    return TB_OK;
}

int alloc_mat(tb_qwen3* m, Mat& w, int64_t N, int64_t K)
{
    w.N = N; w.K = K;
    int rc = alloc(m, &w.pack, (size_t)N * K / 8);
    if (!rc) rc = alloc(m, &w.scales, (size_t)N * K / 32);
    return rc;
}

// the slice of a full [rows][cols] tensor that rank r keeps (rows x cols block)
struct Slice { int64_t row0, nrows, col0, ncols; };

int shard_of(const tb_qwen3_config& c, int kind, Slice& s, int64_t* full_rows, int64_t* full_cols)
{
    const int64_t P = c.tp_size, r = c.tp_rank, H = c.hidden, hd = c.head_dim;
    const int64_t qN = (int64_t)c.n_heads * hd, kvN = (int64_t)c.n_kv_heads * hd, I = c.intermediate, V = c.vocab;
    int64_t R = 0, C = 0;
    switch (kind) {
    case TB_QW_EMBED: R = V; C = H; s = {0, V, 0, H}; break;
    case TB_QW_LM_HEAD: R = V; C = H; s = {r * (V / P), V / P, 0, H}; break;
    case TB_QW_FINAL_NORM: case TB_QW_LN_ATTN: case TB_QW_LN_MLP: R = 1; C = H; s = {0, 1, 0, H}; break;
    case TB_QW_Q_NORM: case TB_QW_K_NORM: R = 1; C = hd; s = {0, 1, 0, hd}; break;
    case TB_QW_Q: R = qN; C = H; s = {r * (qN / P), qN / P, 0, H}; break;
    case TB_QW_K: case TB_QW_V: R = kvN; C = H; s = {r * (kvN / P), kvN / P, 0, H}; break;
    case TB_QW_O: R = H; C = qN; s = {0, H, r * (qN / P), qN / P}; break;
    case TB_QW_GATE: case TB_QW_UP: R = I; C = H; s = {r * (I / P), I / P, 0, H}; break;
    case TB_QW_DOWN: R = H; C = I; s = {0, H, r * (I / P), I / P}; break;
    default: return TB_ERR_INVALID;
    }
    if (full_rows) *full_rows = R;
    if (full_cols) *full_cols = C;
    return TB_OK;
}

int check_config(const tb_qwen3_config& c, char* why, size_t n)
{
    const int P = c.tp_size;
    auto bad = [&](const char* s) { snprintf(why, n, "%s", s); return TB_ERR_INVALID; };
    if (c.hidden <= 0 || c.layers <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0 ||
        c.intermediate <= 0 || c.vocab <= 0 || c.max_seq <= 0)
        return bad("all sizes must be positive");
    if (P < 1 || c.tp_rank < 0 || c.tp_rank >= P) return bad("bad tp_size / tp_rank");
    if (c.batch < 1 || c.batch > 16) return bad("batch must be 1..16");
    if (c.head_dim != 64 && c.head_dim != 128) return bad("head_dim must be 64 or 128");
    if (c.n_heads % c.n_kv_heads) return bad("n_heads must be a multiple of n_kv_heads");
    const int grp = c.n_heads / c.n_kv_heads;
    if (grp != 1 && grp != 2 && grp != 4 && grp != 8) return bad("n_heads / n_kv_heads must be 1, 2, 4 or 8");
    if (c.n_kv_heads % P) return bad("n_kv_heads must be a multiple of tp_size (kv heads are sharded whole)");
    if (c.hidden % 32 || c.hidden % 4) return bad("hidden must be a multiple of 32");
    if (c.intermediate % (32 * P)) return bad("intermediate must be a multiple of 32 * tp_size");
    if (c.vocab % P) return bad("vocab must be a multiple of tp_size");
    if ((int64_t)c.batch * (c.n_kv_heads / P) > TB_ATTN_MAX_KV) return bad("batch * kv heads per rank too large");
    if (c.vocab >= (1LL << 31)) return bad("vocab too large");
    if (c.ternary != 0 && c.ternary != 1) return bad("ternary must be 0 or 1");
    return TB_OK;
}

// ---- the step, issued on ctx->stream ------------------------------------------
#define TRY(x) do { int rc_ = (x); if (rc_) return rc_; } while (0)

int nccl_check(tb_qwen3* m, ncclResult_t r, const char* what)
{
    if (r == ncclSuccess) return TB_OK;
    return tb_fail(m->ctx, TB_ERR_CUDA, "%s: %s", what, nccl().GetErrorString(r));
}

// The tensor-core GEMV (every weight read once for up to MMA_MAX_B rows) runs
// the matrices of a call when the batch has at least MMA_MIN_B rows and their
// shapes fit it; otherwise the dp4a GEMV in launches of GEMV_MAX_B rows.
bool use_mma(const tb_qwen3* m, const int64_t* Ns, int count, int64_t K)
{
    return m->mma_act && m->c.batch >= MMA_MIN_B && tb_gemv_mma_fits(K, Ns, count, MMA_MIN_B);
}

// y (+)= W . x over B rows, in launches of at most GEMV_MAX_B rows (fused int8
// quantization of x, optional fused RMSNorm with norm_w); with preq, x's rows are
// already in the tensor-core GEMV's fragment order there (one launch)
int gemv_rows(tb_qwen3* m, float* y, const float* x, const Mat& w, const uint16_t* norm_w, int acc,
              void* preq = nullptr)
{
    const int B = m->c.batch;
    const bool mma = use_mma(m, &w.N, 1, w.K);
    if (preq) {   // the rows are already quantized by their producer (all B in one launch)
        return tb_gemv_mma_impl(m->ctx, 1, &y, &w.pack, &w.scales, &w.N, x, nullptr, m->c.rms_eps, w.K, B, acc,
                                w.tern, false, preq, false);
    }
    const int chunk = mma ? MMA_MAX_B : GEMV_MAX_B;
    for (int b0 = 0; b0 < B; b0 += chunk) {
        const int nb = std::min(chunk, B - b0);
        float* yb = y + (int64_t)b0 * w.N;
        const float* xb = x + (int64_t)b0 * w.K;
        if (mma && nb >= MMA_MIN_B)
            TRY(tb_gemv_mma_impl(m->ctx, 1, &yb, &w.pack, &w.scales, &w.N, xb, norm_w, m->c.rms_eps, w.K, nb, acc,
                                 w.tern, false, m->mma_act));
        else if (w.tern)
            TRY(tb_gemv_tern_wgsl_impl(m->ctx, 1, &yb, &w.pack, &w.scales, &w.N, xb, norm_w, m->c.rms_eps, w.K, nb,
                                       acc));
        else
            TRY(tb_gemv_int4_dp4a(m->ctx, yb, xb, norm_w, m->c.rms_eps, w.pack, w.scales, w.N, w.K, nb, acc));
    }
    return TB_OK;
}

// x_next = x + sum over ranks of (W_r . a_r); `cur` names the buffer holding
// x_next afterwards.  xi: index of this exchange within the step.
int proj_residual(tb_qwen3* m, int& cur, const float* a, const Mat& w, int xi, void* preq = nullptr)
{
    if (m->P == 1) return gemv_rows(m, m->x[cur], a, w, nullptr, 1, preq);
    if (m->p2p) {
        const int64_t n = (int64_t)m->c.batch * m->c.hidden;
        float* part; unsigned long long* keys; unsigned *flag, *flag2, *step;
        tb_tp_arena_layout(m->arena, n, &part, &keys, &flag, &flag2, &step);
        TRY(gemv_rows(m, part + (size_t)((xi + 1) & 1) * n, a, w, nullptr, 0, preq));
        return tb_tp_allreduce_impl(m->ctx, m->peer_arena, m->P, m->r, n, m->x[cur], xi, 2 * m->c.layers);
    }
    const int nxt = cur ^ 1;
    const size_t bytes = (size_t)m->c.batch * m->c.hidden * sizeof(float);
    if (m->r == 0) {
        // rank 0 carries the residual into the sum
        cudaError_t e = cudaMemcpyAsync(m->x[nxt], m->x[cur], bytes, cudaMemcpyDeviceToDevice, m->ctx->stream);
        if (e != cudaSuccess) return tb_fail(m->ctx, TB_ERR_CUDA, "residual copy: %s", cudaGetErrorString(e));
        TRY(gemv_rows(m, m->x[nxt], a, w, nullptr, 1, preq));
    } else {
        TRY(gemv_rows(m, m->x[nxt], a, w, nullptr, 0, preq));
    }
    TRY(nccl_check(m, nccl().AllReduce(m->x[nxt], m->x[nxt], (size_t)m->c.batch * m->c.hidden, ncclFloat32, ncclSum,
                                       m->comm, m->ctx->stream), "allreduce"));
    m->ncoll++;
    cur = nxt;
    return TB_OK;
}

int issue_head(tb_qwen3* m, int cur);

// Can this model's step run as the persistent kernel?  (batch 1, one GPU or
// tensor parallel over the peer-memory exchange arenas, q/k/v/o/gate/up/down
// all int4 or all ternary in every layer, sizes tb_step_plan_make accepts)
bool persistent_ok(tb_qwen3* m)
{
    if (m->c.batch != 1 || m->L.empty() || (m->P > 1 && !m->p2p)) return false;
    const bool tern = m->L[0].q.tern;
    for (const Layer& Ly : m->L) {
        const Mat* ms[7] = {&Ly.q, &Ly.k, &Ly.v, &Ly.o, &Ly.gate, &Ly.up, &Ly.down};
        for (const Mat* w : ms)
            if (w->tern != tern) return false;
    }
    if (m->step && m->step_tern != (int)tern) {   // the weights changed format since the plan was made
        tb_step_plan_free(m->step);
        m->step = nullptr;
    }
    if (!m->step) {
        if (tb_step_plan_make(m->ctx, m->c.layers, m->c.hidden, (int)m->nHq, (int)m->nKv, m->c.head_dim, (int)m->I,
                              m->nsplit, m->c.max_seq, (int)tern, m->P, &m->step) != TB_OK)
            return false;
        m->step_tern = (int)tern;
    }
    if (!m->step_layers) {
        const size_t rec = tb_step_layer_bytes();
        std::vector<unsigned char> host(rec * m->L.size());
        for (size_t l = 0; l < m->L.size(); l++) {
            const Layer& Ly = m->L[l];
            const uint32_t* packs[7] = {Ly.q.pack, Ly.k.pack, Ly.v.pack, Ly.o.pack, Ly.gate.pack, Ly.up.pack,
                                        Ly.down.pack};
            const uint16_t* scs[7] = {Ly.q.scales, Ly.k.scales, Ly.v.scales, Ly.o.scales, Ly.gate.scales,
                                      Ly.up.scales, Ly.down.scales};
            tb_step_layer_fill(host.data() + rec * l, packs, scs, Ly.ln1, Ly.ln2, Ly.qn, Ly.kn, Ly.Kq, Ly.Ks, Ly.Vq,
                               Ly.Vs);
        }
        if (alloc(m, &m->step_layers, host.size()) || alloc(m, &m->step_ctrl, 256) ||
            alloc(m, &m->step_heads, (size_t)m->c.layers * m->nKv) ||
            alloc(m, &m->step_pk, (size_t)m->c.hidden) ||
            alloc(m, &m->step_attnq, (size_t)m->nHq * m->c.head_dim / 32 * 40))
            return false;
        if (cudaMemcpy(m->step_layers, host.data(), host.size(), cudaMemcpyHostToDevice) != cudaSuccess ||
            cudaMemset(m->step_ctrl, 0, 256 * 4) != cudaSuccess ||
            cudaMemset(m->step_pk, 0, (size_t)m->c.hidden * 8) != cudaSuccess) {
            cudaGetLastError();
            m->step_layers = nullptr;
            return false;
        }
    }
    return true;
}

// the step as embed + 28 layers in one persistent kernel, then the shared head
tb_step_io step_io(tb_qwen3* m)
{
    tb_step_io io{};
    io.layers = m->step_layers;
    io.eps = m->c.rms_eps;
    io.theta = m->c.rope_theta;
    io.ids = m->ids;
    io.pos = m->pos;
    io.embed = m->embed;
    io.x = m->x[0]; io.q = m->q; io.k = m->k; io.v = m->v; io.qr = m->qr; io.attn = m->attn; io.swi = m->swi;
    io.PO = m->PO; io.PML = m->PML; io.counters = m->counters; io.ctrl = m->step_ctrl; io.head_cnt = m->step_heads;
    io.pk = m->step_pk;
    io.trace = m->step_trace;
    io.attnq = m->step_attnq;
    io.P = m->P;
    io.rank = m->r;
    if (m->P > 1) {
        const int64_t n = (int64_t)m->c.batch * m->c.hidden;
        for (int s = 0; s < m->P; s++) io.tp_inbox[s] = tb_tp_arena_step_inbox(m->peer_arena[s], n);
        float* part; unsigned long long* keys; unsigned *flag, *flag2, *step;
        tb_tp_arena_layout(m->arena, n, &part, &keys, &flag, &flag2, &step);
        io.xpart = part;
        io.tp_poison = step + 1;
    }
    return io;
}

int issue_step_persistent(tb_qwen3* m)
{
    const tb_step_io io = step_io(m);
    TRY(tb_step_launch(m->ctx, m->step, &io));
    return issue_head(m, 0);
}

int issue_step(tb_qwen3* m)
{
    tb_ctx* ctx = m->ctx;
    const tb_qwen3_config& c = m->c;
    const int B = c.batch, H = c.hidden, hd = c.head_dim;
    int cur = 0;
    m->ncoll = 0;
    TRY(tb_embed_gather(ctx, m->ids, 0, m->embed, m->x[cur], B, H));
    for (int l = 0; l < c.layers; l++) {
        Layer& Ly = m->L[l];
        // fused rmsnormQ + q/k/v (one launch per <= 8 rows, or per <= 16 rows on
        // the tensor cores)
        const bool same_kind = Ly.q.tern == Ly.k.tern && Ly.k.tern == Ly.v.tern;
        const int64_t qkvN[3] = {Ly.q.N, Ly.k.N, Ly.v.N};
        const bool qkv_mma = same_kind && use_mma(m, qkvN, 3, H);
        const int qkv_chunk = qkv_mma ? MMA_MAX_B : GEMV_MAX_B;
        for (int b0 = 0; b0 < B; b0 += qkv_chunk) {
            const int nb = std::min(qkv_chunk, B - b0);
            float* ys[3] = {m->q + (int64_t)b0 * Ly.q.N, m->k + (int64_t)b0 * Ly.k.N, m->v + (int64_t)b0 * Ly.v.N};
            const uint32_t* packs[3] = {Ly.q.pack, Ly.k.pack, Ly.v.pack};
            const uint16_t* scs[3] = {Ly.q.scales, Ly.k.scales, Ly.v.scales};
            const int64_t* Ns = qkvN;
            const float* xb = m->x[cur] + (int64_t)b0 * H;
            if (qkv_mma && nb >= MMA_MIN_B) {
                TRY(tb_gemv_mma_impl(ctx, 3, ys, packs, scs, Ns, xb, Ly.ln1, c.rms_eps, H, nb, 0, Ly.q.tern, false,
                                     m->mma_act));
            } else if (same_kind) {
                if (Ly.q.tern) TRY(tb_gemv_tern_wgsl_impl(ctx, 3, ys, packs, scs, Ns, xb, Ly.ln1, c.rms_eps, H, nb, 0));
                else TRY(tb_gemv_int4_dp4a_multi(ctx, 3, ys, packs, scs, Ns, xb, Ly.ln1, c.rms_eps, H, nb, 0));
            } else {   // mixed weight kinds: one launch per matrix
                const Mat* ms[3] = {&Ly.q, &Ly.k, &Ly.v};
                for (int i = 0; i < 3; i++) {
                    if (ms[i]->tern)
                        TRY(tb_gemv_tern_wgsl_impl(ctx, 1, &ys[i], &packs[i], &scs[i], &Ns[i], xb, Ly.ln1, c.rms_eps,
                                                   H, nb, 0));
                    else
                        TRY(tb_gemv_int4_dp4a(ctx, ys[i], xb, Ly.ln1, c.rms_eps, packs[i], scs[i], Ns[i], H, nb, 0));
                }
            }
        }
        TRY(tb_attn_prep_q8_batch(ctx, m->q, m->k, m->v, Ly.qn, Ly.kn, m->qr, Ly.Kq, Ly.Ks, Ly.Vq, Ly.Vs, m->nHq,
                                  m->nKv, hd, B, c.max_seq, m->pos, c.rope_theta, c.rms_eps));
        // the whole batch in one tensor-core launch: the attention writes the o GEMV's
        // rows already quantized, and the gate/up epilogue the down GEMV's
        const bool one_mma = m->mma_act2 && B <= MMA_MAX_B;
        const bool o_fused = one_mma && use_mma(m, &Ly.o.N, 1, Ly.o.K) && (m->nHq / m->nKv * hd) % 128 == 0;
        const int ts = B > 8 ? 16 : 8;
        unsigned char* oxa = o_fused ? m->mma_act : nullptr;
        uint2* oxk = o_fused ? reinterpret_cast<uint2*>(m->mma_act + (size_t)(Ly.o.K / 32) * ts * 32) : nullptr;
        TRY(tb_attn_decode_impl(ctx, m->attn, m->qr, Ly.Kq, Ly.Ks, Ly.Vq, Ly.Vs, c.max_seq, m->nHq, m->nKv, hd,
                                m->nsplit, m->PO, m->PML, m->counters, B, c.max_seq, m->pos, true, oxa, oxk, ts,
                                Ly.o.tern));
        TRY(proj_residual(m, cur, m->attn, Ly.o, 2 * l, oxa));
        const int64_t guN[2] = {m->I, m->I};
        const bool gu_mma = Ly.gate.tern == Ly.up.tern && use_mma(m, guN, 2, H);
        const bool down_fused = one_mma && gu_mma && m->I % 32 == 0 && use_mma(m, &Ly.down.N, 1, Ly.down.K);
        const int gu_chunk = gu_mma ? MMA_MAX_B : GEMV_MAX_B;
        for (int b0 = 0; b0 < B; b0 += gu_chunk) {
            const int nb = std::min(gu_chunk, B - b0);
            if (gu_mma && nb >= MMA_MIN_B) {
                float* ys[2] = {m->swi + (int64_t)b0 * m->I, m->swi + (int64_t)b0 * m->I};
                const uint32_t* packs[2] = {Ly.gate.pack, Ly.up.pack};
                const uint16_t* scs[2] = {Ly.gate.scales, Ly.up.scales};
                TRY(tb_gemv_mma_impl(ctx, 2, ys, packs, scs, guN, m->x[cur] + (int64_t)b0 * H, Ly.ln2, c.rms_eps, H,
                                     nb, 0, Ly.gate.tern, true, m->mma_act, true,
                                     down_fused ? m->mma_act2 : nullptr, Ly.down.tern));
            } else if (Ly.gate.tern)   // gateUpSiluQ's ternary branch (qwen3.js:730)
                TRY(tb_gateup_silu_tern_wgsl_dp4a(ctx, m->swi + (int64_t)b0 * m->I, m->x[cur] + (int64_t)b0 * H,
                                                  Ly.ln2, c.rms_eps, Ly.gate.pack, Ly.gate.scales, Ly.up.pack,
                                                  Ly.up.scales, m->I, H, nb));
            else
                TRY(tb_gateup_silu_int4_dp4a(ctx, m->swi + (int64_t)b0 * m->I, m->x[cur] + (int64_t)b0 * H, Ly.ln2,
                                             c.rms_eps, Ly.gate.pack, Ly.gate.scales, Ly.up.pack, Ly.up.scales, m->I,
                                             H, nb));
        }
        TRY(proj_residual(m, cur, m->swi, Ly.down, 2 * l + 1, down_fused ? m->mma_act2 : nullptr));
    }
    return issue_head(m, cur);
}

// final norm + lm_head + argmax of the step (x[cur] holds the last layer's output)
int issue_head(tb_qwen3* m, int cur)
{
    tb_ctx* ctx = m->ctx;
    const tb_qwen3_config& c = m->c;
    const int B = c.batch, H = c.hidden;
    // final norm + lm_head: gemvQ (f32 activation) at one row, as linearQ routes
    // T = 1 with N >= 16384; the int8 DP4A GEMV for several rows; a ternary
    // lm_head takes gemvTern at every N (qwen3.js:1594-1598)
    if (B == 1 && m->V >= 16384 && !m->lm.tern) {
        TRY(tb_gemv_int4_f32_norm(ctx, m->logits, m->x[cur], m->fnorm, c.rms_eps, m->lm.pack, m->lm.scales, m->V, H, 1,
                                  0));
    } else {
        TRY(gemv_rows(m, m->logits, m->x[cur], m->lm, m->fnorm, 0));
    }
    if (m->P == 1) {
        TRY(tb_argmax_impl(ctx, m->logits, m->V, B, m->ids, m->amax_part, m->amax_nparts, nullptr, 0, m->pos));
    } else if (m->p2p) {
        const int64_t n = (int64_t)B * H;
        float* part; unsigned long long* keys; unsigned *flag, *flag2, *step;
        tb_tp_arena_layout(m->arena, n, &part, &keys, &flag, &flag2, &step);
        TRY(tb_argmax_impl(ctx, m->logits, m->V, B, nullptr, m->amax_part, m->amax_nparts, keys,
                           (uint32_t)(m->r * m->V), nullptr));
        TRY(tb_tp_argmax_merge_impl(ctx, m->peer_arena, m->P, m->r, n, B, m->ids, m->pos));
    } else {
        TRY(tb_argmax_impl(ctx, m->logits, m->V, B, nullptr, m->amax_part, m->amax_nparts, m->amax_key,
                           (uint32_t)(m->r * m->V), nullptr));
        TRY(nccl_check(m, nccl().AllGather(m->amax_key, m->amax_all, (size_t)B, ncclUint64, m->comm, ctx->stream),
                       "allgather"));
        m->ncoll++;
        TRY(tb_argmax_merge_impl(ctx, m->amax_all, m->P, B, m->ids, m->pos));
    }
    return TB_OK;
}

void free_prefill(tb_qwen3* m)
{
    for (void* p : {(void*)m->pf_x, (void*)m->pf_q, (void*)m->pf_k, (void*)m->pf_v,
                    (void*)m->pf_qr, (void*)m->pf_attn, (void*)m->pf_gate, (void*)m->pf_xs, (void*)m->pf_xq,
                    (void*)m->pf_ids, (void*)m->pf_pos})
        if (p) cudaFree(p);
    m->pf_x = m->pf_q = m->pf_k = m->pf_v = m->pf_qr = m->pf_attn = m->pf_gate = m->pf_xs = nullptr;
    m->pf_xq = nullptr;
    m->pf_ids = nullptr;
    m->pf_pos = nullptr;
    m->pf_cap = 0;
}

int prefill_buffers(tb_qwen3* m, int64_t Tp)
{
    if (m->pf_cap >= Tp) return TB_OK;
    cudaStreamSynchronize(m->ctx->stream);   // earlier prefills may still use the old buffers
    free_prefill(m);
    const tb_qwen3_config& c = m->c;
    const int64_t H = c.hidden, qN = (int64_t)c.n_heads * c.head_dim, kvN = (int64_t)c.n_kv_heads * c.head_dim;
    const int64_t kmax = std::max(H, std::max(qN, (int64_t)c.intermediate));
    bool ok = true;
    auto get = [&](auto** p, size_t bytes) {
        if (ok && cudaMalloc((void**)p, (bytes + 255) & ~size_t(255)) != cudaSuccess) { cudaGetLastError(); ok = false; }
    };
    get(&m->pf_x, Tp * H * 4);
    get(&m->pf_q, Tp * qN * 4); get(&m->pf_k, Tp * kvN * 4); get(&m->pf_v, Tp * kvN * 4);
    get(&m->pf_qr, Tp * qN * 4); get(&m->pf_attn, Tp * qN * 4); get(&m->pf_gate, Tp * c.intermediate * 4);
    get(&m->pf_xq, Tp * kmax); get(&m->pf_xs, Tp * (kmax / 32) * 4);
    get(&m->pf_ids, Tp * 4); get(&m->pf_pos, Tp * 4);
    if (!ok) {
        free_prefill(m);
        return tb_fail(m->ctx, TB_ERR_NOMEM, "qwen3 prefill: cudaMalloc for %lld rows failed", (long long)Tp);
    }
    m->pf_cap = Tp;
    return TB_OK;
}

// y (=, +=, = silu(y) *) W . x for the prefill rows, x already quantized (QUANTQ8T)
int pf_gemm(tb_qwen3* m, float* y, const Mat& w, int64_t Tp, int epi)
{
    return tb_gemm_dp4_impl(m->ctx, y, m->pf_xq, m->pf_xs, w.pack, w.scales, Tp, w.N, w.K, epi, w.tern);
}

int pf_quant(tb_qwen3* m, const float* x, int64_t Tp, int64_t K)
{
    return tb_quant_q8_impl(m->ctx, x, m->pf_xq, m->pf_xs, nullptr, Tp, K);
}

// x += W . a for the prefill rows: one rank adds into x; under tensor
// parallelism (row-split W) rank 0 carries the residual, the others write their
// partial sums over x, and an allreduce over all ranks completes x
int pf_residual(tb_qwen3* m, const Mat& w, int64_t Tp)
{
    if (m->P == 1) return pf_gemm(m, m->pf_x, w, Tp, 1);
    TRY(pf_gemm(m, m->pf_x, w, Tp, m->r == 0 ? 1 : 0));
    return nccl_check(m, nccl().AllReduce(m->pf_x, m->pf_x, (size_t)(Tp * m->c.hidden), ncclFloat32, ncclSum, m->comm,
                                          m->ctx->stream), "prefill allreduce");
}

// forward(ids, posBase) at T > 1 for sequence `seq` (models/qwen3.js:3938-4069,
// the prefill branch): rmsnorm -> q/k/v (linearQ: QUANTQ8T + gemmDP4A, or
// gemmTern, with exact group sums) -> rope + quantized KV write -> int8-KV prefill attention -> o
// (+= residual) -> rmsnorm -> gate, up (swiglu fused) -> down (+= residual);
// final rmsnorm + lm_head of the last row; argmax into ids[seq]; pos[seq] =
// pos0 + T.  Rows are padded to the GEMM's 128 (zero rows stay zero).
int prefill(tb_qwen3* m, int seq, const uint32_t* ids_host, int64_t T, int64_t pos0)
{
    tb_ctx* ctx = m->ctx;
    const tb_qwen3_config& c = m->c;
    const int64_t H = c.hidden, hd = c.head_dim, qN = m->nHq * hd, kvN = m->nKv * hd, I = m->I, V = m->V;
    const int64_t Tp = (T + 127) / 128 * 128;
    TRY(prefill_buffers(m, Tp));
    std::vector<int32_t> posv((size_t)T);
    for (int64_t t = 0; t < T; t++) posv[t] = (int32_t)(pos0 + t);
    cudaError_t e = cudaMemcpyAsync(m->pf_ids, ids_host, (size_t)T * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(m->pf_pos, posv.data(), (size_t)T * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess && Tp > T) e = cudaMemsetAsync(m->pf_x + T * H, 0, (size_t)(Tp - T) * H * 4, ctx->stream);
    if (e == cudaSuccess && Tp > T) e = cudaMemsetAsync(m->pf_attn + T * qN, 0, (size_t)(Tp - T) * qN * 4, ctx->stream);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "prefill setup: %s", cudaGetErrorString(e));
    TRY(tb_embed_gather(ctx, m->pf_ids, 0, m->embed, m->pf_x, T, H));
    const int64_t crow = (int64_t)seq * c.max_seq * kvN;   // this sequence's cache
    for (int l = 0; l < c.layers; l++) {
        Layer& Ly = m->L[l];
        // rmsnormQ of the rows straight into the GEMM's int8 input (the same bits
        // as rmsnorm then QUANTQ8T, without the f32 round trip)
        TRY(tb_rmsnorm_q8(ctx, m->pf_x, Ly.ln1, c.rms_eps, m->pf_xq, m->pf_xs, nullptr, Tp, H));
        TRY(pf_gemm(m, m->pf_q, Ly.q, Tp, 0));
        TRY(pf_gemm(m, m->pf_k, Ly.k, Tp, 0));
        TRY(pf_gemm(m, m->pf_v, Ly.v, Tp, 0));
        TRY(tb_attn_prep_rows_impl(ctx, m->pf_q, m->pf_k, m->pf_v, Ly.qn, Ly.kn, m->pf_qr, Ly.Kq + crow,
                                   Ly.Ks + crow / 32, Ly.Vq + crow, Ly.Vs + crow / 32, m->nHq, m->nKv, hd, T,
                                   c.max_seq, m->pf_pos, c.rope_theta, c.rms_eps));
        TRY(tb_attn_prefill_q8(ctx, m->pf_attn, m->pf_qr, Ly.Kq + crow, Ly.Ks + crow / 32, Ly.Vq + crow,
                               Ly.Vs + crow / 32, T, pos0 + T, m->nHq, m->nKv, hd));
        TRY(pf_quant(m, m->pf_attn, Tp, qN));
        TRY(pf_residual(m, Ly.o, Tp));
        TRY(tb_rmsnorm_q8(ctx, m->pf_x, Ly.ln2, c.rms_eps, m->pf_xq, m->pf_xs, nullptr, Tp, H));
        TRY(pf_gemm(m, m->pf_gate, Ly.gate, Tp, 0));
        TRY(pf_gemm(m, m->pf_gate, Ly.up, Tp, 2));
        TRY(pf_quant(m, m->pf_gate, Tp, I));
        TRY(pf_residual(m, Ly.down, Tp));
    }
    // the last row: final norm + lm_head (linearQ at T = 1) + argmax into the history
    const float* xl = m->pf_x + (T - 1) * H;
    float* lg = m->logits + (int64_t)seq * V;
    if (m->lm.tern) {
        TRY(tb_gemv_tern_wgsl_impl(ctx, 1, &lg, &m->lm.pack, &m->lm.scales, &m->V, xl, m->fnorm, c.rms_eps, H, 1, 0));
    } else if (V >= 16384) {
        TRY(tb_gemv_int4_f32_norm(ctx, lg, xl, m->fnorm, c.rms_eps, m->lm.pack, m->lm.scales, V, H, 1, 0));
    } else {
        TRY(tb_gemv_int4_dp4a(ctx, lg, xl, m->fnorm, c.rms_eps, m->lm.pack, m->lm.scales, V, H, 1, 0));
    }
    if (m->P == 1) {
        TRY(tb_argmax_impl(ctx, lg, V, 1, m->ids + seq, m->amax_part, m->amax_nparts, nullptr, 0, nullptr));
    } else {   // vocab shards: ordered keys of every rank, gathered and merged
        TRY(tb_argmax_impl(ctx, lg, V, 1, nullptr, m->amax_part, m->amax_nparts, m->amax_key + seq,
                           (uint32_t)(m->r * V), nullptr));
        TRY(nccl_check(m, nccl().AllGather(m->amax_key + seq, m->amax_all, 1, ncclUint64, m->comm, ctx->stream),
                       "prefill allgather"));
        TRY(tb_argmax_merge_impl(ctx, m->amax_all, m->P, 1, m->ids + seq, nullptr));
    }
    const int32_t next = (int32_t)(pos0 + T);
    e = cudaMemcpyAsync(m->pos + seq, &next, 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);   // host arrays above are released on return
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "prefill: %s", cudaGetErrorString(e));
    return TB_OK;
}

void release_graph(tb_qwen3* m)
{
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    m->exec = nullptr;
    m->graph = nullptr;
    m->step_direct = false;
}

}  // namespace

extern "C" {

TB_API int tb_qwen3_shard(const tb_qwen3_config* c, int kind, int64_t* row0, int64_t* nrows, int64_t* col0,
                          int64_t* ncols)
{
    if (!c || !row0 || !nrows || !col0 || !ncols) return TB_ERR_INVALID;
    char why[128];
    if (check_config(*c, why, sizeof why)) return TB_ERR_INVALID;
    Slice s{};
    if (shard_of(*c, kind, s, nullptr, nullptr)) return TB_ERR_INVALID;
    *row0 = s.row0; *nrows = s.nrows; *col0 = s.col0; *ncols = s.ncols;
    return TB_OK;
}

TB_API int tb_qwen3_create(tb_ctx* ctx, const tb_qwen3_config* cfg, tb_qwen3** out)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, cfg && out, "null pointer");
    *out = nullptr;
    char why[160];
    if (check_config(*cfg, why, sizeof why)) return tb_fail(ctx, TB_ERR_INVALID, "qwen3 config: %s", why);
    tb_qwen3* m = new (std::nothrow) tb_qwen3();
    if (!m) return TB_ERR_NOMEM;
    m->ctx = ctx;
    m->c = *cfg;
    const tb_qwen3_config& c = m->c;
    m->P = c.tp_size; m->r = c.tp_rank;
    m->nHq = c.n_heads / m->P; m->nKv = c.n_kv_heads / m->P;
    m->I = c.intermediate / m->P; m->V = c.vocab / m->P;
    const int64_t B = c.batch, H = c.hidden, hd = c.head_dim;
    const int64_t kvrow = m->nKv * hd;
    m->L.resize(c.layers);
    int rc = TB_OK;
    auto fail = [&](int code) { tb_qwen3_destroy(m); return code; };
    for (int l = 0; l < c.layers && !rc; l++) {
        Layer& Ly = m->L[l];
        rc = alloc_mat(m, Ly.q, m->nHq * hd, H);
        if (!rc) rc = alloc_mat(m, Ly.k, kvrow, H);
        if (!rc) rc = alloc_mat(m, Ly.v, kvrow, H);
        if (!rc) rc = alloc_mat(m, Ly.o, H, m->nHq * hd);
        if (!rc) rc = alloc_mat(m, Ly.gate, m->I, H);
        if (!rc) rc = alloc_mat(m, Ly.up, m->I, H);
        if (!rc) rc = alloc_mat(m, Ly.down, H, m->I);
        if (!rc) rc = alloc(m, &Ly.ln1, H);
        if (!rc) rc = alloc(m, &Ly.ln2, H);
        if (!rc) rc = alloc(m, &Ly.qn, hd);
        if (!rc) rc = alloc(m, &Ly.kn, hd);
        const size_t cache = (size_t)B * c.max_seq * kvrow;
        if (!rc) rc = alloc(m, &Ly.Kq, cache);
        if (!rc) rc = alloc(m, &Ly.Vq, cache);
        if (!rc) rc = alloc(m, &Ly.Ks, cache / 32);
        if (!rc) rc = alloc(m, &Ly.Vs, cache / 32);
    }
    if (!rc) rc = alloc(m, &m->embed, (size_t)c.vocab * H);
    if (!rc) rc = alloc(m, &m->fnorm, H);
    if (!rc) rc = alloc_mat(m, m->lm, m->V, H);
    if (!rc) rc = alloc(m, &m->x[0], B * H);
    if (!rc) rc = alloc(m, &m->x[1], B * H);
    if (!rc) rc = alloc(m, &m->q, B * m->nHq * hd);
    if (!rc) rc = alloc(m, &m->k, B * kvrow);
    if (!rc) rc = alloc(m, &m->v, B * kvrow);
    if (!rc) rc = alloc(m, &m->attn, B * m->nHq * hd);
    if (!rc) rc = alloc(m, &m->swi, B * m->I);
    if (!rc) rc = alloc(m, &m->logits, B * m->V);
    if (!rc && B >= MMA_MIN_B) {
        const int64_t kmax = std::max<int64_t>({(int64_t)H, m->nHq * hd, m->I});
        rc = alloc(m, &m->mma_act, tb_gemv_mma_act_bytes(kmax, (int)std::min<int64_t>(B, MMA_MAX_B)));
        if (!rc) rc = alloc(m, &m->mma_act2, tb_gemv_mma_act_bytes(m->I, (int)std::min<int64_t>(B, MMA_MAX_B)));
        // row slots past the batch stay zero: producers write only the batch's rows
        if (!rc && (cudaMemsetAsync(m->mma_act, 0, tb_gemv_mma_act_bytes(kmax, (int)std::min<int64_t>(B, MMA_MAX_B)),
                                    ctx->stream) != cudaSuccess ||
                    cudaMemsetAsync(m->mma_act2, 0, tb_gemv_mma_act_bytes(m->I, (int)std::min<int64_t>(B, MMA_MAX_B)),
                                    ctx->stream) != cudaSuccess))
            rc = tb_fail(ctx, TB_ERR_CUDA, "qwen3: clearing the activation buffers failed");
    }
    m->nsplit = tb_attn_auto_nsplit(ctx, c.max_seq, m->nKv * B);
    if (B == 1 && m->P == 1) {
        // one sequence on one GPU: one (kv head, split) unit per SM, the split
        // count the persistent step runs best with (both step kinds use it, so
        // they compute the same bits); under TP both kinds keep the rule above,
        // and the persistent step applies where it gives one 32-key tile per warp
        const long long by_keys = (c.max_seq + 127) / 128;
        // (a long context past the persistent step keeps this count too: three
        // single-stage units an SM with three times the splits measured slower at
        // 32k than one two-stage unit an SM, 571 vs 633 tok/s; with the scores on
        // the tensor cores, five 4-warp single-stage units an SM at 92 splits were
        // still slower, 675 vs 701 tok/s)
        m->nsplit = (int)std::max(1LL, std::min(by_keys, (long long)(ctx->num_sms / m->nKv)));
    }
    if (!rc) rc = alloc(m, &m->qr, B * m->nHq * hd);
    if (!rc) rc = alloc(m, &m->PO, (size_t)B * m->nHq * m->nsplit * hd);
    if (!rc) rc = alloc(m, &m->PML, (size_t)B * m->nHq * m->nsplit * 2);
    if (!rc) rc = alloc(m, &m->counters, (size_t)B * m->nKv);
    if (!rc) rc = alloc(m, &m->ids, B);
    if (!rc) rc = alloc(m, &m->pos, B);
    m->amax_nparts = tb_argmax_parts(ctx, m->V);
    if (!rc) rc = alloc(m, &m->amax_part, (size_t)B * m->amax_nparts);
    if (!rc) rc = alloc(m, &m->amax_key, B);
    if (!rc) rc = alloc(m, &m->amax_all, (size_t)B * m->P);
    if (!rc && m->P > 1) {
        rc = alloc(m, &m->arena, tb_tp_arena_bytes(m->P, B * H));
        if (!rc && cudaMemset(m->arena, 0, tb_tp_arena_bytes(m->P, B * H)) != cudaSuccess) rc = TB_ERR_CUDA;
    }
    if (rc) return fail(rc);
    // counters start at zero; ids/pos start at token 0, position 0
    for (void* p : {(void*)m->counters, (void*)m->ids, (void*)m->pos}) {
        size_t bytes = p == (void*)m->counters ? (size_t)B * m->nKv * 4 : (size_t)B * 4;
        if (cudaMemset(p, 0, bytes) != cudaSuccess) { cudaGetLastError(); return fail(TB_ERR_CUDA); }
    }
    if (cudaStreamCreateWithFlags(&m->cap_stream, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        return fail(TB_ERR_CUDA);
    }
    *out = m;
    return TB_OK;
}

TB_API int tb_qwen3_destroy(tb_qwen3* m)
{
    if (!m) return TB_OK;
    cudaStreamSynchronize(m->ctx->stream);
    release_graph(m);
    if (m->comm) nccl().CommDestroy(m->comm);
    for (int s = 0; s < m->P && s < 8; s++)
        if (s != m->r && m->peer_arena[s]) cudaIpcCloseMemHandle(m->peer_arena[s]);
    for (void* p : m->allocs) cudaFree(p);
    free_prefill(m);
    if (m->step) tb_step_plan_free(m->step);
    if (m->cap_stream) cudaStreamDestroy(m->cap_stream);
    delete m;
    return TB_OK;
}

TB_API int tb_qwen3_set_weight(tb_qwen3* m, int kind, int layer, const uint16_t* bf16, int64_t rows, int64_t cols)
{
    if (!m) return TB_ERR_INVALID;
    tb_ctx* ctx = m->ctx;
    TB_REQUIRE(ctx, bf16 != nullptr, "null weight");
    Slice s{};
    int64_t R = 0, C = 0;
    TB_REQUIRE(ctx, shard_of(m->c, kind, s, &R, &C) == TB_OK, "unknown weight kind %d", kind);
    TB_REQUIRE(ctx, rows == R && cols == C, "weight kind %d: expected %lld x %lld, got %lld x %lld", kind,
               (long long)R, (long long)C, (long long)rows, (long long)cols);
    const bool per_layer = kind >= TB_QW_Q;
    TB_REQUIRE(ctx, !per_layer || (layer >= 0 && layer < m->c.layers), "layer %d out of range", layer);
    release_graph(m);   // weights are baked into the recorded step only by address, but be conservative
    const uint16_t* src = bf16 + s.row0 * C + s.col0;
    auto quant = [&](Mat& w) {
        // _uploadTensor (qwen3.js:3508-3523): the lossless ternary record when the
        // WHOLE tensor is ternary, else int4.  This rank's slice must start and end
        // on 64-column boundaries for the ternary layout; otherwise int4.
        if (m->c.ternary && C % 64 == 0 && s.col0 % 64 == 0 && s.ncols % 64 == 0) {
            int* flag = static_cast<int*>(tb_ctx_scratch(ctx, 256));
            if (!flag) return (int)TB_ERR_NOMEM;
            int h = 1;
            cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int), ctx->stream);
            if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "memset: %s", cudaGetErrorString(e));
            TRY(tb_quant_tern_wgsl_strided_impl(ctx, bf16, C, nullptr, nullptr, R, C, flag));
            e = cudaMemcpyAsync(&h, flag, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream);
            if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
            if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "ternary check: %s", cudaGetErrorString(e));
            if (h == 0) {
                TRY(tb_quant_tern_wgsl_strided_impl(ctx, src, C, w.pack, w.scales, s.nrows, s.ncols, flag));
                w.tern = true;
                w.set = true;
                return (int)TB_OK;
            }
        }
        int rc = tb_quant_int4_strided_impl(ctx, src, C, w.pack, w.scales, s.nrows, s.ncols);
        if (!rc) { w.set = true; w.tern = false; }
        return rc;
    };
    auto f16 = [&](uint16_t* dst) { return tb_convert_bf16_f16(ctx, src, dst, s.nrows * s.ncols); };
    Layer* Ly = per_layer ? &m->L[layer] : nullptr;
    switch (kind) {
    case TB_QW_EMBED: return f16(m->embed);
    case TB_QW_LM_HEAD: return quant(m->lm);
    case TB_QW_FINAL_NORM: return f16(m->fnorm);
    case TB_QW_Q: return quant(Ly->q);
    case TB_QW_K: return quant(Ly->k);
    case TB_QW_V: return quant(Ly->v);
    case TB_QW_O: return quant(Ly->o);
    case TB_QW_GATE: return quant(Ly->gate);
    case TB_QW_UP: return quant(Ly->up);
    case TB_QW_DOWN: return quant(Ly->down);
    case TB_QW_LN_ATTN: return f16(Ly->ln1);
    case TB_QW_LN_MLP: return f16(Ly->ln2);
    case TB_QW_Q_NORM: return f16(Ly->qn);
    case TB_QW_K_NORM: return f16(Ly->kn);
    }
    return tb_fail(ctx, TB_ERR_INVALID, "unknown weight kind %d", kind);
}

// the Mat or f16 buffer behind a weight kind
static int weight_slot(tb_qwen3* m, int kind, int layer, Mat** mat, uint16_t** buf)
{
    *mat = nullptr;
    *buf = nullptr;
    const bool per_layer = kind >= TB_QW_Q;
    if (per_layer && (layer < 0 || layer >= m->c.layers)) return TB_ERR_INVALID;
    Layer* Ly = per_layer ? &m->L[layer] : nullptr;
    switch (kind) {
    case TB_QW_EMBED: *buf = m->embed; break;
    case TB_QW_LM_HEAD: *mat = &m->lm; break;
    case TB_QW_FINAL_NORM: *buf = m->fnorm; break;
    case TB_QW_Q: *mat = &Ly->q; break;
    case TB_QW_K: *mat = &Ly->k; break;
    case TB_QW_V: *mat = &Ly->v; break;
    case TB_QW_O: *mat = &Ly->o; break;
    case TB_QW_GATE: *mat = &Ly->gate; break;
    case TB_QW_UP: *mat = &Ly->up; break;
    case TB_QW_DOWN: *mat = &Ly->down; break;
    case TB_QW_LN_ATTN: *buf = Ly->ln1; break;
    case TB_QW_LN_MLP: *buf = Ly->ln2; break;
    case TB_QW_Q_NORM: *buf = Ly->qn; break;
    case TB_QW_K_NORM: *buf = Ly->kn; break;
    default: return TB_ERR_INVALID;
    }
    return TB_OK;
}

TB_API int tb_qwen3_set_weight_q(tb_qwen3* m, int kind, int layer, int fmt, const void* data, const void* scales,
                                 int64_t rows, int64_t cols)
{
    if (!m) return TB_ERR_INVALID;
    tb_ctx* ctx = m->ctx;
    TB_REQUIRE(ctx, data != nullptr, "null weight");
    Slice s{};
    int64_t R = 0, C = 0;
    TB_REQUIRE(ctx, shard_of(m->c, kind, s, &R, &C) == TB_OK, "unknown weight kind %d", kind);
    TB_REQUIRE(ctx, rows == R && cols == C, "weight kind %d: expected %lld x %lld, got %lld x %lld", kind,
               (long long)R, (long long)C, (long long)rows, (long long)cols);
    Mat* w = nullptr;
    uint16_t* buf = nullptr;
    TB_REQUIRE(ctx, weight_slot(m, kind, layer, &w, &buf) == TB_OK, "layer %d out of range", layer);
    release_graph(m);
    auto copy2d = [&](void* dst, const void* src, size_t spitch, size_t width, size_t height) {
        cudaError_t e = cudaMemcpy2DAsync(dst, width, src, spitch, width, height, cudaMemcpyDefault, ctx->stream);
        if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "set_weight_q copy: %s", cudaGetErrorString(e));
        return (int)TB_OK;
    };
    if (buf) {
        TB_REQUIRE(ctx, fmt == TB_QW_FMT_F16, "weight kind %d is an f16 tensor (fmt %d given)", kind, fmt);
        const char* src = static_cast<const char*>(data) + (size_t)(s.row0 * C + s.col0) * 2;
        return copy2d(buf, src, (size_t)C * 2, (size_t)s.ncols * 2, (size_t)s.nrows);
    }
    TB_REQUIRE(ctx, fmt == TB_QW_FMT_INT4 || fmt == TB_QW_FMT_TERN, "weight kind %d is quantized (fmt %d given)", kind,
               fmt);
    TB_REQUIRE(ctx, scales != nullptr, "null scales");
    const bool tern = fmt == TB_QW_FMT_TERN;
    const int64_t align = tern ? 64 : 32;
    TB_REQUIRE(ctx, C % align == 0 && s.col0 % align == 0 && s.ncols % align == 0,
               "weight kind %d: this shard's columns are not %lld-aligned for the %s layout", kind, (long long)align,
               tern ? "ternary" : "int4");
    const int64_t per = tern ? 4 : 2;   // weights per byte
    const char* ps = static_cast<const char*>(data) + (size_t)(s.row0 * (C / per) + s.col0 / per);
    TRY(copy2d(w->pack, ps, (size_t)(C / per), (size_t)(s.ncols / per), (size_t)s.nrows));
    const char* ss = static_cast<const char*>(scales) + (size_t)(s.row0 * (C / 32) + s.col0 / 32) * 2;
    TRY(copy2d(w->scales, ss, (size_t)(C / 32) * 2, (size_t)(s.ncols / 32) * 2, (size_t)s.nrows));
    w->tern = tern;
    w->set = true;
    return TB_OK;
}

TB_API int tb_qwen3_weight_format(const tb_qwen3* m, int kind, int layer)
{
    if (!m) return -1;
    Mat* w = nullptr;
    uint16_t* buf = nullptr;
    if (weight_slot(const_cast<tb_qwen3*>(m), kind, layer, &w, &buf) != TB_OK) return -1;
    if (buf) return TB_QW_FMT_F16;
    return w->set ? (w->tern ? TB_QW_FMT_TERN : TB_QW_FMT_INT4) : -1;
}

TB_API int tb_qwen3_prefill(tb_qwen3* m, int seq, const uint32_t* ids, int64_t T, int64_t pos0)
{
    if (!m) return TB_ERR_INVALID;
    tb_ctx* ctx = m->ctx;
    const tb_qwen3_config& c = m->c;
    TB_REQUIRE(ctx, ids != nullptr, "null ids");
    TB_REQUIRE(ctx, seq >= 0 && seq < c.batch, "sequence %d out of range", seq);
    TB_REQUIRE(ctx, T >= 1 && pos0 >= 0 && pos0 + T <= c.max_seq && T <= 65535,
               "prefill of %lld tokens at %lld does not fit the %d-row cache", (long long)T, (long long)pos0, c.max_seq);
    if (m->P != 1 && !m->comm)
        return tb_fail(ctx, TB_ERR_UNSUPPORTED,
                       "qwen3 prefill: tensor-parallel prefill uses the NCCL exchange (tb_qwen3_tp_init), tp_size %d",
                       m->P);
    const int64_t hd = c.head_dim, qN = m->nHq * hd, kvN = m->nKv * hd, H = c.hidden;
    const int64_t Ns[4] = {qN, kvN, H, m->I};
    for (int64_t n : Ns)
        if (n % 128)
            return tb_fail(ctx, TB_ERR_UNSUPPORTED, "qwen3 prefill: GEMM needs every projection's size %% 128 == 0 (%lld)",
                           (long long)n);
    return prefill(m, seq, ids, T, pos0);
}

TB_API int tb_qwen3_kv(tb_qwen3* m, int layer, int8_t** Kq, float** Ks, int8_t** Vq, float** Vs)
{
    if (!m) return TB_ERR_INVALID;
    TB_REQUIRE(m->ctx, layer >= 0 && layer < m->c.layers && Kq && Ks && Vq && Vs, "bad layer or null pointer");
    Layer& Ly = m->L[layer];
    *Kq = Ly.Kq; *Ks = Ly.Ks; *Vq = Ly.Vq; *Vs = Ly.Vs;
    return TB_OK;
}

TB_API int tb_qwen3_io(tb_qwen3* m, uint32_t** ids, int32_t** pos, float** logits)
{
    if (!m) return TB_ERR_INVALID;
    if (ids) *ids = m->ids;
    if (pos) *pos = m->pos;
    if (logits) *logits = m->logits;
    return TB_OK;
}

TB_API int tb_nccl_unique_id(void* out128)
{
    if (!out128) return TB_ERR_INVALID;
    NcclApi& api = nccl();
    if (!api.ok) return TB_ERR_UNSUPPORTED;
    ncclUniqueId id;
    if (api.GetUniqueId(&id) != ncclSuccess) return TB_ERR_CUDA;
    memcpy(out128, &id, sizeof id);
    return TB_OK;
}

TB_API int tb_qwen3_tp_init(tb_qwen3* m, const void* unique_id128)
{
    if (!m) return TB_ERR_INVALID;
    tb_ctx* ctx = m->ctx;
    TB_REQUIRE(ctx, unique_id128 != nullptr, "null unique id");
    if (m->P == 1) return TB_OK;
    NcclApi& api = nccl();
    if (!api.ok) return tb_fail(ctx, TB_ERR_UNSUPPORTED, "NCCL unavailable: %s", api.why.c_str());
    TB_REQUIRE(ctx, m->comm == nullptr, "tensor parallelism already initialised");
    ncclUniqueId id;
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
    memcpy(&id, unique_id128, sizeof id);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ctx->device);
    ncclResult_t r = api.CommInitRank(&m->comm, m->P, id, m->r);
    cudaSetDevice(prev);
    if (r != ncclSuccess) {
        m->comm = nullptr;
        return tb_fail(ctx, TB_ERR_CUDA, "ncclCommInitRank: %s", api.GetErrorString(r));
    }
    return TB_OK;
}

TB_API int tb_qwen3_tp_handle(tb_qwen3* m, void* out64)
{
    if (!m || !out64) return TB_ERR_INVALID;
    TB_REQUIRE(m->ctx, m->P > 1 && m->arena, "tp_handle: model is not tensor-parallel");
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle is 64 bytes");
    cudaIpcMemHandle_t h;
    cudaError_t e = cudaIpcGetMemHandle(&h, m->arena);
    if (e != cudaSuccess) return tb_fail(m->ctx, TB_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
    memcpy(out64, &h, sizeof h);
    return TB_OK;
}

TB_API int tb_qwen3_tp_connect(tb_qwen3* m, const void* handles)
{
    if (!m || !handles) return TB_ERR_INVALID;
    tb_ctx* ctx = m->ctx;
    TB_REQUIRE(ctx, m->P > 1 && m->P <= 8 && m->arena, "tp_connect: model is not tensor-parallel (2..8 ranks)");
    TB_REQUIRE(ctx, !m->p2p, "tp_connect: already connected");
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(ctx->device);
    int rc = TB_OK;
    for (int s = 0; s < m->P && !rc; s++) {
        if (s == m->r) { m->peer_arena[s] = m->arena; continue; }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char*>(handles) + 64 * s, sizeof h);
        void* p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) rc = tb_fail(ctx, TB_ERR_CUDA, "cudaIpcOpenMemHandle(rank %d): %s", s, cudaGetErrorString(e));
        else m->peer_arena[s] = static_cast<char*>(p);
    }
    cudaSetDevice(prev);
    if (rc) {
        for (int s = 0; s < m->P; s++)
            if (s != m->r && m->peer_arena[s]) { cudaIpcCloseMemHandle(m->peer_arena[s]); m->peer_arena[s] = nullptr; }
        return rc;
    }
    release_graph(m);
    m->p2p = true;
    return TB_OK;
}

// Recovery after a device-side wait gave up under tensor parallelism: the
// exchanges' epochs may disagree between the ranks from then on, so the rank
// poisoned itself and its exchanges refuse to run.  This clears this rank's
// exchange arena (partials, flags, step counter, poison word, inbox), the
// persistent step's barrier and abort words and the attention split counters,
// and waits for it.  Contract: call it on EVERY rank, after every rank's stream
// is idle (no step in flight anywhere) and behind a host barrier, and let no
// rank step again until every rank has returned from it (a second barrier).
TB_API int tb_qwen3_tp_reset(tb_qwen3* m)
{
    if (!m) return TB_ERR_INVALID;
    tb_ctx* ctx = m->ctx;
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e == cudaSuccess && m->arena)
        e = cudaMemsetAsync(m->arena, 0, tb_tp_arena_bytes(m->P, (int64_t)m->c.batch * m->c.hidden), ctx->stream);
    if (e == cudaSuccess && m->step_ctrl) e = cudaMemsetAsync(m->step_ctrl, 0, 256 * 4, ctx->stream);
    if (e == cudaSuccess && m->counters)
        e = cudaMemsetAsync(m->counters, 0, (size_t)m->c.batch * m->nKv * sizeof(unsigned), ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "tp_reset: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_qwen3_decode_step(tb_qwen3* m)
{
    if (!m) return TB_ERR_INVALID;
    tb_ctx* ctx = m->ctx;
    TB_REQUIRE(ctx, m->P == 1 || m->p2p || m->comm != nullptr,
               "tensor parallel model needs tb_qwen3_tp_connect (or tb_qwen3_tp_init) first");
    for (const Layer& Ly : m->L)
        TB_REQUIRE(ctx, Ly.q.set && Ly.k.set && Ly.v.set && Ly.o.set && Ly.gate.set && Ly.up.set && Ly.down.set,
                   "a projection weight was never set");
    TB_REQUIRE(ctx, m->lm.set, "lm_head weight was never set");
    if (!m->exec && !m->step_direct) {
        // AUTO takes the persistent kernel wherever it applies: on one GPU, and under
        // TP over peer memory, where its in-kernel packet exchange measured faster
        // than the multi-kernel step (1016 vs 841 tok/s at TP = 2)
        const bool want = m->step_mode == TB_QW_STEP_PERSISTENT || m->step_mode == TB_QW_STEP_AUTO;
        const bool pers = want && persistent_ok(m);
        if (m->step_mode == TB_QW_STEP_PERSISTENT && !pers)
            return tb_fail(ctx, TB_ERR_UNSUPPORTED,
                           "persistent decode step needs batch 1, one GPU or tensor parallel over peer memory "
                           "(tp_connect), layer weights all int4 or all ternary and sizes it supports");
        m->step_kind = pers ? TB_QW_STEP_PERSISTENT : TB_QW_STEP_KERNELS;
        // record the step once on a private stream, after everything queued so far
        cudaStream_t user = ctx->stream;
        cudaEvent_t ev;
        cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
        cudaEventRecord(ev, user);
        cudaStreamWaitEvent(m->cap_stream, ev, 0);
        cudaEventDestroy(ev);
        ctx->stream = m->cap_stream;
        cudaError_t e = cudaStreamBeginCapture(m->cap_stream, cudaStreamCaptureModeThreadLocal);
        int rc = e == cudaSuccess ? (pers ? issue_step_persistent(m) : issue_step(m))
                                  : tb_fail(ctx, TB_ERR_CUDA, "begin capture: %s", cudaGetErrorString(e));
        cudaGraph_t g = nullptr;
        cudaError_t e2 = cudaStreamEndCapture(m->cap_stream, &g);
        ctx->stream = user;
        if (!rc && e2 != cudaSuccess) rc = tb_fail(ctx, TB_ERR_CUDA, "end capture: %s", cudaGetErrorString(e2));
        if (!rc) {
            e = cudaGraphInstantiate(&m->exec, g, 0);
            if (e != cudaSuccess) rc = tb_fail(ctx, TB_ERR_CUDA, "instantiate: %s", cudaGetErrorString(e));
        }
        if (rc && pers) {
            // a driver that cannot capture the cooperative launch: launch the
            // persistent step directly on every call (the graph of the head
            // alone is kept for launch counting)
            if (g) cudaGraphDestroy(g);
            g = nullptr;
            cudaGetLastError();
            ctx->stream = m->cap_stream;
            e = cudaStreamBeginCapture(m->cap_stream, cudaStreamCaptureModeThreadLocal);
            rc = e == cudaSuccess ? issue_head(m, 0) : TB_ERR_CUDA;
            e2 = cudaStreamEndCapture(m->cap_stream, &g);
            ctx->stream = user;
            if (rc || e2 != cudaSuccess) {
                if (g) cudaGraphDestroy(g);
                cudaGetLastError();
                return tb_fail(ctx, TB_ERR_CUDA, "decode step: cannot record the step");
            }
            m->graph = g;
            m->step_direct = true;
            tb_fail(ctx, TB_OK, "");
            return issue_step_persistent(m);
        }
        if (rc) {
            if (g) cudaGraphDestroy(g);
            m->exec = nullptr;
            cudaGetLastError();
            return rc;
        }
        m->graph = g;
    }
    if (m->step_direct) return issue_step_persistent(m);
    cudaError_t e = cudaGraphLaunch(m->exec, ctx->stream);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "graph launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_qwen3_set_step_mode(tb_qwen3* m, int mode)
{
    if (!m) return TB_ERR_INVALID;
    TB_REQUIRE(m->ctx, mode == TB_QW_STEP_AUTO || mode == TB_QW_STEP_KERNELS || mode == TB_QW_STEP_PERSISTENT,
               "step mode %d", mode);
    m->step_mode = mode;
    release_graph(m);
    return TB_OK;
}

TB_API int tb_qwen3_step_kind(tb_qwen3* m)
{
    return m ? m->step_kind : 0;
}

// Phase trace of the persistent kernel: trace (device, u64 [SMs][1 + 38 * layers])
// receives %globaltimer stamps from every later launch (null: off).  Per CTA:
// kernel start, then per layer and phase (qkv, attention, o, gate/up, down):
// weights ready, activation row loaded, activation staged, phase done, barrier
// passed; then per layer 8 stamps of the CTA's first attention unit; then per
// layer and phase the moment its next-buffer request was issued.
TB_API int tb_qwen3_step_trace(tb_qwen3* m, void* trace)
{
    if (!m) return TB_ERR_INVALID;
    m->step_trace = trace;
    release_graph(m);
    return TB_OK;
}

// The persistent kernel alone (embed + every layer, no lm_head / argmax) on the
// context's stream, for timing it apart from the step's head; ids and pos are
// left as they are, so repeated calls recompute the same position.
TB_API int tb_qwen3_step_layers(tb_qwen3* m)
{
    if (!m) return TB_ERR_INVALID;
    TB_REQUIRE(m->ctx, m->step_kind == TB_QW_STEP_PERSISTENT && m->step && m->step_layers,
               "step_layers: the recorded step is not the persistent kernel");
    const tb_step_io io = step_io(m);
    return tb_step_launch(m->ctx, m->step, &io);
}

TB_API int tb_qwen3_launches_per_step(tb_qwen3* m, int* kernels, int* collectives)
{
    if (!m || !kernels) return TB_ERR_INVALID;
    if (!m->graph) return tb_fail(m->ctx, TB_ERR_INVALID, "step not recorded yet");
    // kernel nodes of the recorded step; NCCL's own kernels (one per collective)
    // are among them, and are reported apart
    size_t n = 0;
    if (cudaGraphGetNodes(m->graph, nullptr, &n) != cudaSuccess) return TB_ERR_CUDA;
    std::vector<cudaGraphNode_t> nodes(n);
    if (cudaGraphGetNodes(m->graph, nodes.data(), &n) != cudaSuccess) return TB_ERR_CUDA;
    int k = 0;
    for (auto nd : nodes) {
        cudaGraphNodeType t;
        if (cudaGraphNodeGetType(nd, &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) k++;
    }
    const int coll = m->ncoll;      // each NCCL call records one kernel node
    *kernels = k - coll;
    if (collectives) *collectives = coll;
    return TB_OK;
}

}  // extern "C"
