// tb_tp.cu -- tensor-parallel exchanges of the decode step over NVLink peer
// memory: one kernel per exchange, no library collective.
//
// Every rank owns a small "exchange arena" in its own HBM, mapped into every
// other rank with CUDA IPC:
//   part[2][n]   f32 partial products of the row-split o / down GEMVs, double
//                buffered by exchange parity
//   keys[16]     u64 argmax keys of this rank's vocab shard (value, index)
//   flag[P]      u32 epochs written by the peers ("my part for epoch e is ready")
//   flag2[P]     the same for the argmax keys
//   step         u32 steps completed (local)
//   poison       u32 set when any exchange wait of this rank gave up (see below)
//   inbox[8][2][n] u64 packets of the persistent decode step's exchanges
//                (tb_step.cu): (epoch << 32) | f32 bits of row i of rank s's
//                partial, written by rank s with one 8-byte store, parity 2
// An exchange: after the producing kernel finished (griddepcontrol.wait), rank
// r stores epoch e into flag[r] of every rank with a system-scope release,
// waits until its own flag[s] >= e for every s (acquire, bounded), then reads
// the P partials straight from the peers' arenas and adds them in rank order,
// so every rank computes the identical sum.  Epochs e = step * nx + i + 1 grow
// monotonically, so the flags never need clearing and the recorded step can be
// replayed.  Reuse is safe with two part buffers: rank r overwrites
// part[parity(e)] at exchange e+2 only after every peer signalled e+1, which a
// peer does only after it finished reading exchange e.
//
// Poison: epochs stay in step only while every rank ran every exchange.  A wait
// that gives up (a peer died, or ran more than ~1 s late) leaves the ranks at
// different epochs, after which a later exchange could accept a stale flag or
// packet.  So a rank whose wait gave up sets its poison word, and every
// exchange (these kernels and the persistent step) starts by reading it: when
// set, the exchange does nothing but record ERR_TP_POISONED in the device error
// word.  tb_qwen3_tp_reset clears the arena on every rank (all ranks idle,
// behind a host barrier) and the epochs restart together from zero.
#include "tb_internal.h"

namespace {

constexpr int TP_MAX = 8;
constexpr long long TP_WAIT_LIMIT = 1LL << 22;    // polls (sleeping 64+ ns after the first 4096): ~1 s
constexpr int ERR_TP_WAIT = 0x7a01;
constexpr int ERR_TP_POISONED = 0x7a02;

struct TpArgs {
    const float* part[TP_MAX];      // this exchange's part buffer on every rank
    unsigned* peer_flag[TP_MAX];    // &flag[r] on every rank (where this rank signals)
    const unsigned* my_flag;        // flag[0..P) of this rank
    const unsigned* step;           // steps completed
    unsigned* poison;               // this rank's poison word
    float* x;                       // residual, updated in place: x += sum_s part_s
    int n, P, xi, nx;
    int* err;
};

// The CTA-wide poison check every exchange starts with: true when an earlier
// wait of this rank gave up (the error word is set once, by CTA 0).
__device__ __forceinline__ bool tp_poisoned(const unsigned* poison, int* err)
{
    const bool p = __syncthreads_or(threadIdx.x == 0 && *reinterpret_cast<const volatile unsigned*>(poison) != 0u);
    if (p && blockIdx.x == 0 && threadIdx.x == 0) atomicCAS(err, 0, ERR_TP_POISONED);   // keeps a first error
    return p;
}

// signal flag slot of every rank, then wait for every rank's signal (bounded);
// false (for the whole CTA) when a wait gave up, which poisons this rank
__device__ __forceinline__ bool tp_signal_wait(unsigned* const* peer_flag, const unsigned* my_flag, int P, unsigned e,
                                               bool signal, int* err, unsigned* poison)
{
    if (signal && threadIdx.x < P) st_release_sys(peer_flag[threadIdx.x], e);
    bool gave_up = false;
    if (threadIdx.x < P) {
        long long it = 0;
        while ((int)(ld_acquire_sys(my_flag + threadIdx.x) - e) < 0) {
            if (++it > TP_WAIT_LIMIT) {
                atomicExch(err, ERR_TP_WAIT);
                atomicExch(poison, 1u);
                gave_up = true;
                break;
            }
            if (it > 4096) __nanosleep(64);   // a healthy peer answers within the first polls
        }
    }
    return !__syncthreads_or(gave_up);
}

// x[i] += part_0[i] + part_1[i] + ... (rank order), float4 per thread
__global__ void __launch_bounds__(256) k_tp_allreduce(const TpArgs a)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    if (tp_poisoned(a.poison, a.err)) return;
    const unsigned e = *a.step * (unsigned)a.nx + (unsigned)a.xi + 1u;
    if (!tp_signal_wait(a.peer_flag, a.my_flag, a.P, e, blockIdx.x == 0, a.err, a.poison)) return;
    const int n4 = a.n >> 2;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
        float4 v = reinterpret_cast<const float4*>(a.x)[i];
        for (int s = 0; s < a.P; s++) {
            const float4 p = ld_volatile_f4(a.part[s] + 4 * i);
            v.x += p.x; v.y += p.y; v.z += p.z; v.w += p.w;
        }
        reinterpret_cast<float4*>(a.x)[i] = v;
    }
}

struct TpKeyArgs {
    const unsigned long long* keys[TP_MAX];   // every rank's argmax keys
    unsigned* peer_flag2[TP_MAX];
    const unsigned* my_flag2;
    unsigned* step;                           // incremented here: the last kernel of a step
    unsigned* poison;
    uint32_t* ids;
    int32_t* pos;
    int rows, P;
    int* err;
};

// the argmax over all vocab shards: the largest key (value, then lower global
// index) of the P ranks; ids/pos updated, step counter advanced
__global__ void __launch_bounds__(32) k_tp_argmax_merge(const TpKeyArgs a)
{
    tb_pdl_wait();
    tb_pdl_trigger();
    if (tp_poisoned(a.poison, a.err)) return;
    const unsigned e = *a.step + 1u;
    if (!tp_signal_wait(a.peer_flag2, a.my_flag2, a.P, e, true, a.err, a.poison)) return;
    for (int row = threadIdx.x; row < a.rows; row += blockDim.x) {
        unsigned long long best = 0ull;
        for (int s = 0; s < a.P; s++) {
            const unsigned long long k = *reinterpret_cast<const volatile unsigned long long*>(a.keys[s] + row);
            best = k > best ? k : best;
        }
        a.ids[row] = 0xffffffffu - (uint32_t)(best & 0xffffffffu);
        a.pos[row] += 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) *a.step = e;
}

}  // namespace

// ---- arena layout -----------------------------------------------------------
static size_t tp_base_bytes(int64_t n)
{
    const size_t part = ((size_t)2 * n * 4 + 255) & ~size_t(255);
    return part + 16 * 8 + 2 * TP_MAX * 4 + 256;
}

size_t tb_tp_arena_bytes(int P, int64_t n)
{
    (void)P;
    return ((tp_base_bytes(n) + 255) & ~size_t(255)) + (size_t)TB_TP_MAX * 2 * n * 8;
}

unsigned long long* tb_tp_arena_step_inbox(char* base, int64_t n)
{
    return reinterpret_cast<unsigned long long*>(base + ((tp_base_bytes(n) + 255) & ~size_t(255)));
}

void tb_tp_arena_layout(char* base, int64_t n, float** part, unsigned long long** keys, unsigned** flag,
                        unsigned** flag2, unsigned** step)
{
    const size_t part_b = ((size_t)2 * n * 4 + 255) & ~size_t(255);
    *part = reinterpret_cast<float*>(base);
    *keys = reinterpret_cast<unsigned long long*>(base + part_b);
    *flag = reinterpret_cast<unsigned*>(base + part_b + 16 * 8);
    *flag2 = *flag + TP_MAX;
    *step = *flag2 + TP_MAX;      // step[1] is the poison word
}

// x += sum over ranks of part (exchange xi of nx per step, parity buffer
// (xi + 1) & 1 of every rank's arena)
int tb_tp_allreduce_impl(tb_ctx* ctx, char* const* arenas, int P, int r, int64_t n, float* x, int xi, int nx)
{
    TB_REQUIRE(ctx, P >= 2 && P <= TP_MAX && n % 4 == 0 && TB_ALIGNED(x, 16), "tp allreduce: bad arguments");
    TpArgs a{};
    for (int s = 0; s < P; s++) {
        float* part; unsigned long long* keys; unsigned *flag, *flag2, *step;
        tb_tp_arena_layout(arenas[s], n, &part, &keys, &flag, &flag2, &step);
        a.part[s] = part + (size_t)((xi + 1) & 1) * n;
        a.peer_flag[s] = flag + r;
        if (s == r) { a.my_flag = flag; a.step = step; a.poison = step + 1; }
    }
    a.x = x; a.n = (int)n; a.P = P; a.xi = xi; a.nx = nx; a.err = ctx->dev_error;
    const int grid = (int)std::min<int64_t>(std::max<int64_t>(1, (n / 4 + 255) / 256), 32);
    cudaError_t e = tb_launch(ctx, k_tp_allreduce, dim3(grid), dim3(256), 0, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "tp allreduce launch: %s", cudaGetErrorString(e));
    return TB_OK;
}

int tb_tp_argmax_merge_impl(tb_ctx* ctx, char* const* arenas, int P, int r, int64_t n, int rows, uint32_t* ids,
                            int32_t* pos)
{
    TB_REQUIRE(ctx, P >= 2 && P <= TP_MAX && rows >= 1 && rows <= 16, "tp argmax: bad arguments");
    TpKeyArgs a{};
    for (int s = 0; s < P; s++) {
        float* part; unsigned long long* keys; unsigned *flag, *flag2, *step;
        tb_tp_arena_layout(arenas[s], n, &part, &keys, &flag, &flag2, &step);
        a.keys[s] = keys;
        a.peer_flag2[s] = flag2 + r;
        if (s == r) { a.my_flag2 = flag2; a.step = step; a.poison = step + 1; }
    }
    a.ids = ids; a.pos = pos; a.rows = rows; a.P = P; a.err = ctx->dev_error;
    cudaError_t e = tb_launch(ctx, k_tp_argmax_merge, dim3(1), dim3(32), 0, a);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "tp argmax launch: %s", cudaGetErrorString(e));
    return TB_OK;
}
