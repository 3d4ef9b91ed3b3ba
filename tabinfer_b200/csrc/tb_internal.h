// tb_internal.h -- library-internal entry points shared between translation
// units (not part of the C ABI): the unchecked launch paths behind the public
// calls, for callers that own their buffers (the model runner records them into
// one CUDA graph, so nothing may allocate).
#pragma once
#include <cuda.h>
#include "tb_common.cuh"

// 2-D TMA tensor map over a row-major [rows][cols] matrix of esize-byte elements,
// box_cols x box_rows boxes (cuTensorMapEncodeTiled from the driver)
int tb_encode_2d(tb_ctx* ctx, CUtensorMap* map, const void* base, CUtensorMapDataType dt, int esize, int64_t cols,
                 int64_t rows, int box_cols, int box_rows, CUtensorMapSwizzle swz);

int tb_gemv_dp4a_impl(tb_ctx* ctx, int count, float* const* ys, const uint32_t* const* packs,
                      const uint16_t* const* scales, const int64_t* Ns, const float* x, const uint16_t* normw,
                      float eps, int64_t K, int batch, int acc);
// decode GEMVs over 2..16 rows on the tensor cores (one weight read): quantize
// x into buf (tb_gemv_mma_act_bytes bytes; quantize = false: buf already holds the
// rows, written by their producer) and run `count` matrices, or gate/up with silu
// when gateup (count 2, ys[0] the output; with obuf, swi is written QUANTQ8'd into
// obuf for a next GEMV of kind otern instead of as f32)
size_t tb_gemv_mma_act_bytes(int64_t K, int batch);
bool tb_gemv_mma_fits(int64_t K, const int64_t* Ns, int count, int batch);
int tb_gemv_mma_impl(tb_ctx* ctx, int count, float* const* ys, const uint32_t* const* packs,
                     const uint16_t* const* scales, const int64_t* Ns, const float* x, const uint16_t* normw,
                     float eps, int64_t K, int batch, int acc, bool tern, bool gateup, void* buf,
                     bool quantize = true, void* obuf = nullptr, bool otern = false);
int tb_gemv_f32_impl(tb_ctx* ctx, float* y, const float* x, const uint32_t* pack, const uint16_t* scales,
                     int64_t N, int64_t K, int batch, int acc);
int tb_gemv_tern_impl(tb_ctx* ctx, float* out, const uint8_t* codes, const float* scales, const int8_t* act,
                      const int32_t* xsum, int64_t N, int64_t K, int batch, const float* act_scale);
// wasm: the WASM engine's quantize (asc = amax/127, nearest-even, asc stored)
int tb_quant_act_impl(tb_ctx* ctx, const float* x, int8_t* act, int32_t* xsum, float* scale, int64_t T, int64_t K,
                      bool wasm = false);

// split-KV decode attention over `batch` sequences; sequence b's cache starts
// cache_rows rows after sequence b-1's; with dpos, S_b = dpos[b] + 1 is read on
// the device.  PO/PML: batch*nHq*nsplit*(hd, 2) floats; counters: batch*nKv
// words that are zero between calls.  early: dpos and every cache row below
// S_b - 1 are complete before the preceding kernel in the stream runs (only
// that kernel may write row S_b - 1), so the first tiles are fetched before
// griddepcontrol.wait.
// mxa / mxk (optional): the outputs also QUANTQ8'd in the tensor-core GEMVs' fragment
// order, mts row slots (sequence = slot), for int4 or (mtern) ternary weights; needs
// (nHq/nKv)·hd a multiple of 128.
int tb_attn_decode_impl(tb_ctx* ctx, float* out, const float* qr, const int8_t* Kq, const float* Ks,
                        const int8_t* Vq, const float* Vs, int64_t S, int64_t nHq, int64_t nKv, int64_t hd,
                        int nsplit, float* PO, float* PML, unsigned* counters, int64_t batch = 1,
                        int64_t cache_rows = 0, const int32_t* dpos = nullptr, bool early = false,
                        unsigned char* mxa = nullptr, uint2* mxk = nullptr, int mts = 0, bool mtern = false);
int tb_attn_auto_nsplit(tb_ctx* ctx, int64_t S, int64_t nKv);
// two-stage argmax of `rows` rows of n; part holds rows*nparts keys.  out gets
// the index + idx_base, out_key the ordered key (for tb_argmax_merge_impl),
// pos_inc[row] += 1 when given.
int tb_argmax_impl(tb_ctx* ctx, const float* x, int64_t n, int64_t rows, uint32_t* out, unsigned long long* part,
                   int nparts, unsigned long long* out_key, uint32_t idx_base, int32_t* pos_inc);
int tb_argmax_parts(tb_ctx* ctx, int64_t n);
int tb_argmax_merge_impl(tb_ctx* ctx, const unsigned long long* keys, int nshard, int rows, uint32_t* out,
                         int32_t* pos_inc);

// int4 G32 quantization of an N x K slice with source row stride ld (elements)
int tb_quant_int4_strided_impl(tb_ctx* ctx, const uint16_t* w, int64_t ld, uint32_t* pack, uint16_t* scales,
                               int64_t N, int64_t K);

// tensor-parallel exchanges over IPC-mapped peer arenas (tb_tp.cu)
size_t tb_tp_arena_bytes(int P, int64_t n);
// the persistent decode step's exchange inbox in an arena: u64
// [TB_TP_MAX][2][n] packets (epoch << 32 | f32 bits), row s written by rank s
// (zero at creation and after tb_qwen3_tp_reset)
constexpr int TB_TP_MAX = 8;
unsigned long long* tb_tp_arena_step_inbox(char* base, int64_t n);
void tb_tp_arena_layout(char* base, int64_t n, float** part, unsigned long long** keys, unsigned** flag,
                        unsigned** flag2, unsigned** step);
int tb_tp_allreduce_impl(tb_ctx* ctx, char* const* arenas, int P, int r, int64_t n, float* x, int xi, int nx);
int tb_tp_argmax_merge_impl(tb_ctx* ctx, char* const* arenas, int P, int r, int64_t n, int rows, uint32_t* ids,
                            int32_t* pos);

// prefill GEMM Y (+)= f16(X) . f16(deq(W))^T on tcgen05 (M % 128, N % 256, K % 64);
// X's f16 copy and any split-K partials live in context scratch
int tb_gemm_int4_impl(tb_ctx* ctx, float* y, const void* x, int x_bf16, const uint32_t* pack, const uint16_t* scales,
                      int64_t M, int64_t N, int64_t K, int acc);
// the same GEMM for ternary weights (WebGPU layout) against QUANTQ8T int8 rows
int tb_gemm_tern_wgsl_impl(tb_ctx* ctx, float* y, const int8_t* xq, const float* xs, const uint32_t* pack,
                           const uint16_t* scales, int64_t M, int64_t N, int64_t K, int acc);
// quantQ8 (+ optional RMSNorm) and the ternary (WebGPU layout) GEMV, batch 1..8
int tb_gemv_tern_wgsl_impl(tb_ctx* ctx, int count, float* const* ys, const uint32_t* const* packs,
                           const uint16_t* const* scales, const int64_t* Ns, const float* x, const uint16_t* normw,
                           float eps, int64_t K, int batch, int acc);
// per-32 int8 quantization of T rows (QUANTQ8 / QUANTQ8T)
int tb_quant_q8_impl(tb_ctx* ctx, const float* x, int8_t* xq, float* xs, int32_t* xsum16, int64_t T, int64_t K);
// ternary (WebGPU layout) detect + pack of an N x K slice, rows ld elements apart;
// flag |= 1 when not ternary (zero it first); pack == nullptr checks only
int tb_quant_tern_wgsl_strided_impl(tb_ctx* ctx, const uint16_t* w, int64_t ld, uint32_t* pack, uint16_t* scales,
                                    int64_t N, int64_t K, int* flag);
// gemmDP4A on the tensor cores (QUANTQ8T rows x int4); epilogue 0 store, 1 add, 2 SwiGLU
int tb_gemm_q8_int4_impl(tb_ctx* ctx, float* y, const int8_t* xq, const float* xs, const uint32_t* pack,
                         const uint16_t* scales, int64_t M, int64_t N, int64_t K, int epilogue);
// attention prep of T tokens of one sequence (prefill): cache row dpos[t] of one cache
int tb_attn_prep_rows_impl(tb_ctx* ctx, const float* q, const float* k, const float* v, const uint16_t* qw16,
                           const uint16_t* kw16, float* qr, int8_t* Kq, float* Ks, int8_t* Vq, float* Vs, int64_t nHq,
                           int64_t nKv, int64_t hd, int64_t T, int64_t cache_rows, const int32_t* dpos, float theta,
                           float eps);
// the reference's integer prefill GEMM (gemmDP4A / gemmTern) with exact per-32-group
// int8 sums (tb_gemm_dp4.cu); M % 128, N % 128, K % 128; epilogue 0 store, 1 add, 2 SwiGLU
int tb_gemm_dp4_impl(tb_ctx* ctx, float* y, const int8_t* xq, const float* xs, const uint32_t* pack,
                     const uint16_t* scales, int64_t M, int64_t N, int64_t K, int epilogue, bool tern);
// the same GEMM on the warp-level tensor-core MMA (mma.sync), kept as a second
// implementation of the identical arithmetic (bit-equal outputs)
int tb_gemm_dp4_warp_impl(tb_ctx* ctx, float* y, const int8_t* xq, const float* xs, const uint32_t* pack,
                          const uint16_t* scales, int64_t M, int64_t N, int64_t K, int epilogue, bool tern);

// the decode step as one persistent kernel (tb_step.cu): batch 1, one GPU
struct tb_step_plan;
struct tb_step_io {
    const void* layers;            // device array of the per-layer records (tb_step_layer_fill)
    float eps, theta;
    const uint32_t* ids;
    const int32_t* pos;
    const uint16_t* embed;
    float *x, *q, *k, *v, *qr, *attn, *swi, *PO, *PML;
    unsigned char* attnq;          // nHq*hd/32 * 40 bytes: the attention output in the GEMV activation layout
    unsigned* counters;            // [nKv] attention split arrivals, zero between steps
    unsigned* ctrl;                // [256] zero-initialised: grid barrier counter (u64 at word 64), abort word (128)
    unsigned* head_cnt;            // [layers][kv heads] phase-A arrival counters (every launch zeroes them)
    unsigned long long* pk;        // [hidden] phase-boundary packets of x after o (zeroed at creation)
    void* trace;                   // optional: u64 [grid][1 + 38 * layers] %globaltimer stamps
    // tensor parallel over peer memory (P > 1): every rank's exchange-arena part
    // buffers (f32 [2][hidden]) and step flags, mapped here; this rank's index
    int P, rank;
    float* xpart;                              // this rank's part[2][hidden]
    unsigned long long* tp_inbox[TB_TP_MAX];   // every rank's inbox [TB_TP_MAX][2][hidden]
    unsigned* tp_poison;                       // this rank's poison word (step[1] of its arena)
};
// tern: the layer weights are ternary (WebGPU layout) instead of int4 G32
// P > 1: this rank's shard of a tensor-parallel model (nHq, nKv, I per rank)
int tb_step_plan_make(tb_ctx* ctx, int L, int H, int nHq, int nKv, int hd, int I, int nsplit, int max_seq,
                      int tern, int P, tb_step_plan** out);
void tb_step_plan_free(tb_step_plan* p);
size_t tb_step_plan_smem(const tb_step_plan* p);
int tb_step_launch(tb_ctx* ctx, tb_step_plan* p, const tb_step_io* io);
size_t tb_step_layer_bytes();
void tb_step_layer_fill(void* dst, const uint32_t* const* packs, const uint16_t* const* scales, const uint16_t* ln1,
                        const uint16_t* ln2, const uint16_t* qn, const uint16_t* kn, int8_t* Kq, float* Ks, int8_t* Vq,
                        float* Vs);
