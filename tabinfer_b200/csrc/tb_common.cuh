// tb_common.cuh -- shared device helpers and the context object behind the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <algorithm>
#include <string>

#include "../../include/tabinfer_b200.h"

struct tb_ctx {
    int device = 0;
    int num_sms = 148;
    cudaStream_t stream = nullptr;      // stream all calls are ordered on
    cudaStream_t own_stream = nullptr;  // created by tb_ctx_create, destroyed with the context
    std::string last_error;
    int* dev_error = nullptr;           // device word written by bounded waits that gave up
    // split-arrival counters of the decode attention, one per kv head; zero
    // between calls (the last split of a head resets its counter)
    unsigned* attn_counters = nullptr;
    // scratch for the combined calls (quantized activations); grown on demand, never shrunk
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    bool pdl = true;                    // launch with programmatic dependent launch
};

// ---------------------------------------------------------------------------
// host-side error plumbing
// ---------------------------------------------------------------------------
int tb_fail(tb_ctx* ctx, int code, const char* fmt, ...);
int tb_check_launch(tb_ctx* ctx, const char* what);
void* tb_ctx_scratch(tb_ctx* ctx, size_t bytes);   // nullptr on failure (error recorded)

#define TB_REQUIRE(ctx, cond, ...) \
    do { if (!(cond)) return tb_fail((ctx), TB_ERR_INVALID, __VA_ARGS__); } while (0)
#define TB_ALIGNED(p, a) ((((uintptr_t)(p)) & ((a) - 1)) == 0)

// Launch helper: every kernel goes through this so programmatic dependent
// launch (PDL) is applied uniformly.  Kernels call tb_pdl_wait() before they
// read anything a previous kernel in the stream wrote.
template <typename... KArgs, typename... Args>
static inline cudaError_t tb_launch(tb_ctx* ctx, void (*kern)(KArgs...), dim3 grid, dim3 block,
                                    size_t smem, Args... args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = ctx->pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
// Wait until the grids this one depends on have finished and their writes are
// visible (griddepcontrol.wait); a no-op when launched without PDL.
__device__ __forceinline__ void tb_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next grid in the stream to begin launching (its pre-wait prologue).
__device__ __forceinline__ void tb_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float tb_h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ uint4 ldg_stream_v4(const void* p)
{
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ uint16_t ldg_u16(const uint16_t* p)
{
    unsigned short r;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

__device__ __forceinline__ int dp4a_s8(int a, int b, int c) { return __dp4a(a, b, c); }

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// packed f32x2 arithmetic (sm_100): two IEEE round-to-nearest lanes per instruction
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c)
{
    float2 d;
    asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2,%3};\n mov.b64 rb, {%4,%5};\n mov.b64 rc, {%6,%7};\n"
        " fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0,%1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b)
{
    float2 d;
    asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2,%3};\n mov.b64 rb, {%4,%5};\n"
        " add.rn.f32x2 rd, ra, rb;\n mov.b64 {%0,%1}, rd;\n}"
        : "=f"(d.x), "=f"(d.y) : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}

// signed bytes 0,1 (lo) or 2,3 (hi) of w as exact floats: PRMT builds 2^23 + (c+128),
// one packed add removes the bias.
__device__ __forceinline__ float2 sbytes_f2(uint32_t w, int hi)
{
    const uint32_t x = w ^ 0x80808080u;
    const int b = hi ? 2 : 0;
    return fadd2(make_float2(__uint_as_float(__byte_perm(x, 0x4B000000u, 0x7540 + b)),
                             __uint_as_float(__byte_perm(x, 0x4B000000u, 0x7541 + b))),
                 make_float2(-8388736.0f, -8388736.0f));
}

// system-scope flag handshakes between GPUs (peer memory over NVLink)
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v)
{
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p)
{
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ float4 ld_volatile_f4(const float* p)
{
    float4 v;
    asm volatile("ld.volatile.global.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p) : "memory");
    return v;
}

constexpr int TB_ATTN_MAX_KV = 1024;   // kv heads per decode call (counter slots)

static inline int tb_cdiv(long long a, long long b) { return (int)((a + b - 1) / b); }
