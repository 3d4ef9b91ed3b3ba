// tb_ctx.cu -- context lifetime, streams, error strings and context-owned scratch.
#include <stdarg.h>
#include <new>

#include "tb_common.cuh"

int tb_fail(tb_ctx* ctx, int code, const char* fmt, ...)
{
    if (ctx) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        ctx->last_error = buf;
    }
    return code;
}

int tb_check_launch(tb_ctx* ctx, const char* what)
{
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return TB_OK;
}

void* tb_ctx_scratch(tb_ctx* ctx, size_t bytes)
{
    if (bytes <= ctx->scratch_bytes) return ctx->scratch;
    // The old buffer may still be read by work queued on the stream: finish it first.
    if (ctx->scratch) {
        cudaStreamSynchronize(ctx->stream);
        cudaFree(ctx->scratch);
        ctx->scratch = nullptr;
        ctx->scratch_bytes = 0;
    }
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    want = (want + 255) & ~size_t(255);
    if (cudaMalloc(&ctx->scratch, want) != cudaSuccess) {
        cudaGetLastError();
        tb_fail(ctx, TB_ERR_NOMEM, "scratch allocation of %zu bytes failed", want);
        return nullptr;
    }
    ctx->scratch_bytes = want;
    return ctx->scratch;
}

extern "C" {

TB_API int tb_version(void) { return 100; }

TB_API int tb_ctx_create(int device, tb_ctx** out)
{
    if (!out) return TB_ERR_INVALID;
    *out = nullptr;
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
        cudaGetLastError();
        return TB_ERR_INVALID;
    }
    tb_ctx* c = new (std::nothrow) tb_ctx();
    if (!c) return TB_ERR_NOMEM;
    c->device = device;
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(device) != cudaSuccess) { delete c; return TB_ERR_CUDA; }
    cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
    if (major < 10) {
        delete c;
        cudaSetDevice(prev);
        return TB_ERR_UNSUPPORTED;   // the kernels are built for sm_100a only
    }
    if (cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&c->dev_error, sizeof(int)) != cudaSuccess ||
        cudaMemset(c->dev_error, 0, sizeof(int)) != cudaSuccess ||
        cudaMalloc(&c->attn_counters, TB_ATTN_MAX_KV * sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(c->attn_counters, 0, TB_ATTN_MAX_KV * sizeof(unsigned)) != cudaSuccess) {
        cudaGetLastError();
        if (c->dev_error) cudaFree(c->dev_error);
        if (c->attn_counters) cudaFree(c->attn_counters);
        if (c->own_stream) cudaStreamDestroy(c->own_stream);
        delete c;
        cudaSetDevice(prev);
        return TB_ERR_CUDA;
    }
    c->stream = c->own_stream;
    *out = c;
    return TB_OK;
}

TB_API int tb_ctx_destroy(tb_ctx* ctx)
{
    if (!ctx) return TB_OK;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->dev_error) cudaFree(ctx->dev_error);
    if (ctx->attn_counters) cudaFree(ctx->attn_counters);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return TB_OK;
}

TB_API int tb_ctx_set_stream(tb_ctx* ctx, void* s)
{
    if (!ctx) return TB_ERR_INVALID;
    ctx->stream = s ? (cudaStream_t)s : ctx->own_stream;
    return TB_OK;
}

TB_API void* tb_ctx_get_stream(tb_ctx* ctx) { return ctx ? (void*)ctx->stream : nullptr; }

TB_API int tb_ctx_set_pdl(tb_ctx* ctx, int enable)
{
    if (!ctx) return TB_ERR_INVALID;
    ctx->pdl = enable != 0;
    return TB_OK;
}

TB_API const char* tb_last_error(tb_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

TB_API int tb_ctx_synchronize(tb_ctx* ctx)
{
    if (!ctx) return TB_ERR_INVALID;
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "synchronize: %s", cudaGetErrorString(e));
    return TB_OK;
}

struct tb_batch {
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
};

TB_API int tb_batch_begin(tb_ctx* ctx)
{
    if (!ctx) return TB_ERR_INVALID;
    TB_REQUIRE(ctx, ctx->stream == ctx->own_stream, "recording needs the context's own stream");
    cudaError_t e = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "begin capture: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_batch_end(tb_ctx* ctx, tb_batch** out)
{
    if (!ctx || !out) return TB_ERR_INVALID;
    *out = nullptr;
    tb_batch* b = new (std::nothrow) tb_batch();
    if (!b) return TB_ERR_NOMEM;
    cudaError_t e = cudaStreamEndCapture(ctx->stream, &b->graph);
    if (e == cudaSuccess) e = cudaGraphInstantiate(&b->exec, b->graph, 0);
    if (e != cudaSuccess) {
        if (b->graph) cudaGraphDestroy(b->graph);
        delete b;
        cudaGetLastError();
        return tb_fail(ctx, TB_ERR_CUDA, "end capture: %s", cudaGetErrorString(e));
    }
    *out = b;
    return TB_OK;
}

TB_API int tb_batch_submit(tb_ctx* ctx, tb_batch* b)
{
    if (!ctx || !b) return TB_ERR_INVALID;
    cudaError_t e = cudaGraphLaunch(b->exec, ctx->stream);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "batch submit: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_batch_destroy(tb_batch* b)
{
    if (!b) return TB_OK;
    if (b->exec) cudaGraphExecDestroy(b->exec);
    if (b->graph) cudaGraphDestroy(b->graph);
    delete b;
    return TB_OK;
}

TB_API int tb_copy_h2d(tb_ctx* ctx, void* dst, const void* src, size_t bytes)
{
    if (!ctx) return TB_ERR_INVALID;
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "h2d copy: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_copy_d2h(tb_ctx* ctx, void* dst, const void* src, size_t bytes)
{
    if (!ctx) return TB_ERR_INVALID;
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, ctx->stream);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "d2h copy: %s", cudaGetErrorString(e));
    return TB_OK;
}

TB_API int tb_ctx_device_error(tb_ctx* ctx, int* code)
{
    if (!ctx || !code) return TB_ERR_INVALID;
    int v = 0;
    cudaError_t e = cudaMemcpyAsync(&v, ctx->dev_error, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e == cudaSuccess && v) e = cudaMemsetAsync(ctx->dev_error, 0, sizeof(int), ctx->stream);
    if (e != cudaSuccess) return tb_fail(ctx, TB_ERR_CUDA, "device error read: %s", cudaGetErrorString(e));
    *code = v;
    return v ? tb_fail(ctx, TB_ERR_TIMEOUT, "device-side bounded wait gave up (code %d)", v) : TB_OK;
}

}  // extern "C"
