/*
 * tb_cpu_ref.c -- the reference's CPU path for the hot path, transcribed to C,
 * used as the timed CPU baseline (bench.py cpu_baseline and --impl reference).
 *
 * TEST / BASELINE INFRASTRUCTURE ONLY: never linked into the product.
 *
 * The reference's own CPU code cannot run here (no cargo, no node), so these
 * are faithful transcriptions:
 *   - tbr_gemv_tern_scalar: tern.rs:100-140 (gemv_tern_scalar), plain loops;
 *   - tbr_gemv_tern_avx2: native/crates/n2-kernels/src/tern.rs:268-338, the
 *     same AVX2 intrinsics (vpmaddubsw + vpmaddwd, two 64-blocks per 256-bit
 *     step, scale lanes split per 128-bit half, one horizontal sum per row);
 *   - tbr_linear_int4: the int4 decode GEMV math as linearQ routes it
 *     (models/qwen3.js:1588-1608): N < 16384 -> quantQ8 + gemvDP4 integer math
 *     (qwen3.js:332-400), else gemvQ f32 math (qwen3.js:293-311), written as
 *     plain scalar loops (the JS engine is scalar on the CPU);
 *   - row partitioning over worker threads as cpu/kernel/cpuengine-mt.js and
 *     cpu/cpukern-fwd-worker.js:101-127 do it (CH=128-row chunks claimed from
 *     an atomic cursor).
 * Built with -O3 -mavx2 -ffp-contract=off by oracle/build.py.
 */
#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define TBR_API __attribute__((visibility("default")))

/* ---------------- ternary Q2_0_g64, AVX2 (tern.rs:268-338) ---------------- */

static inline float hsum256(__m256 v)
{
    __m128 lo = _mm256_castps256_ps128(v), hi = _mm256_extractf128_ps(v, 1);
    __m128 s = _mm_add_ps(lo, hi);
    s = _mm_add_ps(s, _mm_movehl_ps(s, s));
    s = _mm_add_ss(s, _mm_shuffle_ps(s, s, 0x55));
    return _mm_cvtss_f32(s);
}

static void tern_rows_avx2(float *out, const uint8_t *codes, const float *scales,
                           const int8_t *act, const int32_t *xsum,
                           int64_t r0, int64_t r1, int64_t K)
{
    const int64_t nb = K / 64, bpr = K / 4, pairs = nb / 2;
    const __m256i m3 = _mm256_set1_epi8(3), ones = _mm256_set1_epi16(1);
    for (int64_t row = r0; row < r1; row++) {
        const uint8_t *rc = codes + row * bpr;
        const float *rs = scales + row * nb;
        __m256 facc = _mm256_setzero_ps();
        float sxs = 0.0f;
        for (int64_t p = 0; p < pairs; p++) {
            int64_t b = 2 * p;
            __m256i raw = _mm256_loadu_si256((const __m256i *)(rc + b * 16));
            __m256i iacc = _mm256_setzero_si256();
            for (int j = 0; j < 4; j++) {
                __m256i pl = _mm256_and_si256(_mm256_srli_epi16(raw, 2 * j), m3);
                __m128i lo = _mm_loadu_si128((const __m128i *)(act + b * 64 + j * 16));
                __m128i hi = _mm_loadu_si128((const __m128i *)(act + (b + 1) * 64 + j * 16));
                __m256i a = _mm256_inserti128_si256(_mm256_castsi128_si256(lo), hi, 1);
                __m256i prod = _mm256_maddubs_epi16(pl, a);
                iacc = _mm256_add_epi32(iacc, _mm256_madd_epi16(prod, ones));
            }
            float s0 = rs[b], s1 = rs[b + 1];
            __m256 sv = _mm256_insertf128_ps(_mm256_castps128_ps256(_mm_set1_ps(s0)), _mm_set1_ps(s1), 1);
            facc = _mm256_add_ps(facc, _mm256_mul_ps(_mm256_cvtepi32_ps(iacc), sv));
            sxs += s0 * (float)xsum[b];
            sxs += s1 * (float)xsum[b + 1];
        }
        float acc = hsum256(facc);
        for (int64_t b = pairs * 2; b < nb; b++) {
            int32_t dot = 0;
            for (int j = 0; j < 4; j++)
                for (int i = 0; i < 16; i++)
                    dot += (int32_t)((rc[b * 16 + i] >> (2 * j)) & 3) * (int32_t)act[b * 64 + j * 16 + i];
            acc += rs[b] * (float)dot;
            sxs += rs[b] * (float)xsum[b];
        }
        out[row] = acc - sxs;
    }
}

/* ---------------- ternary Q2_0_g64, scalar (tern.rs:100-140) --------------
 * Per row: for every 64-block the exact i32 dot of the unsigned codes with the
 * int8 activations, plane j (bits 2j of each byte) holding codes j*16..j*16+15;
 * acc += s*dot and sxs += s*xsum in block order, out = acc - sxs. */
static void tern_rows_scalar(float *out, const uint8_t *codes, const float *scales,
                             const int8_t *act, const int32_t *xsum,
                             int64_t r0, int64_t r1, int64_t K)
{
    const int64_t nb = K / 64, bpr = K / 4;
    for (int64_t row = r0; row < r1; row++) {
        const uint8_t *rc = codes + row * bpr;
        const float *rs = scales + row * nb;
        float acc = 0.0f, sxs = 0.0f;
        for (int64_t b = 0; b < nb; b++) {
            const uint8_t *blk = rc + b * 16;
            const int8_t *ab = act + b * 64;
            int32_t dot = 0;
            for (int j = 0; j < 4; j++)
                for (int i = 0; i < 16; i++)
                    dot += (int32_t)((blk[i] >> (2 * j)) & 3) * (int32_t)ab[j * 16 + i];
            acc += rs[b] * (float)dot;
            sxs += rs[b] * (float)xsum[b];
        }
        out[row] = acc - sxs;
    }
}

/* ---------------- int4 G32 decode GEMV, scalar (linearQ math) ------------- */

static inline float f16_to_f32(uint16_t h)
{
    int s = (h >> 15) & 1, e = (h >> 10) & 0x1f, f = h & 0x3ff;
    float sg = s ? -1.0f : 1.0f;
    if (e == 0) return sg * ldexpf((float)f, -24);
    if (e == 31) return f ? NAN : sg * INFINITY;
    return sg * ldexpf(1.0f + (float)f / 1024.0f, e - 15);
}

/* gemvQ row math, qwen3.js:293-307: per u32 word, s*(dot(lo.x,hi.x,lo.y,hi.y . xa)
 * + dot(lo.z,hi.z,lo.w,hi.w . xb)). */
static void int4_rows_f32(float *y, const float *x, const uint32_t *pack,
                          const uint16_t *scales, int64_t r0, int64_t r1, int64_t K, int acc_flag)
{
    const int64_t words = K / 8, gpr = K / 32;
    for (int64_t n = r0; n < r1; n++) {
        const uint32_t *wr = pack + n * words;
        float acc = 0.0f;
        for (int64_t w = 0; w < words; w++) {
            uint32_t p = wr[w];
            float s = f16_to_f32(scales[n * gpr + (w * 8) / 32]);
            const float *xv = x + 8 * w;
            float d = 0.0f;
            for (int i = 0; i < 8; i++) d += (float)((int)((p >> (4 * i)) & 0xFu) - 8) * xv[i];
            acc += s * d;
        }
        y[n] = (acc_flag ? y[n] : 0.0f) + acc;
    }
}

/* gemvDP4 row math, qwen3.js:377-394: per word, f32(s16*xs) * f32(int dot). */
static void int4_rows_q8(float *y, const int8_t *xq, const float *xs, const uint32_t *pack,
                         const uint16_t *scales, int64_t r0, int64_t r1, int64_t K, int acc_flag)
{
    const int64_t words = K / 8, gpr = K / 32;
    for (int64_t n = r0; n < r1; n++) {
        const uint32_t *wr = pack + n * words;
        float acc = 0.0f;
        for (int64_t w = 0; w < words; w++) {
            uint32_t p = wr[w];
            int64_t g = (w * 8) / 32;
            float s = f16_to_f32(scales[n * gpr + g]) * xs[g];
            const int8_t *xv = xq + 8 * w;
            int32_t d = 0;
            for (int i = 0; i < 8; i++) d += ((int)((p >> (4 * i)) & 0xFu) - 8) * (int32_t)xv[i];
            acc += s * (float)d;
        }
        y[n] = (acc_flag ? y[n] : 0.0f) + acc;
    }
}

/* quantQ8 for one row, qwen3.js:332-358 (WGSL round = half-to-even). */
static void quant_q8_row(const float *x, int64_t K, int8_t *xq, float *xs)
{
    for (int64_t g = 0; g < K / 32; g++) {
        float m = 0.0f;
        for (int j = 0; j < 32; j++) m = fmaxf(m, fabsf(x[g * 32 + j]));
        float scale = m / 127.0f, inv = scale > 0.0f ? 1.0f / scale : 0.0f;
        xs[g] = scale;
        for (int j = 0; j < 32; j++) {
            int v = (int)rintf(x[g * 32 + j] * inv);
            xq[g * 32 + j] = (int8_t)(v < -127 ? -127 : (v > 127 ? 127 : v));
        }
    }
}

/* ---------------- row-partitioned worker pool ------------------------------ */

enum { JOB_TERN = 0, JOB_INT4_F32 = 1, JOB_INT4_Q8 = 2, JOB_TERN_SCALAR = 3 };
#define CHUNK_ROWS 128

typedef struct {
    int kind;
    int64_t N, K;
    int acc;
    float *out;
    const void *w;
    const void *s;
    const void *x;
    const void *xs;
    const int32_t *xsum;
    volatile int64_t cursor;
} job_t;

static void run_rows(job_t *j, int64_t r0, int64_t r1)
{
    switch (j->kind) {
    case JOB_TERN:
        tern_rows_avx2(j->out, (const uint8_t *)j->w, (const float *)j->s, (const int8_t *)j->x,
                       j->xsum, r0, r1, j->K);
        break;
    case JOB_TERN_SCALAR:
        tern_rows_scalar(j->out, (const uint8_t *)j->w, (const float *)j->s, (const int8_t *)j->x,
                         j->xsum, r0, r1, j->K);
        break;
    case JOB_INT4_F32:
        int4_rows_f32(j->out, (const float *)j->x, (const uint32_t *)j->w, (const uint16_t *)j->s,
                      r0, r1, j->K, j->acc);
        break;
    default:
        int4_rows_q8(j->out, (const int8_t *)j->x, (const float *)j->xs, (const uint32_t *)j->w,
                     (const uint16_t *)j->s, r0, r1, j->K, j->acc);
        break;
    }
}

static void *worker(void *arg)
{
    job_t *j = (job_t *)arg;
    for (;;) {
        int64_t r0 = __atomic_fetch_add(&j->cursor, CHUNK_ROWS, __ATOMIC_RELAXED);
        if (r0 >= j->N) break;
        int64_t r1 = r0 + CHUNK_ROWS < j->N ? r0 + CHUNK_ROWS : j->N;
        run_rows(j, r0, r1);
    }
    return NULL;
}

/* Persistent worker pool, as the reference's CPU engines keep their workers
 * (cpu/kernel/cpuengine-mt.js spawns them once): a call publishes the job under
 * a new generation number, workers 1 .. threads-1 join the chunk loop with the
 * caller, and the caller waits until every participant has left it.  Workers
 * spin briefly on the generation before sleeping on a condition variable. */
#define POOL_MAX 256
static struct {
    pthread_mutex_t mu;
    pthread_cond_t go, done;
    pthread_t tid[POOL_MAX];
    int n;                       /* workers started */
    volatile unsigned gen;       /* job generation */
    job_t *volatile job;
    volatile int want;           /* workers taking part in the current job */
    int left;                    /* participants still in the job */
} g_pool = {PTHREAD_MUTEX_INITIALIZER, PTHREAD_COND_INITIALIZER, PTHREAD_COND_INITIALIZER};

static void *pool_worker(void *arg)
{
    const int idx = (int)(intptr_t)arg;
    unsigned seen = 0;
    for (;;) {
        unsigned g;
        int spins = 0;
        while ((g = __atomic_load_n(&g_pool.gen, __ATOMIC_ACQUIRE)) == seen && spins < 200000) { spins++; }
        if (g == seen) {
            pthread_mutex_lock(&g_pool.mu);
            while ((g = g_pool.gen) == seen) pthread_cond_wait(&g_pool.go, &g_pool.mu);
            pthread_mutex_unlock(&g_pool.mu);
        }
        seen = g;
        if (idx < g_pool.want) {
            worker(g_pool.job);
            pthread_mutex_lock(&g_pool.mu);
            if (--g_pool.left == 0) pthread_cond_signal(&g_pool.done);
            pthread_mutex_unlock(&g_pool.mu);
        }
    }
    return NULL;
}

static void run_job(job_t *j, int threads)
{
    j->cursor = 0;
    if (threads <= 1) { run_rows(j, 0, j->N); return; }
    if (threads > POOL_MAX) threads = POOL_MAX;
    pthread_mutex_lock(&g_pool.mu);
    while (g_pool.n < threads - 1) {
        pthread_create(&g_pool.tid[g_pool.n], NULL, pool_worker, (void *)(intptr_t)g_pool.n);
        g_pool.n++;
    }
    g_pool.job = j;
    g_pool.want = threads - 1;
    g_pool.left = threads - 1;
    __atomic_store_n(&g_pool.gen, g_pool.gen + 1, __ATOMIC_RELEASE);
    pthread_cond_broadcast(&g_pool.go);
    pthread_mutex_unlock(&g_pool.mu);
    worker(j);
    pthread_mutex_lock(&g_pool.mu);
    while (g_pool.left > 0) pthread_cond_wait(&g_pool.done, &g_pool.mu);
    pthread_mutex_unlock(&g_pool.mu);
}

/* Ternary GEMV (tern.rs gemv_tern, AVX2 backend) over N rows with `threads`
 * workers; out[N] raw (caller scales by 1/act_scale). */
TBR_API void tbr_gemv_tern_avx2(float *out, const uint8_t *codes, const float *scales,
                                const int8_t *act, const int32_t *xsum, int64_t N, int64_t K,
                                int threads)
{
    job_t j = {JOB_TERN, N, K, 0, out, codes, scales, act, NULL, xsum, 0};
    run_job(&j, threads);
}

/* Ternary GEMV, scalar backend (tern.rs gemv_tern_scalar) over N rows. */
TBR_API void tbr_gemv_tern_scalar(float *out, const uint8_t *codes, const float *scales,
                                  const int8_t *act, const int32_t *xsum, int64_t N, int64_t K,
                                  int threads)
{
    job_t j = {JOB_TERN_SCALAR, N, K, 0, out, codes, scales, act, NULL, xsum, 0};
    run_job(&j, threads);
}

/* int4 decode linear as linearQ routes it at T=1 (qwen3.js:1598-1602).
 * x f32 [K]; q8 scratch xq [K], xs [K/32] supplied by the caller. */
TBR_API void tbr_linear_int4(float *y, const float *x, const uint32_t *pack,
                             const uint16_t *scales, int64_t N, int64_t K, int acc,
                             int8_t *xq, float *xs, int threads)
{
    if (N < 16384) {
        quant_q8_row(x, K, xq, xs);
        job_t j = {JOB_INT4_Q8, N, K, acc, y, pack, scales, xq, xs, NULL, 0};
        run_job(&j, threads);
    } else {
        job_t j = {JOB_INT4_F32, N, K, acc, y, pack, scales, x, NULL, NULL, 0};
        run_job(&j, threads);
    }
}

/* gemvQ math (f32 activations) over all N rows, whatever N: the route linearQ
 * takes for the lm_head (qwen3.js:1602). */
TBR_API void tbr_gemv_int4_f32(float *y, const float *x, const uint32_t *pack, const uint16_t *scales,
                               int64_t N, int64_t K, int acc, int threads)
{
    job_t j = {JOB_INT4_F32, N, K, acc, y, pack, scales, x, NULL, NULL, 0};
    run_job(&j, threads);
}
