/*
 * ki_oracle.c -- CPU restatement of the semantics the B200 kernels must reproduce.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: only the test-suite, the
 * smoke entry point and the CPU-baseline leg of the benchmark load it.  The
 * product library never links, loads or calls it.
 *
 * Reference being restated: epilliat/KernelIntrinsics.jl v0.1.6.  That package
 * ships device-side intrinsics only; the device-wide operations built from them
 * follow Julia Base semantics:
 *   sum      -> Base.sum of Float32 data, checked against a Float64 accumulation
 *   cumsum   -> Base.cumsum of Int64 (two's-complement wrap-around)
 *   filter / findall -> order preserving, 1-based indices
 *   copyto!  -> byte copy
 * and the warp / vector primitives restated here follow
 *   src/warp.jl:226-237        (@warpreduce: inclusive Up-shuffle scan, lane > offset)
 *   src/warp.jl:273-282        (@warpfold: Down-shuffle fold, lane 1 holds the total)
 *   src/vectorization.jl:306-338 (generate_partN: naturally aligned piece patterns)
 *   src/vectorization.jl:374-379 (vload_multi: mod = (ptr/sizeof(T) + i-1) % N + 1)
 *
 * Synthetic inputs come from a counter-based splitmix64 stream so that the host
 * and the device generators produce bit-identical data: element i of stream
 * `seed` is mix64(seed + (i+1) * 0x9E3779B97F4A7C15), i.e. the (i+1)-th output
 * of Vigna's splitmix64 generator started at `seed`.
 *
 * The fp8 e4m3 codec follows the OCP 8-bit floating point specification (E4M3FN:
 * bias 7, no infinities, S.1111.111 is NaN, largest finite 448), with
 * round-to-nearest-even and saturation to +-448.
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define KO_GOLDEN 0x9E3779B97F4A7C15ull

/* ------------------------------------------------------------------------ */
/* splitmix64 stream                                                         */
/* ------------------------------------------------------------------------ */

uint64_t ko_mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

uint64_t ko_rand64(uint64_t seed, uint64_t i) { return ko_mix64(seed + (i + 1) * KO_GOLDEN); }

/* ------------------------------------------------------------------------ */
/* small pthread helper: run fn(arg, lo, hi, tid) over [0,n) split in chunks  */
/* ------------------------------------------------------------------------ */

typedef void (*ko_range_fn)(void* arg, size_t lo, size_t hi, int tid);

typedef struct {
    ko_range_fn fn;
    void* arg;
    size_t lo, hi;
    int tid;
} ko_job;

static void* ko_job_main(void* p) {
    ko_job* j = (ko_job*)p;
    j->fn(j->arg, j->lo, j->hi, j->tid);
    return NULL;
}

int ko_default_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

static void ko_parallel(ko_range_fn fn, void* arg, size_t n, int threads) {
    if (threads <= 0) threads = ko_default_threads();
    if (threads > 256) threads = 256;
    if ((size_t)threads > n) threads = n > 0 ? (int)n : 1;
    if (threads == 1) {
        fn(arg, 0, n, 0);
        return;
    }
    pthread_t th[256];
    ko_job jobs[256];
    for (int t = 0; t < threads; ++t) {
        jobs[t].fn = fn;
        jobs[t].arg = arg;
        jobs[t].lo = n * (size_t)t / (size_t)threads;
        jobs[t].hi = n * (size_t)(t + 1) / (size_t)threads;
        jobs[t].tid = t;
        pthread_create(&th[t], NULL, ko_job_main, &jobs[t]);
    }
    for (int t = 0; t < threads; ++t) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------ */
/* generators (bit-identical to the device generators)                       */
/* ------------------------------------------------------------------------ */

typedef struct {
    uint64_t seed;
    void* out;
    int64_t lo, span;
    float scale;
} ko_gen_arg;

/* U[0,1): the top 24 bits of the stream, scaled by 2^-24 (exact in binary32). */
static inline float ko_u01(uint64_t r) { return (float)(r >> 40) * 0x1p-24f; }

static void ko_gen_u01_part(void* a, size_t lo, size_t hi, int tid) {
    (void)tid;
    ko_gen_arg* g = (ko_gen_arg*)a;
    float* o = (float*)g->out;
    for (size_t i = lo; i < hi; ++i) o[i] = ko_u01(ko_rand64(g->seed, i));
}

void ko_gen_uniform_f32(uint64_t seed, float* out, size_t n, int threads) {
    ko_gen_arg g = {seed, out, 0, 0, 0.f};
    ko_parallel(ko_gen_u01_part, &g, n, threads);
}

/* Integers in [lo, lo+span): r % span + lo (the modulo bias is part of the
 * definition and is reproduced identically by the device generator). */
static void ko_gen_int_part(void* a, size_t lo, size_t hi, int tid) {
    (void)tid;
    ko_gen_arg* g = (ko_gen_arg*)a;
    int64_t* o = (int64_t*)g->out;
    for (size_t i = lo; i < hi; ++i) o[i] = (int64_t)(ko_rand64(g->seed, i) % (uint64_t)g->span) + g->lo;
}

void ko_gen_int_range_i64(uint64_t seed, int64_t lo, int64_t hi, int64_t* out, size_t n, int threads) {
    ko_gen_arg g = {seed, out, lo, hi - lo + 1, 0.f};
    ko_parallel(ko_gen_int_part, &g, n, threads);
}

/* Bytes: byte i is byte (i % 8) (little-endian) of stream word i / 8. */
static void ko_gen_bytes_part(void* a, size_t lo, size_t hi, int tid) {
    (void)tid;
    ko_gen_arg* g = (ko_gen_arg*)a;
    uint8_t* o = (uint8_t*)g->out;
    for (size_t i = lo; i < hi; ++i) o[i] = (uint8_t)(ko_rand64(g->seed, i >> 3) >> (8 * (i & 7)));
}

void ko_gen_bytes(uint64_t seed, uint8_t* out, size_t n, int threads) {
    ko_gen_arg g = {seed, out, 0, 0, 0.f};
    ko_parallel(ko_gen_bytes_part, &g, n, threads);
}

/* ------------------------------------------------------------------------ */
/* fp8 e4m3 (OCP E4M3FN) codec                                              */
/* ------------------------------------------------------------------------ */

float ko_e4m3_decode(uint8_t b) {
    int s = b >> 7, e = (b >> 3) & 15, m = b & 7;
    float v;
    if (e == 15 && m == 7) return s ? -NAN : NAN;
    if (e == 0)
        v = ldexpf((float)m, -9); /* subnormal: m * 2^-9 */
    else
        v = ldexpf((float)(8 + m), e - 10); /* (1 + m/8) * 2^(e-7) */
    return s ? -v : v;
}

/* Round-to-nearest-even with saturation to +-448 (the cvt ... .satfinite rule). */
uint8_t ko_e4m3_encode(float x) {
    if (isnan(x)) return 0x7F;
    uint8_t s = signbit(x) ? 0x80 : 0;
    double a = fabs((double)x);
    if (a >= 448.0) return s | 0x7E;
    if (a == 0.0) return s;
    int e;
    frexp(a, &e);         /* a = f * 2^e, f in [0.5,1) -> unbiased exponent e-1 */
    int ue = e - 1;
    if (ue < -6) {        /* subnormal range: quantum 2^-9 */
        double q = nearbyint(a * 512.0);
        if (q >= 8.0) return s | 0x08; /* rounds up to the smallest normal */
        return s | (uint8_t)q;
    }
    double q = nearbyint(ldexp(a, 3 - ue)); /* in [8,16] */
    if (q >= 16.0) {
        q = 8.0;
        ue += 1;
    }
    if (ue > 8 || (ue == 8 && q > 14.0)) return s | 0x7E;
    return s | (uint8_t)(((ue + 7) << 3) | ((int)q - 8));
}

/* U[-1,1) * scale rounded to e4m3.  Computed in binary32 in this exact order
 * ((2u - 1) * scale, each step correctly rounded) so the device generator can
 * reproduce it bit for bit. */
static void ko_gen_e4m3_part(void* a, size_t lo, size_t hi, int tid) {
    (void)tid;
    ko_gen_arg* g = (ko_gen_arg*)a;
    uint8_t* o = (uint8_t*)g->out;
    for (size_t i = lo; i < hi; ++i) {
        volatile float u = ko_u01(ko_rand64(g->seed, i));
        volatile float c = 2.0f * u - 1.0f;
        volatile float x = c * g->scale;
        o[i] = ko_e4m3_encode(x);
    }
}

void ko_gen_e4m3_uniform(uint64_t seed, float scale, uint8_t* out, size_t n, int threads) {
    ko_gen_arg g = {seed, out, 0, 0, scale};
    ko_parallel(ko_gen_e4m3_part, &g, n, threads);
}

/* ------------------------------------------------------------------------ */
/* sum: Float64 accumulation of Float32 data                                 */
/* ------------------------------------------------------------------------ */

typedef struct {
    const float* x;
    double part[256];
} ko_sum_arg;

static void ko_sum_part(void* a, size_t lo, size_t hi, int tid) {
    ko_sum_arg* s = (ko_sum_arg*)a;
    double acc = 0.0;
    for (size_t i = lo; i < hi; ++i) acc += (double)s->x[i];
    s->part[tid] = acc;
}

double ko_sum_f32(const float* x, size_t n, int threads) {
    if (threads <= 0) threads = ko_default_threads();
    if (threads > 256) threads = 256;
    ko_sum_arg s;
    memset(&s, 0, sizeof(s));
    s.x = x;
    ko_parallel(ko_sum_part, &s, n, threads);
    double acc = 0.0;
    for (int t = 0; t < 256; ++t) acc += s.part[t];
    return acc;
}

/* ------------------------------------------------------------------------ */
/* cumsum: inclusive Int64 prefix sum with wrap-around, optional seed        */
/* ------------------------------------------------------------------------ */

typedef struct {
    const int64_t* x;
    int64_t* y;
    uint64_t part[256];
    size_t lo[256];
} ko_scan_arg;

static void ko_scan_reduce_part(void* a, size_t lo, size_t hi, int tid) {
    ko_scan_arg* s = (ko_scan_arg*)a;
    uint64_t acc = 0;
    for (size_t i = lo; i < hi; ++i) acc += (uint64_t)s->x[i];
    s->part[tid] = acc;
    s->lo[tid] = lo;
}

static void ko_scan_write_part(void* a, size_t lo, size_t hi, int tid) {
    ko_scan_arg* s = (ko_scan_arg*)a;
    uint64_t acc = s->part[tid]; /* exclusive prefix of this chunk */
    for (size_t i = lo; i < hi; ++i) {
        acc += (uint64_t)s->x[i];
        s->y[i] = (int64_t)acc;
    }
}

void ko_cumsum_i64(const int64_t* x, int64_t* y, size_t n, int64_t seed, int threads) {
    if (threads <= 0) threads = ko_default_threads();
    if (threads > 256) threads = 256;
    if ((size_t)threads > n) threads = n > 0 ? (int)n : 1;
    ko_scan_arg s;
    memset(&s, 0, sizeof(s));
    s.x = x;
    s.y = y;
    ko_parallel(ko_scan_reduce_part, &s, n, threads);
    uint64_t run = (uint64_t)seed;
    for (int t = 0; t < threads; ++t) {
        uint64_t tot = s.part[t];
        s.part[t] = run;
        run += tot;
    }
    ko_parallel(ko_scan_write_part, &s, n, threads);
}

int64_t ko_sum_i64(const int64_t* x, size_t n, int threads) {
    ko_scan_arg s;
    memset(&s, 0, sizeof(s));
    s.x = x;
    if (threads <= 0) threads = ko_default_threads();
    if (threads > 256) threads = 256;
    ko_parallel(ko_scan_reduce_part, &s, n, threads);
    uint64_t acc = 0;
    for (int t = 0; t < 256; ++t) acc += s.part[t];
    return (int64_t)acc;
}

/* ------------------------------------------------------------------------ */
/* filter / findall: order preserving compaction of x > thr                  */
/* ------------------------------------------------------------------------ */

typedef struct {
    const float* x;
    float thr;
    float* vals;
    int32_t* idx;
    int64_t base;
    size_t cnt[256];
} ko_filt_arg;

static void ko_filt_count(void* a, size_t lo, size_t hi, int tid) {
    ko_filt_arg* f = (ko_filt_arg*)a;
    size_t c = 0;
    for (size_t i = lo; i < hi; ++i) c += f->x[i] > f->thr;
    f->cnt[tid] = c;
}

static void ko_filt_write(void* a, size_t lo, size_t hi, int tid) {
    ko_filt_arg* f = (ko_filt_arg*)a;
    size_t o = f->cnt[tid];
    for (size_t i = lo; i < hi; ++i) {
        float v = f->x[i];
        if (v > f->thr) {
            if (f->vals) f->vals[o] = v;
            if (f->idx) f->idx[o] = (int32_t)((int64_t)i + f->base);
            ++o;
        }
    }
}

size_t ko_filter_gt_f32(const float* x, size_t n, float thr, float* vals, int32_t* idx, int64_t index_base,
                        int threads) {
    if (threads <= 0) threads = ko_default_threads();
    if (threads > 256) threads = 256;
    if ((size_t)threads > n) threads = n > 0 ? (int)n : 1;
    ko_filt_arg f;
    memset(&f, 0, sizeof(f));
    f.x = x;
    f.thr = thr;
    f.vals = vals;
    f.idx = idx;
    f.base = index_base;
    ko_parallel(ko_filt_count, &f, n, threads);
    size_t run = 0;
    for (int t = 0; t < threads; ++t) {
        size_t c = f.cnt[t];
        f.cnt[t] = run;
        run += c;
    }
    if (vals || idx) ko_parallel(ko_filt_write, &f, n, threads);
    return run;
}

/* ------------------------------------------------------------------------ */
/* copyto!: byte copy                                                        */
/* ------------------------------------------------------------------------ */

typedef struct {
    uint8_t* dst;
    const uint8_t* src;
} ko_copy_arg;

static void ko_copy_part(void* a, size_t lo, size_t hi, int tid) {
    (void)tid;
    ko_copy_arg* c = (ko_copy_arg*)a;
    memcpy(c->dst + lo, c->src + lo, hi - lo);
}

void ko_copy_bytes(void* dst, const void* src, size_t n, int threads) {
    ko_copy_arg c = {(uint8_t*)dst, (const uint8_t*)src};
    ko_parallel(ko_copy_part, &c, n, threads);
}

/* ------------------------------------------------------------------------ */
/* GEMM of dequantised e4m3 operands in Float64                              */
/* A: M x K row-major, B: K x N row-major, C: rows [r0, r1) x N row-major    */
/* ------------------------------------------------------------------------ */

typedef struct {
    const uint8_t* A;
    const uint8_t* B;
    double* C;
    int N, K, r0;
    double scale;
    const double* lut;
} ko_gemm_arg;

static void ko_gemm_part(void* a, size_t lo, size_t hi, int tid) {
    (void)tid;
    ko_gemm_arg* g = (ko_gemm_arg*)a;
    const int N = g->N, K = g->K;
    double* row = (double*)malloc(sizeof(double) * (size_t)N);
    for (size_t r = lo; r < hi; ++r) {
        const uint8_t* arow = g->A + ((size_t)g->r0 + r) * (size_t)K;
        for (int n = 0; n < N; ++n) row[n] = 0.0;
        for (int k = 0; k < K; ++k) {
            double av = g->lut[arow[k]];
            if (av == 0.0) continue;
            const uint8_t* brow = g->B + (size_t)k * (size_t)N;
            for (int n = 0; n < N; ++n) row[n] += av * g->lut[brow[n]];
        }
        double* crow = g->C + r * (size_t)N;
        for (int n = 0; n < N; ++n) crow[n] = row[n] * g->scale;
    }
    free(row);
}

void ko_gemm_e4m3_rows(const uint8_t* A, const uint8_t* B, double* C, int r0, int r1, int N, int K, double scale,
                       int threads) {
    double lut[256];
    for (int i = 0; i < 256; ++i) lut[i] = (double)ko_e4m3_decode((uint8_t)i);
    ko_gemm_arg g = {A, B, C, N, K, r0, scale, lut};
    ko_parallel(ko_gemm_part, &g, (size_t)(r1 - r0), threads);
}

/* ------------------------------------------------------------------------ */
/* generate_partN (src/vectorization.jl:306-338)                             */
/* pieces for alignment residue r in [0,N); returns the piece count          */
/* ------------------------------------------------------------------------ */

int ko_generate_partN(int N, int r, int* pieces) {
    if (N <= 0 || (N & (N - 1)) || r < 0 || r >= N) return -1;
    if (r == 0) {
        pieces[0] = N;
        return 1;
    }
    int cnt = 0, remaining = N, pos = r;
    while (remaining > 0) {
        int max_load = N / 2; /* never more than N/2 when misaligned */
        while (max_load > 0) {
            if (pos % max_load == 0 && max_load <= remaining) break;
            max_load /= 2;
        }
        if (max_load == 0) max_load = 1;
        pieces[cnt++] = max_load;
        remaining -= max_load;
        pos = (pos + max_load) % N;
    }
    return cnt;
}
