/*
 * zpu_oracle.c -- CPU restatement of zpu's CPU path for the data-parallel hot
 * path (matmul, jit elementwise/reduction chains, the MLP train step).
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle: only the test
 * suite, the smoke check and bench.py's CPU-baseline / reference arm may load
 * it, and only as the checker or as the timed CPU baseline.  The product
 * (libzpucuda.so) never links, loads or calls it, and has no CPU fallback.
 *
 * Every function names the reference file:line it follows (paths relative to
 * the umiturtle/ZPU project root).  Build flags matter: -ffp-contract=off keeps
 * `a*b + c` as two roundings, exactly as Zig's default (strict) float mode
 * does, while the explicit fmaf/fma calls restate Zig's `@mulAdd`.
 *
 * Parity is pinned by tests/golden (fixtures extracted from the reference's
 * own snapshot files and unit tests): splitmix64 / Box-Muller exactly, matmul,
 * tanh, sum, vmap, jit replay and Adam within the snapshot tolerance.
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define ZO_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* RNG: src/zpu/rng.zig:15-102                                               */
/* ------------------------------------------------------------------------ */

/* splitmix64 step, rng.zig:23-29 (wrapping add of the golden gamma, two
 * xor-shift-multiply rounds, final xor-shift). */
static inline uint64_t sm_next(uint64_t *s) {
    *s += 0x9E3779B97F4A7C15ULL;
    uint64_t z = *s;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

/* rng.zig:32-35: the top 53 bits scaled by 2^-53. */
static inline double sm_f64(uint64_t *s) {
    return (double)(sm_next(s) >> 11) * (1.0 / 9007199254740992.0);
}

ZO_EXPORT uint64_t zo_rng_next(uint64_t *state) { return sm_next(state); }
ZO_EXPORT double zo_rng_next_f64(uint64_t *state) { return sm_f64(state); }

/* Rng.uniformRange, rng.zig:46-51: low + (high - low) * u, two roundings,
 * then Tensor.writeF64 rounds to the element type. */
ZO_EXPORT void zo_uniform_range_f64(uint64_t seed, double *out, size_t n, double lo, double hi) {
    uint64_t s = seed;
    for (size_t i = 0; i < n; i++) out[i] = lo + (hi - lo) * sm_f64(&s);
}
ZO_EXPORT void zo_uniform_range_f32(uint64_t seed, float *out, size_t n, double lo, double hi) {
    uint64_t s = seed;
    for (size_t i = 0; i < n; i++) out[i] = (float)(lo + (hi - lo) * sm_f64(&s));
}

/* Rng.normal, rng.zig:54-71: basic Box-Muller, one (cos, sin) pair per two
 * uniforms, u1 clamped below at 1e-12, theta = (2*pi) * u2. */
#define ZO_TWO_PI 6.283185307179586 /* 2 * (pi rounded to f64), exact doubling */
ZO_EXPORT void zo_normal_f64(uint64_t seed, double *out, size_t n) {
    uint64_t s = seed;
    size_t i = 0;
    while (i < n) {
        double a1 = sm_f64(&s);
        if (a1 < 1e-12) a1 = 1e-12;
        double a2 = sm_f64(&s);
        double r = sqrt(-2.0 * log(a1));
        double th = ZO_TWO_PI * a2;
        out[i++] = r * cos(th);
        if (i < n) out[i++] = r * sin(th);
    }
}
ZO_EXPORT void zo_normal_f32(uint64_t seed, float *out, size_t n) {
    uint64_t s = seed;
    size_t i = 0;
    while (i < n) {
        double a1 = sm_f64(&s);
        if (a1 < 1e-12) a1 = 1e-12;
        double a2 = sm_f64(&s);
        double r = sqrt(-2.0 * log(a1));
        double th = ZO_TWO_PI * a2;
        out[i++] = (float)(r * cos(th));
        if (i < n) out[i++] = (float)(r * sin(th));
    }
}

/* Rng.randint, rng.zig:93-101: low + next() % span. */
ZO_EXPORT int zo_randint_i64(uint64_t seed, int64_t *out, size_t n, int64_t lo, int64_t hi) {
    if (hi <= lo) return -1;
    uint64_t s = seed;
    uint64_t span = (uint64_t)(hi - lo);
    for (size_t i = 0; i < n; i++) out[i] = lo + (int64_t)(sm_next(&s) % span);
    return 0;
}

/* ------------------------------------------------------------------------ */
/* GEMM: src/zpu/kernels.zig:325-430                                         */
/* ------------------------------------------------------------------------ */

/* kernels.gemm (kernels.zig:339-408).  The result tile is MR=32 rows by
 * NB=128 columns; each output element is the FMA chain
 *     c = 0; for p in 0..k: c = fma(a[i,p], b[p,j], c)
 * over the vector-covered columns of the panel (the first floor(nb/L)*L of
 * them, L = 32 bytes / sizeof(T)), and c = c + a*b (two roundings) for the
 * leftover columns (kernels.zig:398).  Blocking changes traversal only, never
 * the per-element order, so this is bit-exact with zpu. */
#define ZO_MR 32
#define ZO_NB 128

#define DEFINE_GEMM(NAME, T, FMA, L)                                              \
    static void NAME(const T *a, const T *b, T *d, size_t m, size_t k, size_t n) { \
        if (m == 0 || n == 0) return;                                              \
        if (k == 0) {                                                              \
            memset(d, 0, m * n * sizeof(T));                                       \
            return;                                                                \
        }                                                                          \
        T *tile = (T *)aligned_alloc(64, ZO_MR * ZO_NB * sizeof(T));               \
        for (size_t jb = 0; jb < n; jb += ZO_NB) {                                 \
            size_t nb = n - jb < ZO_NB ? n - jb : ZO_NB;                           \
            size_t nv = (nb / (L)) * (L);                                          \
            for (size_t ib = 0; ib < m; ib += ZO_MR) {                             \
                size_t mb = m - ib < ZO_MR ? m - ib : ZO_MR;                       \
                memset(tile, 0, mb * ZO_NB * sizeof(T));                           \
                for (size_t p = 0; p < k; p++) {                                   \
                    const T *brow = b + p * n + jb;                                \
                    for (size_t i = 0; i < mb; i++) {                              \
                        const T av = a[(ib + i) * k + p];                          \
                        T *row = tile + i * ZO_NB;                                 \
                        for (size_t j = 0; j < nv; j++)                            \
                            row[j] = FMA(av, brow[j], row[j]);                     \
                        for (size_t j = nv; j < nb; j++) row[j] += av * brow[j];   \
                    }                                                              \
                }                                                                  \
                for (size_t i = 0; i < mb; i++)                                    \
                    memcpy(d + (ib + i) * n + jb, tile + i * ZO_NB,                \
                           nb * sizeof(T));                                        \
            }                                                                      \
        }                                                                          \
        free(tile);                                                                \
    }

DEFINE_GEMM(gemm_f32, float, fmaf, 8)
DEFINE_GEMM(gemm_f64, double, fma, 4)

ZO_EXPORT void zo_gemm_f32(const float *a, const float *b, float *d, size_t m, size_t k, size_t n) {
    gemm_f32(a, b, d, m, k, n);
}
ZO_EXPORT void zo_gemm_f64(const double *a, const double *b, double *d, size_t m, size_t k, size_t n) {
    gemm_f64(a, b, d, m, k, n);
}

/* ops.gemmBatched (ops.zig:1226-1282): walks the flattened broadcast batch in
 * row-major order; per batch axis `ax` the operand offsets advance by
 * acs[ax] / bcs[ax] elements (0 = broadcast along that axis); the output is
 * contiguous, batch after batch.  Each matrix goes through kernels.gemm. */
#define DEFINE_GEMM_BATCHED(NAME, T, G)                                                      \
    ZO_EXPORT void NAME(const T *a, const T *b, T *d, size_t m, size_t k, size_t n,          \
                        int nax, const int64_t *dims, const int64_t *acs, const int64_t *bcs) { \
        int64_t idx[8] = {0};                                                                 \
        int64_t aoff = 0, boff = 0;                                                           \
        size_t total = 1;                                                                     \
        for (int i = 0; i < nax; i++) total *= (size_t)dims[i];                               \
        for (size_t bt = 0; bt < total; bt++) {                                               \
            G(a + aoff, b + boff, d + bt * m * n, m, k, n);                                   \
            for (int ax = nax - 1; ax >= 0; ax--) {                                           \
                idx[ax] += 1;                                                                 \
                aoff += acs[ax];                                                              \
                boff += bcs[ax];                                                              \
                if (idx[ax] < dims[ax]) break;                                                \
                aoff -= dims[ax] * acs[ax];                                                   \
                boff -= dims[ax] * bcs[ax];                                                   \
                idx[ax] = 0;                                                                  \
            }                                                                                 \
        }                                                                                     \
    }
DEFINE_GEMM_BATCHED(zo_gemm_batched_f32, float, gemm_f32)
DEFINE_GEMM_BATCHED(zo_gemm_batched_f64, double, gemm_f64)

/* ------------------------------------------------------------------------ */
/* Reductions: src/zpu/kernels.zig:232-279 (sum/prod), :254-267 (max/min)   */
/* ------------------------------------------------------------------------ */

/* reduceAll(.sum) for f32: four 8-lane accumulators stride 32; leftover full
 * vectors into acc0; ((acc0+acc1)+acc2)+acc3 lanewise; lanes left to right;
 * then the scalar tail as `src[i] + best`. */
ZO_EXPORT float zo_reduce_sum_f32(const float *src, size_t n) {
    float acc[4][8];
    memset(acc, 0, sizeof acc);
    size_t i = 0;
    for (; i + 32 <= n; i += 32)
        for (int k = 0; k < 4; k++)
            for (int l = 0; l < 8; l++) acc[k][l] = acc[k][l] + src[i + k * 8 + l];
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) acc[0][l] = acc[0][l] + src[i + l];
    float tot[8];
    for (int l = 0; l < 8; l++) tot[l] = ((acc[0][l] + acc[1][l]) + acc[2][l]) + acc[3][l];
    float best = tot[0];
    for (int l = 1; l < 8; l++) best = best + tot[l];
    for (; i < n; i++) best = src[i] + best;
    return best;
}

ZO_EXPORT double zo_reduce_sum_f64(const double *src, size_t n) {
    double acc[4][4];
    memset(acc, 0, sizeof acc);
    size_t i = 0;
    for (; i + 16 <= n; i += 16)
        for (int k = 0; k < 4; k++)
            for (int l = 0; l < 4; l++) acc[k][l] = acc[k][l] + src[i + k * 4 + l];
    for (; i + 4 <= n; i += 4)
        for (int l = 0; l < 4; l++) acc[0][l] = acc[0][l] + src[i + l];
    double tot[4];
    for (int l = 0; l < 4; l++) tot[l] = ((acc[0][l] + acc[1][l]) + acc[2][l]) + acc[3][l];
    double best = tot[0];
    for (int l = 1; l < 4; l++) best = best + tot[l];
    for (; i < n; i++) best = src[i] + best;
    return best;
}

/* max/min (kernels.zig:254-267, pick at :300-302): the first vector is the
 * accumulator, lanewise max over full vectors, lanes left to right, then the
 * scalar tail as pick(src[i], best); NaN propagates. */
static inline float pick_max(float a, float b) { return (b != b) ? b : (b > a ? b : a); }
static inline float pick_min(float a, float b) { return (b != b) ? b : (b < a ? b : a); }
static inline float vmaxf(float a, float b) { return a > b ? a : (b > a ? b : (a != a ? a : b)); }
static inline float vminf(float a, float b) { return a < b ? a : (b < a ? b : (a != a ? a : b)); }
ZO_EXPORT float zo_reduce_maxmin_f32(const float *src, size_t n, int is_max) {
    if (n >= 8) {
        float first[8];
        memcpy(first, src, sizeof first);
        size_t i = 8;
        for (; i + 8 <= n; i += 8)
            for (int l = 0; l < 8; l++)
                first[l] = is_max ? vmaxf(first[l], src[i + l]) : vminf(first[l], src[i + l]);
        float best = first[0];
        for (int l = 1; l < 8; l++) best = is_max ? pick_max(best, first[l]) : pick_min(best, first[l]);
        for (; i < n; i++) best = is_max ? pick_max(src[i], best) : pick_min(src[i], best);
        return best;
    }
    float best = is_max ? -INFINITY : INFINITY;
    for (size_t i = 0; i < n; i++) best = is_max ? pick_max(best, src[i]) : pick_min(best, src[i]);
    return best;
}

/* A plain f64 left-to-right sum of f32 data: the accuracy reference the
 * GPU's (re-associated) sums are held to. */
ZO_EXPORT double zo_sum_f64_of_f32(const float *src, size_t n) {
    double s = 0.0;
    for (size_t i = 0; i < n; i++) s += (double)src[i];
    return s;
}
ZO_EXPORT double zo_abssum_f64_of_f32(const float *src, size_t n) {
    double s = 0.0;
    for (size_t i = 0; i < n; i++) s += fabs((double)src[i]);
    return s;
}

/* ------------------------------------------------------------------------ */
/* Elementwise semantics: src/zpu/scalar.zig:178-302, kernels.zig:60-206     */
/* ------------------------------------------------------------------------ */

/* Primitive codes shared with the product's region descriptor (the enum
 * order of src/zpu/prims.zig:9-109 for the element-wise subset). */
enum {
    P_NEG = 0, P_ABS, P_EXP, P_EXPM1, P_LOG, P_LOG1P, P_SQRT, P_RSQRT, P_SQUARE, P_RECIP,
    P_CBRT, P_SIN, P_COS, P_TAN, P_ASIN, P_ACOS, P_ATAN, P_SINH, P_COSH, P_TANH, P_ASINH,
    P_ACOSH, P_ATANH, P_ERF, P_SIGMOID, P_SOFTPLUS, P_RELU, P_FLOOR, P_CEIL, P_ROUND,
    P_TRUNC, P_SIGN,
    P_ADD = 35, P_SUB, P_MUL, P_DIV, P_POW, P_MAXIMUM, P_MINIMUM, P_ATAN2, P_HYPOT, P_MOD
};

/* scalar.zig:74-134: zpu's own erf (Maclaurin series below 1, Lentz
 * continued fraction for erfc above). */
static double erf_series(double x) {
    const double two_over_sqrt_pi = 1.1283791670955125738961589031215;
    double sum = 0, term = x, x2 = x * x;
    for (unsigned n = 0; n < 200; n++) {
        double fn = (double)n;
        double add = term / (2.0 * fn + 1.0);
        sum += add;
        term *= -x2 / (fn + 1.0);
        if (fabs(add) < 1e-19) break;
    }
    return two_over_sqrt_pi * sum;
}
static double erfc_cf(double z) {
    const double a = 0.5, x = z * z, fpmin = 1e-300;
    double b = x + 1.0 - a, c = 1.0 / fpmin, d = 1.0 / b, h = d;
    for (unsigned i = 1; i <= 300; i++) {
        double fi = (double)i;
        double an = -fi * (fi - a);
        b += 2.0;
        d = an * d + b;
        if (fabs(d) < fpmin) d = fpmin;
        c = b + an / c;
        if (fabs(c) < fpmin) c = fpmin;
        d = 1.0 / d;
        double del = d * c;
        h *= del;
        if (fabs(del - 1.0) < 1e-16) break;
    }
    /* Q(1/2, x) = exp(-x + a log x - lgamma(1/2)) * h, lgamma(1/2) = log(sqrt(pi)) */
    return exp(-x + a * log(x) - 0.5723649429247000871) * h;
}
static double zo_erf(double x) {
    if (x != x) return x;
    double ax = fabs(x);
    if (ax < 1.0) { double v = erf_series(ax); return x < 0 ? -v : v; }
    double v = 1.0 - erfc_cf(ax);
    return x < 0 ? -v : v;
}

/* scalar.unaryF (scalar.zig:178-212): the f64 definition of each primitive. */
static double unary_f64(int p, double x) {
    switch (p) {
    case P_NEG: return -x;
    case P_ABS: return fabs(x);
    case P_EXP: return exp(x);
    case P_EXPM1: return expm1(x);
    case P_LOG: return log(x);
    case P_LOG1P: return log1p(x);
    case P_SQRT: return sqrt(x);
    case P_RSQRT: return 1.0 / sqrt(x);
    case P_SQUARE: return x * x;
    case P_RECIP: return 1.0 / x;
    case P_CBRT: return cbrt(x);
    case P_SIN: return sin(x);
    case P_COS: return cos(x);
    case P_TAN: return tan(x);
    case P_ASIN: return asin(x);
    case P_ACOS: return acos(x);
    case P_ATAN: return atan(x);
    case P_SINH: return sinh(x);
    case P_COSH: return cosh(x);
    case P_TANH: return tanh(x);
    case P_ASINH: return asinh(x);
    case P_ACOSH: return acosh(x);
    case P_ATANH: return atanh(x);
    case P_ERF: return zo_erf(x);
    case P_SIGMOID: return 1.0 / (1.0 + exp(-x));
    case P_SOFTPLUS: return fmax(x, 0.0) + log1p(exp(-fabs(x))); /* scalar.zig:143-146 */
    case P_RELU: return x > 0 ? x : 0;
    case P_FLOOR: return floor(x);
    case P_CEIL: return ceil(x);
    case P_ROUND: return round(x);
    case P_TRUNC: return trunc(x);
    case P_SIGN: return x > 0 ? 1.0 : (x < 0 ? -1.0 : 0.0);
    default: return NAN;
    }
}

/* kernels.applyUnary (kernels.zig:72-100): the f32 vector form, used by zpu
 * instead of the f64 scalar path whenever hasVectorForm (kernels.zig:60-67)
 * holds.  Everything else (tanh, erf, expm1, ...) is f64 then rounded. */
static int has_vector_form(int p) {
    switch (p) {
    case P_NEG: case P_ABS: case P_EXP: case P_LOG: case P_SQRT: case P_RSQRT: case P_SQUARE:
    case P_RECIP: case P_SIN: case P_COS: case P_TAN: case P_FLOOR: case P_CEIL: case P_ROUND:
    case P_TRUNC: case P_RELU: case P_SIGMOID: case P_SIGN:
        return 1;
    default: return 0;
    }
}
static float unary_vec_f32(int p, float x) {
    switch (p) {
    case P_NEG: return -x;
    case P_ABS: return fabsf(x);
    case P_EXP: return expf(x);
    case P_LOG: return logf(x);
    case P_SQRT: return sqrtf(x);
    case P_RSQRT: return 1.0f / sqrtf(x);
    case P_SQUARE: return x * x;
    case P_RECIP: return 1.0f / x;
    case P_SIN: return sinf(x);
    case P_COS: return cosf(x);
    case P_TAN: return tanf(x);
    case P_FLOOR: return floorf(x);
    case P_CEIL: return ceilf(x);
    case P_ROUND: return roundf(x);
    case P_TRUNC: return truncf(x);
    case P_RELU: return x > 0.0f ? x : 0.0f;
    case P_SIGMOID: return 1.0f / (1.0f + expf(-x));
    case P_SIGN: return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f);
    default: return NAN;
    }
}

/* ops.unaryKernel on contiguous f32 (ops.zig:157-177): vector form when it
 * exists, otherwise scalar.unary = (f32)unaryF((f64)x) (scalar.zig:262-266). */
ZO_EXPORT float zo_unary_f32(int p, float x) {
    if (has_vector_form(p)) return unary_vec_f32(p, x);
    return (float)unary_f64(p, (double)x);
}
ZO_EXPORT double zo_unary_f64(int p, double x) { return unary_f64(p, x); }

static double go_pow(double x, double y);

/* scalar.binaryF (scalar.zig:214-228) rounded to f32; for + - * / the vector
 * form (kernels.zig:141-150) gives the same bits (f64 is wide enough that the
 * double rounding is innocuous). */
static double binary_f64(int p, double a, double b) {
    switch (p) {
    case P_ADD: return a + b;
    case P_SUB: return a - b;
    case P_MUL: return a * b;
    case P_DIV: return a / b;
    case P_POW: return go_pow(a, b); /* scalar.zig:152-154 -> std.math.pow */
    case P_MAXIMUM: return (a != a) ? a : ((b != b) ? b : (a > b ? a : b));
    case P_MINIMUM: return (a != a) ? a : ((b != b) ? b : (a < b ? a : b));
    case P_ATAN2: return atan2(a, b);
    case P_HYPOT: return hypot(a, b);
    case P_MOD: { /* scalar.zig:155-160: truncated remainder, sign of b */
        if (b == 0) return NAN;
        double r = fmod(a, b);
        if (r != 0 && ((r < 0) != (b < 0))) r += b;
        return r;
    }
    default: return NAN;
    }
}
ZO_EXPORT float zo_binary_f32(int p, float a, float b) {
    switch (p) {
    case P_ADD: return a + b;
    case P_SUB: return a - b;
    case P_MUL: return a * b;
    case P_DIV: return a / b;
    default: return (float)binary_f64(p, (double)a, (double)b);
    }
}
ZO_EXPORT double zo_binary_f64(int p, double a, double b) { return binary_f64(p, a, b); }

/* ------------------------------------------------------------------------ */
/* zpu's CPU threading model: src/zpu/parallel.zig:16-37                     */
/* ------------------------------------------------------------------------ */

static size_t g_cores = 0;
ZO_EXPORT void zo_set_cores(size_t cores) { g_cores = cores; }
static size_t cpu_cores(void) {
    if (g_cores) return g_cores;
    long c = sysconf(_SC_NPROCESSORS_ONLN);
    return c > 0 ? (size_t)c : 1;
}
/* parallel.workerCount (parallel.zig:22-27). */
ZO_EXPORT size_t zo_worker_count(size_t n) {
    if (n < 64000) return 1;
    size_t by_size = n / 16000;
    if (by_size < 1) by_size = 1;
    size_t c = cpu_cores();
    return c < by_size ? c : by_size;
}

typedef struct {
    float *dst;
    const float *a, *b;
    size_t start, end;
    int prim;
} bin_job;
static void *bin_worker(void *arg) {
    bin_job *j = (bin_job *)arg;
    for (size_t i = j->start; i < j->end; i++) j->dst[i] = zo_binary_f32(j->prim, j->a[i], j->b[i]);
    return NULL;
}
/* kernels.binaryParallel (kernels.zig:664-721): spawn-per-call workers over
 * parallel.chunkRange (parallel.zig:31-37). */
static void binary_parallel_f32(int prim, float *dst, const float *a, const float *b, size_t n) {
    size_t w = n >= 64000 ? zo_worker_count(n) : 1;
    if (w <= 1) {
        for (size_t i = 0; i < n; i++) dst[i] = zo_binary_f32(prim, a[i], b[i]);
        return;
    }
    pthread_t th[256];
    bin_job jobs[256];
    if (w > 256) w = 256;
    size_t base = n / w, rem = n % w;
    for (size_t i = 0; i < w; i++) {
        size_t start = i < rem ? (base + 1) * i : base * i + rem;
        size_t end = i < rem ? start + base + 1 : start + base;
        jobs[i] = (bin_job){dst, a, b, start, end, prim};
        pthread_create(&th[i], NULL, bin_worker, &jobs[i]);
    }
    for (size_t i = 0; i < w; i++) pthread_join(th[i], NULL);
}

/* ------------------------------------------------------------------------ */
/* The jit chain y = sumAll(tanh(x*x)*a + b) as jit.Plan.runAll executes it  */
/* (jit.zig:99-126 -> ops.applyPrim per step, every intermediate in memory). */
/* ------------------------------------------------------------------------ */

/* Step by step, with zpu's dispatch:
 *   mul(x,x)  -> binaryKernel fast_a&fast_b -> binaryParallel  (ops.zig:207-217)
 *   tanh      -> unaryKernel -> unaryParallel -> no vector form -> scalar
 *                (f32)tanh((f64)v), single thread          (kernels.zig:603-608)
 *   mul(.,a)  -> binaryScalarFast, single thread           (ops.zig:222-225)
 *   add(.,b)  -> binaryScalarFast, single thread
 *   sumAll    -> reduceAll f32 order                       (ops.zig:820-869)
 * `t_out`, when not NULL, receives the pre-reduction vector tanh(x*x)*a+b.
 * Returns zpu's f32 sum; *sum64 gets the f64 sum of the same vector. */
ZO_EXPORT float zo_jit_chain_tanh_sq_affine_sum(const float *x, size_t n, float a, float b,
                                                float *t_out, double *sum64) {
    float *t1 = (float *)malloc(n * sizeof(float) + 64);
    float *t2 = (float *)malloc(n * sizeof(float) + 64);
    if (!t1 || !t2) { free(t1); free(t2); return NAN; }
    binary_parallel_f32(P_MUL, t1, x, x, n);
    for (size_t i = 0; i < n; i++) t2[i] = (float)tanh((double)t1[i]);
    for (size_t i = 0; i < n; i++) t1[i] = t2[i] * a;
    for (size_t i = 0; i < n; i++) t2[i] = t1[i] + b;
    float s = zo_reduce_sum_f32(t2, n);
    if (sum64) *sum64 = zo_sum_f64_of_f32(t2, n);
    if (t_out) memcpy(t_out, t2, n * sizeof(float));
    free(t1);
    free(t2);
    return s;
}

/* ------------------------------------------------------------------------ */
/* Adam: src/zpu/optim.zig:149-265, std.math.pow restated                    */
/* ------------------------------------------------------------------------ */

/* Zig's std.math.pow(f64), which scalar.zig:151-153 calls, restated branch
 * for branch (it follows Go's math.Pow): the special values of x and y, a
 * half power as sqrt, then the integer part of |y| by repeated squaring of
 * frexp(x)'s mantissa with a separately tracked binary exponent, the
 * fractional part (if any) through exp(yf*log(x)), and one ldexp. */
static int odd_integer(double x) {
    if (fabs(x) >= 9007199254740992.0) return 0; /* 2^53 */
    double ip;
    double fp = modf(x, &ip);
    return fp == 0.0 && (((long long)ip) & 1) == 1;
}
static double go_pow(double x, double y) {
    for (int pass = 0; pass < 2; pass++) {
        if (y == 0.0 || x == 1.0) return 1.0;
        if (x != x || y != y) return NAN;
        if (y == 1.0) return x;
        if (x == 0.0) {
            if (y < 0.0) return odd_integer(y) ? copysign(INFINITY, x) : INFINITY;
            return odd_integer(y) ? x : 0.0;
        }
        if (isinf(y)) {
            if (x == -1.0) return 1.0;
            return ((fabs(x) < 1.0) == (y > 0.0)) ? 0.0 : INFINITY;
        }
        if (!isinf(x)) break;
        if (x > 0.0) return y < 0.0 ? 0.0 : INFINITY;
        x = 1.0 / x; /* pow(-inf, y) = pow(-0, -y) */
        y = -y;
    }
    if (y == 0.5) return sqrt(x);
    if (y == -0.5) return 1.0 / sqrt(x);
    double yi;
    double yf = modf(fabs(y), &yi);
    if (yf != 0.0 && x < 0.0) return NAN;
    if (yi >= 9.223372036854775808e18) return exp(y * log(x));
    double a1 = 1.0;
    int ae = 0;
    if (yf != 0.0) {
        if (yf > 0.5) { yf -= 1.0; yi += 1.0; }
        a1 = exp(yf * log(x));
    }
    int xe;
    double x1 = frexp(x, &xe);
    for (long long i = (long long)yi; i != 0; i >>= 1) {
        if (xe < -(1 << 12) || (1 << 12) < xe) { ae += xe; break; }
        if (i & 1) { a1 *= x1; ae += xe; }
        x1 *= x1;
        xe <<= 1;
        if (x1 < 0.5) { x1 += x1; xe--; }
    }
    if (y < 0) { a1 = 1.0 / a1; ae = -ae; }
    return ldexp(a1, ae);
}
ZO_EXPORT double zo_pow(double x, double y) { return go_pow(x, y); }

/* One Adam.step (optim.zig:183-259) on one parameter with f32 moment state,
 * for f32 params and f32 grads: every op is an f32 op (mulScalar rounds its
 * constant to f32, ops.zig:335-345), and subInPlace is an f64 subtract
 * rounded back to f32 (optim.zig:20-31), i.e. an f32 subtract. */
ZO_EXPORT void zo_adam_step_f32(float *p, const float *g, float *m, float *v, size_t n, long t,
                                double lr, double beta1, double beta2, double eps) {
    const double bc1 = 1.0 - go_pow(beta1, (double)t);
    const double bc2 = 1.0 - go_pow(beta2, (double)t);
    const float b1 = (float)beta1, omb1 = (float)(1.0 - beta1);
    const float b2 = (float)beta2, omb2 = (float)(1.0 - beta2);
    const float fb1 = (float)bc1, fb2 = (float)bc2, feps = (float)eps, flr = (float)lr;
    for (size_t i = 0; i < n; i++) {
        float nm = m[i] * b1 + g[i] * omb1;          /* m1 + m2, each product rounded */
        float sq = g[i] * g[i];
        float nv = v[i] * b2 + sq * omb2;
        m[i] = nm;
        v[i] = nv;
        float mhat = nm / fb1;
        float vhat = nv / fb2;
        float den = sqrtf(vhat) + feps;
        float upd = mhat / den;
        float delta = upd * flr;
        p[i] = p[i] - delta;
    }
}

/* The same step for f64 params and f64 grads (the reference's snapshot
 * case): products with the f32 state are taken in f32 (m1 = m*0.9f), the
 * f64 grad terms in f64, their sum is promoted to f64 (ops.binaryKernelF64),
 * copyInto rounds the new moments to f32 (optim.zig:261-265), but this
 * step's update uses the unrounded f64 moments. */
ZO_EXPORT void zo_adam_step_f64(double *p, const double *g, float *m, float *v, size_t n, long t,
                                double lr, double beta1, double beta2, double eps) {
    const double bc1 = 1.0 - go_pow(beta1, (double)t);
    const double bc2 = 1.0 - go_pow(beta2, (double)t);
    const float b1 = (float)beta1, b2 = (float)beta2;
    for (size_t i = 0; i < n; i++) {
        float m1 = m[i] * b1;
        double m2 = g[i] * (1.0 - beta1);
        double nm = (double)m1 + m2;
        m[i] = (float)nm;
        double sq = g[i] * g[i];
        float v1 = v[i] * b2;
        double v2 = sq * (1.0 - beta2);
        double nv = (double)v1 + v2;
        v[i] = (float)nv;
        double mhat = nm / bc1;
        double vhat = nv / bc2;
        double den = sqrt(vhat) + eps;
        double upd = mhat / den;
        double delta = upd * lr;
        p[i] = p[i] - delta;
    }
}

/* ------------------------------------------------------------------------ */
/* MLP train step: nn.dense (nn.zig:190), tanh, sparseCrossEntropy           */
/* (nn.zig:123-134, ops.logSoftmax ops.zig:998-1010), reverse sweep          */
/* (autodiff.zig:323-330 tanh, :451 sum, :480-487 matmul, :51 unbroadcast),  */
/* then Adam per parameter.                                                  */
/* ------------------------------------------------------------------------ */

/* a [r,c] -> at [c,r] (what toContiguous of a swapLastTwo view produces,
 * tensor.zig:395-404). */
static void transpose_f32(const float *a, float *at, size_t r, size_t c) {
    for (size_t i = 0; i < r; i++)
        for (size_t j = 0; j < c; j++) at[j * r + i] = a[i * c + j];
}

/* The MLP layout: W_l is [in_l, out_l] row-major (x @ W), b_l is [out_l].
 * params = {W1, b1, W2, b2, W3, b3}, grads the same shapes.  Runs the
 * forward pass, the backward pass (gradients of the mean NLL over the batch,
 * f32 throughout with zpu's bit-exact gemm for every product, transposed
 * operands materialised as zpu does), and returns the loss.  `grads` receives
 * the gradients; no optimiser step here. */
ZO_EXPORT float zo_mlp_loss_grad(const float *X, const int64_t *labels, size_t B,
                                 size_t d0, size_t d1, size_t d2, size_t d3,
                                 const float *W1, const float *b1, const float *W2,
                                 const float *b2, const float *W3, const float *b3,
                                 float *gW1, float *gb1, float *gW2, float *gb2,
                                 float *gW3, float *gb3) {
    float *z1 = malloc(B * d1 * 4), *a1 = malloc(B * d1 * 4);
    float *z2 = malloc(B * d2 * 4), *a2 = malloc(B * d2 * 4);
    float *lg = malloc(B * d3 * 4);
    /* forward: dense = matmul + broadcast add; tanh via f64 (no vector form) */
    gemm_f32(X, W1, z1, B, d0, d1);
    for (size_t i = 0; i < B; i++)
        for (size_t j = 0; j < d1; j++) {
            float z = z1[i * d1 + j] + b1[j];
            z1[i * d1 + j] = z;
            a1[i * d1 + j] = (float)tanh((double)z);
        }
    gemm_f32(a1, W2, z2, B, d1, d2);
    for (size_t i = 0; i < B; i++)
        for (size_t j = 0; j < d2; j++) {
            float z = z2[i * d2 + j] + b2[j];
            z2[i * d2 + j] = z;
            a2[i * d2 + j] = (float)tanh((double)z);
        }
    gemm_f32(a2, W3, lg, B, d2, d3);
    for (size_t i = 0; i < B; i++)
        for (size_t j = 0; j < d3; j++) lg[i * d3 + j] = lg[i * d3 + j] + b3[j];

    /* logSoftmax over the last axis: m = max, s = x - m, e = exp(s) (f32
     * vector form), z = sum(e) (reduceRows order), lp = s - log(z) */
    float *s = malloc(B * d3 * 4), *e = malloc(B * d3 * 4), *lp = malloc(B * d3 * 4);
    float *zs = calloc(B, 4), *mx = calloc(B, 4), *nll = calloc(B, 4);
    for (size_t i = 0; i < B; i++) {
        const float *row = lg + i * d3;
        mx[i] = zo_reduce_maxmin_f32(row, d3, 1);
        for (size_t j = 0; j < d3; j++) {
            s[i * d3 + j] = row[j] - mx[i];
            e[i * d3 + j] = expf(s[i * d3 + j]);
        }
        zs[i] = zo_reduce_sum_f32(e + i * d3, d3);
        float lz = logf(zs[i]);
        for (size_t j = 0; j < d3; j++) lp[i * d3 + j] = s[i * d3 + j] - lz;
    }
    /* picked = lp * onehot; nll = sum(picked, -1); loss = -(sum(nll) * (1/B)) */
    float *pk = malloc(B * d3 * 4);
    for (size_t i = 0; i < B; i++) {
        for (size_t j = 0; j < d3; j++)
            pk[i * d3 + j] = lp[i * d3 + j] * ((int64_t)j == labels[i] ? 1.0f : 0.0f);
        nll[i] = zo_reduce_sum_f32(pk + i * d3, d3);
    }
    const float invB = (float)(1.0 / (double)B);
    float loss = -(zo_reduce_sum_f32(nll, B) * invB);

    /* backward.  neg -> -1; mul by 1/B -> -1/B; sum -> broadcast;
     * mul(lp, oh) -> g_lp = g*oh; sub(s, lz) -> g_s = g_lp, g_lz = -sum(g_lp);
     * log -> g_z = g_lz / z; sum -> broadcast; exp -> g_s += g_e * e;
     * sub(x, m) -> g_x = g_s, g_m = -sum(g_s); max -> g_x += g_m*mask/count. */
    float *gl = malloc(B * d3 * 4);
    const float gmean = -1.0f * invB;
    for (size_t i = 0; i < B; i++) {
        float glp[64], gs[64];
        float sum_glp = 0.0f;
        for (size_t j = 0; j < d3; j++) {
            glp[j] = gmean * ((int64_t)j == labels[i] ? 1.0f : 0.0f);
            sum_glp = sum_glp + glp[j];
        }
        float gz = (-sum_glp) / zs[i];
        float sum_gs = 0.0f;
        for (size_t j = 0; j < d3; j++) {
            gs[j] = glp[j] + gz * e[i * d3 + j];
            sum_gs = sum_gs + gs[j];
        }
        float cnt = 0.0f;
        for (size_t j = 0; j < d3; j++) cnt += (lg[i * d3 + j] == mx[i]) ? 1.0f : 0.0f;
        float gm = -sum_gs;
        for (size_t j = 0; j < d3; j++) {
            float share = ((lg[i * d3 + j] == mx[i]) ? 1.0f : 0.0f) / cnt;
            gl[i * d3 + j] = gs[j] + gm * share;
        }
    }
    /* layer 3: g_b3 = column sums (ops.sum axis 0, generic row-order walk),
     * g_W3 = a2^T @ gl, g_a2 = gl @ W3^T */
    float *ta = malloc((d1 > d2 ? d1 : d2) * B * 4);
    float *tw = malloc((d1 * d2 > d2 * d3 ? d1 * d2 : d2 * d3) * 4 + (d0 * d1) * 0 + 64);
    float *ga2 = malloc(B * d2 * 4), *ga1 = malloc(B * d1 * 4);
    for (size_t j = 0; j < d3; j++) gb3[j] = 0.0f;
    for (size_t i = 0; i < B; i++)
        for (size_t j = 0; j < d3; j++) gb3[j] = gb3[j] + gl[i * d3 + j];
    transpose_f32(a2, ta, B, d2);
    gemm_f32(ta, gl, gW3, d2, B, d3);
    transpose_f32(W3, tw, d2, d3);
    gemm_f32(gl, tw, ga2, B, d3, d2);
    /* tanh VJP: g * (1 - y^2) */
    for (size_t i = 0; i < B * d2; i++) {
        float y2 = a2[i] * a2[i];
        ga2[i] = ga2[i] * (1.0f - y2);
    }
    for (size_t j = 0; j < d2; j++) gb2[j] = 0.0f;
    for (size_t i = 0; i < B; i++)
        for (size_t j = 0; j < d2; j++) gb2[j] = gb2[j] + ga2[i * d2 + j];
    transpose_f32(a1, ta, B, d1);
    gemm_f32(ta, ga2, gW2, d1, B, d2);
    transpose_f32(W2, tw, d1, d2);
    gemm_f32(ga2, tw, ga1, B, d2, d1);
    for (size_t i = 0; i < B * d1; i++) {
        float y2 = a1[i] * a1[i];
        ga1[i] = ga1[i] * (1.0f - y2);
    }
    for (size_t j = 0; j < d1; j++) gb1[j] = 0.0f;
    for (size_t i = 0; i < B; i++)
        for (size_t j = 0; j < d1; j++) gb1[j] = gb1[j] + ga1[i * d1 + j];
    float *tx = malloc(B * d0 * 4);
    transpose_f32(X, tx, B, d0);
    gemm_f32(tx, ga1, gW1, d0, B, d1);

    free(z1); free(a1); free(z2); free(a2); free(lg); free(s); free(e); free(lp);
    free(zs); free(mx); free(nll); free(pk); free(gl); free(ta); free(tw); free(ga2);
    free(ga1); free(tx);
    return loss;
}
