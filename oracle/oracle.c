/*
 * CPU oracle for the MX-KMeans Lloyd iteration -- TEST INFRASTRUCTURE ONLY.
 * See oracle.h for what it restates and who may call it.
 *
 * Build: oracle/Makefile (gcc -O3 -ffp-contract=off).  Floating-point
 * contraction is disabled so that every multiply-add is written out: where the
 * reference's CUDA source is compiled by nvcc with its default -fmad=true, a
 * `s += a * b` becomes one fused multiply-add, and the restatement below uses
 * fmaf() at exactly those places.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------------- */
/* small parallel-for over [0, n) with pthreads                               */

typedef void (*range_fn)(int64_t begin, int64_t end, void* ctx);
typedef struct {
    range_fn fn;
    void* ctx;
    int64_t begin, end;
} range_job;

static void* range_thread(void* p) {
    range_job* j = (range_job*)p;
    j->fn(j->begin, j->end, j->ctx);
    return NULL;
}

int orc_hardware_threads(void) {
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

static void parallel_for(int64_t n, int threads, range_fn fn, void* ctx) {
    if (threads <= 0) threads = orc_hardware_threads();
    if (threads > 256) threads = 256;
    if (n < 2 * threads || threads == 1) {
        fn(0, n, ctx);
        return;
    }
    pthread_t tid[256];
    range_job jobs[256];
    int64_t chunk = (n + threads - 1) / threads;
    int started = 0;
    for (int t = 0; t < threads; ++t) {
        int64_t b = t * chunk, e = b + chunk < n ? b + chunk : n;
        if (b >= e) break;
        jobs[t] = (range_job){fn, ctx, b, e};
        if (pthread_create(&tid[t], NULL, range_thread, &jobs[t]) != 0) {
            fn(b, e, ctx);
            jobs[t].fn = NULL;
        }
        started = t + 1;
    }
    for (int t = 0; t < started; ++t)
        if (jobs[t].fn) pthread_join(tid[t], NULL);
}

/* ------------------------------------------------------------------------- */
/* MX element formats.                                                        */
/* The reference's element types are CUTLASS float_e4m3_t / float_e2m3_t /    */
/* float_e2m1_t (include/kmeans.cuh:6-8) and cuda_fp6 __nv_fp6_e3m2           */
/* (src/kernels/quantize.cu:89): IEEE-style encodings converted from FP32 by  */
/* round-to-nearest-even, saturating to the largest finite magnitude.         */

typedef struct {
    int mbits, ebits, bias, sign_shift;
    double maxv;
} fmt_desc;

static const fmt_desc FMTS[4] = {
    {3, 4, 7, 7, 448.0}, /* E4M3 (FN: no inf, 0x7f/0xff NaN) */
    {3, 2, 1, 5, 7.5},   /* E2M3 */
    {1, 2, 1, 3, 6.0},   /* E2M1 */
    {2, 3, 3, 5, 28.0},  /* E3M2 */
};

static inline uint32_t f2u(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    return u;
}
static inline float u2f(uint32_t u) {
    float x;
    memcpy(&x, &u, 4);
    return x;
}

/* UE8M0 scale: the power of two at or above |x| (round toward +inf),
 * saturating at 2^127; values at or below 2^-127 give 2^-127; NaN/Inf give the
 * NaN code 0xff.  This is the rule of cutlass::float_ue8m0_t(float)
 * (cutlass/float8.h:1154-1175, host branch), used by Scale(...) at
 * src/kernels/quantize.cu:9-11. */
static uint8_t ue8m0_encode(float x) {
    if (isnan(x) || isinf(x)) return 0xff;
    uint32_t u = f2u(x);
    uint32_t e = (u >> 23) & 0xff, m = u & 0x7fffff;
    if (m != 0 && e != 0xfe && !(e == 0 && m <= 0x400000)) e += 1;
    return (uint8_t)e;
}

static float ue8m0_decode(uint8_t b) {
    if (b == 0xff) return NAN;
    return ldexpf(1.0f, (int)b - 127);
}

static uint8_t mx_encode(int f, float x) {
    const fmt_desc* d = &FMTS[f];
    uint32_t sign = (f2u(x) >> 31) & 1u;
    uint32_t maxcode = (uint32_t)((((1 << d->ebits) - 1) << d->mbits) | ((1 << d->mbits) - 1));
    if (f == ORC_E4M3) maxcode = 0x7e; /* 0x7f is NaN */
    if (isnan(x)) {
        if (f == ORC_E4M3) return 0x7f;     /* cutlass/float8.h: NaN -> 0x7f */
        if (f == ORC_E3M2) return maxcode;  /* cuda_fp6 __nv_fp6_e3m2: NaN -> +max */
        return (uint8_t)((sign << d->sign_shift) | maxcode); /* exmy_base: signed max */
    }
    double a = fabs((double)x);
    if (isinf(x) || a > d->maxv * 2.0) return (uint8_t)((sign << d->sign_shift) | maxcode);
    if (a == 0.0) return (uint8_t)(sign << d->sign_shift);
    int emin = 1 - d->bias; /* exponent of the smallest normal */
    int e;
    frexp(a, &e);           /* a = f * 2^e, f in [0.5,1) */
    int ex = e - 1;         /* floor(log2 a) */
    if (ex < emin) ex = emin;
    double quantum = ldexp(1.0, ex - d->mbits);
    double q = nearbyint(a / quantum) * quantum; /* default rounding: nearest-even */
    if (q > d->maxv) q = d->maxv;                /* satfinite */
    if (q == 0.0) return (uint8_t)(sign << d->sign_shift);
    /* encode q */
    int qe;
    frexp(q, &qe);
    int qx = qe - 1;
    uint32_t code;
    if (qx < emin) { /* subnormal */
        code = (uint32_t)(q / ldexp(1.0, emin - d->mbits));
    } else {
        uint32_t biased = (uint32_t)(qx + d->bias);
        uint32_t mant = (uint32_t)((q / ldexp(1.0, qx) - 1.0) * (double)(1 << d->mbits));
        code = (biased << d->mbits) | mant;
    }
    return (uint8_t)((sign << d->sign_shift) | code);
}

static float mx_decode(int f, uint8_t b) {
    const fmt_desc* d = &FMTS[f];
    uint32_t sign = (b >> d->sign_shift) & 1u;
    uint32_t mag = b & ((1u << d->sign_shift) - 1);
    if (f == ORC_E4M3 && mag == 0x7f) return NAN;
    uint32_t e = mag >> d->mbits, m = mag & ((1u << d->mbits) - 1);
    double v;
    if (e == 0)
        v = ldexp((double)m, 1 - d->bias - d->mbits);
    else
        v = ldexp(1.0 + (double)m / (double)(1 << d->mbits), (int)e - d->bias);
    return (float)(sign ? -v : v);
}

uint8_t orc_encode(int format, float x) {
    if (format == ORC_UE8M0) return ue8m0_encode(x);
    return mx_encode(format, x);
}

float orc_decode_elem(int format, uint8_t bits) {
    if (format == ORC_UE8M0) return ue8m0_decode(bits);
    return mx_decode(format, bits);
}

void orc_encode_batch(int format, int64_t n, const float* in, uint8_t* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = orc_encode(format, in[i]);
}

void orc_decode_batch(int format, int64_t n, const uint8_t* in, float* out) {
    for (int64_t i = 0; i < n; ++i) out[i] = orc_decode_elem(format, in[i]);
}

static int bits_format(int bits) {
    return bits == 8 ? ORC_E4M3 : bits == 6 ? ORC_E2M3 : ORC_E2M1;
}

/* ------------------------------------------------------------------------- */
/* include/precision.hpp:10-26                                                */

int orc_precision_candidate(float p4, float p6, float lc, int dimensions, float gap) {
    /* delta = p + lc + d*lc: nvcc contracts d*lc + (p + lc) into one FMA. */
    const float delta4 = fmaf((float)dimensions, lc, p4 + lc);
    const float delta6 = fmaf((float)dimensions, lc, p6 + lc);
    if (delta4 / 64.0f <= gap) return 4;
    if (delta6 / 64.0f <= gap) return 6;
    return 8;
}

int orc_select_precision(float p4, float p6, float lc, float ec, int dimensions, float gap) {
    (void)orc_precision_candidate(p4, p6, lc, dimensions, gap);
    (void)ec;
    return 8; /* include/precision.hpp:20-26 discards the candidate */
}

/* ------------------------------------------------------------------------- */
/* src/kernels/assignment.cu:7-16: sequential sum of x*x per row; nvcc fuses   */
/* `sum += x * x` into fmaf(x, x, sum).                                       */

void orc_l2_norm(int64_t rows, int d, const float* x, float* norms) {
    for (int64_t r = 0; r < rows; ++r) {
        float sum = 0.0f;
        const float* row = x + (size_t)r * d;
        for (int j = 0; j < d; ++j) sum = fmaf(row[j], row[j], sum);
        norms[r] = sum;
    }
}

/* ------------------------------------------------------------------------- */
/* src/kernels/quantize.cu:13-72 (kernel) and :111-123 (launcher)             */

int orc_quantize_rows(int bits, int64_t rows, int d, const float* points, const int* pid,
                      uint8_t* values, uint8_t* scales, float* max_errors) {
    if (bits != 4 && bits != 6 && bits != 8) return -2;
    if (rows == 0) return 0;
    if (d % 32) return -2;
    const int fmt = bits_format(bits);
    const float qmax = bits == 8 ? 448.0f : (bits == 6 ? 7.5f : 6.0f); /* quantize.cu:27 */
    const int blocks_per_row = d / 32;
    for (int64_t row = 0; row < rows; ++row) {
        const int64_t src = pid ? pid[row] : row;
        for (int blk = 0; blk < blocks_per_row; ++blk) {
            const float* x = points + (size_t)src * d + blk * 32;
            float amax = 0.0f;
            for (int l = 0; l < 32; ++l) amax = fmaxf(amax, fabsf(x[l])); /* xor-shuffle max */
            const uint8_t s = ue8m0_encode(amax > 0.0f ? amax / qmax : 1.0f);
            const float sf = ue8m0_decode(s);
            uint8_t raw[32];
            float err = 0.0f;
            for (int l = 0; l < 32; ++l) {
                raw[l] = mx_encode(fmt, x[l] / sf);
                const float rec = mx_decode(fmt, raw[l]) * sf;
                const float diff = x[l] - rec;
                err = fmaxf(err, diff * diff);
            }
            const size_t byte_base = ((size_t)row * d + (size_t)blk * 32) * (size_t)bits / 8;
            if (bits == 8) {
                memcpy(values + byte_base, raw, 32);
            } else if (bits == 4) { /* quantize.cu:48-51: low nibble = even feature */
                for (int l = 0; l < 32; l += 2)
                    values[byte_base + l / 2] = (uint8_t)((raw[l] & 0xf) | ((raw[l + 1] & 0xf) << 4));
            } else { /* quantize.cu:53-62: four 6-bit codes in three bytes, LSB first */
                for (int l = 0; l < 32; l += 4) {
                    const unsigned q0 = raw[l], q1 = raw[l + 1], q2 = raw[l + 2], q3 = raw[l + 3];
                    const size_t o = byte_base + (size_t)(l / 4) * 3;
                    values[o] = (uint8_t)((q0 & 0x3f) | ((q1 & 3) << 6));
                    values[o + 1] = (uint8_t)((q1 >> 2) | ((q2 & 0xf) << 4));
                    values[o + 2] = (uint8_t)((q2 >> 4) | (q3 << 2));
                }
            }
            scales[(size_t)row * blocks_per_row + blk] = s;
            if (max_errors && err > max_errors[row]) max_errors[row] = err; /* atomicMax on bits */
        }
    }
    return 0;
}

/* src/kernels/quantize.cu:74-98: per-point FP4 (E2M1) and FP6 (E3M2!) block
 * errors over features 1..31 of each 32-block; `upper` in 96-float tiles per 32
 * points: [norm, norm + d*e6^2, norm + d*e4^2]. */
void orc_point_bounds(int64_t n, int d, const float* points, const float* norms, float* upper) {
    for (int64_t p = 0; p < n; ++p) {
        float e4 = 0.0f, e6 = 0.0f;
        const float* x = points + (size_t)p * d;
        for (int base = 0; base < d; base += 32) {
            float amax = 0.0f;
            for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[base + j]));
            const float s4 = ue8m0_decode(ue8m0_encode(amax > 0.0f ? amax / 6.0f : 1.0f));
            const float s6 = ue8m0_decode(ue8m0_encode(amax > 0.0f ? amax / 7.5f : 1.0f));
            for (int j = 1; j < 32; ++j) {
                const float v = x[base + j];
                const float q4 = mx_decode(ORC_E2M1, mx_encode(ORC_E2M1, v / s4));
                const float q6 = mx_decode(ORC_E3M2, mx_encode(ORC_E3M2, v / s6));
                e4 = fmaxf(e4, fabsf(fmaf(q4, s4, -v)));
                e6 = fmaxf(e6, fabsf(fmaf(q6, s6, -v)));
            }
        }
        const size_t tile = (size_t)(p / 32) * 96;
        const int lane = (int)(p % 32);
        upper[tile + lane] = norms[p];
        upper[tile + 32 + lane] = fmaf((float)d * e6, e6, norms[p]);
        upper[tile + 64 + lane] = fmaf((float)d * e4, e4, norms[p]);
    }
}

/* policy 0: select_precision (the reference); 1: the candidate it discards,
 * the library's test hook mxk_set_precision_policy(1). */
static void assign_precisions_policy(int64_t n, int d, const float* upper, const float* gaps, float lc,
                                     float ec, int* precision, int policy) {
    for (int64_t p = 0; p < n; ++p) {
        const size_t tile = (size_t)(p / 32) * 96;
        const int lane = (int)(p % 32);
        precision[p] = policy ? orc_precision_candidate(upper[tile + 64 + lane], upper[tile + 32 + lane], lc, d,
                                                        gaps[p])
                              : orc_select_precision(upper[tile + 64 + lane], upper[tile + 32 + lane], lc, ec, d,
                                                     gaps[p]);
    }
}

void orc_assign_precisions(int64_t n, int d, const float* upper, const float* gaps, float lc,
                           float ec, int* precision) {
    assign_precisions_policy(n, d, upper, gaps, lc, ec, precision, 0);
}

/* ------------------------------------------------------------------------- */
/* tests/cuda_checks.cu:23-33: generic bit-offset unpacking of packed rows.   */

float orc_decode_packed(const uint8_t* bytes, const uint8_t* scales, int bits, int64_t row, int d,
                        int feature) {
    const size_t bit_offset = ((size_t)row * d + feature) * (size_t)bits;
    const size_t byte = bit_offset / 8;
    unsigned raw = bytes[byte];
    if ((bit_offset % 8) + bits > 8) raw |= (unsigned)bytes[byte + 1] << 8;
    raw = (raw >> (bit_offset % 8)) & ((1u << bits) - 1);
    const float q = mx_decode(bits_format(bits), (uint8_t)raw);
    return q * ue8m0_decode(scales[(size_t)row * (d / 32) + feature / 32]);
}

void orc_dequantize_rows(int bits, int64_t rows, int d, const uint8_t* bytes, const uint8_t* scales,
                         float* out) {
    for (int64_t r = 0; r < rows; ++r)
        for (int f = 0; f < d; ++f) out[(size_t)r * d + f] = orc_decode_packed(bytes, scales, bits, r, d, f);
}

typedef struct {
    int64_t n;
    int k;
    const float *a, *b;
    double* out;
    double* mag;
} gemm_ctx;

static void gemm_rows(int64_t begin, int64_t end, void* p) {
    gemm_ctx* c = (gemm_ctx*)p;
    for (int64_t i = begin; i < end; ++i) {
        const float* ar = c->a + (size_t)i * c->k;
        for (int64_t j = 0; j < c->n; ++j) {
            const float* br = c->b + (size_t)j * c->k;
            double s = 0.0, m = 0.0;
            for (int f = 0; f < c->k; ++f) {
                const double prod = (double)ar[f] * (double)br[f];
                s += prod;
                m += fabs(prod);
            }
            c->out[(size_t)i * c->n + j] = s;
            if (c->mag) c->mag[(size_t)i * c->n + j] = m;
        }
    }
}

void orc_gemm_mx(int bits, int64_t m, int64_t n, int k, const uint8_t* a, const uint8_t* a_scales,
                 const uint8_t* b, const uint8_t* b_scales, double* out, double* magnitude) {
    float* ad = (float*)malloc(sizeof(float) * (size_t)m * k);
    float* bd = (float*)malloc(sizeof(float) * (size_t)n * k);
    orc_dequantize_rows(bits, m, k, a, a_scales, ad);
    orc_dequantize_rows(8, n, k, b, b_scales, bd);
    gemm_ctx c = {n, k, ad, bd, out, magnitude};
    parallel_for(m, 0, gemm_rows, &c);
    free(ad);
    free(bd);
}

void orc_gemm_f32(int64_t m, int64_t n, int k, const float* a, const float* b, double* out) {
    gemm_ctx c = {n, k, a, b, out, NULL};
    parallel_for(m, 0, gemm_rows, &c);
}

/* ------------------------------------------------------------------------- */
/* src/kernels/assignment.cu:19-57 and include/precision.hpp:29-48            */

static inline void insert_largest(float v, float* first, float* second) {
    if (v > *first) {
        *second = *first;
        *first = v;
    } else if (v > *second) {
        *second = v;
    }
}

static inline void insert_distance(float v, int index, float* first, float* second, int* nearest) {
    if (v < *first || (v == *first && index < *nearest)) {
        *second = *first;
        *first = v;
        *nearest = index;
    } else if (v < *second) {
        *second = v;
    }
}

void orc_assign_clusters(int64_t rows, int k, const float* point_norms, const float* centroid_norms,
                         const float* dots, const int* pid, int* labels, float* gaps) {
    for (int64_t row = 0; row < rows; ++row) {
        const int64_t point = pid ? pid[row] : row;
        float first = INFINITY, second = INFINITY;
        float largest = pid ? -1e38f : -1.0f; /* assignment.cu:27 */
        float next_largest = largest;
        int best = 0x7fffffff;
        for (int c = 0; c < k; ++c) {
            const float dist = fmaf(-2.0f, dots[(size_t)row * k + c], point_norms[point] + centroid_norms[c]);
            insert_distance(dist, c, &first, &second, &best);
            insert_largest(dist, &largest, &next_largest);
        }
        labels[point] = best;
        if (gaps) gaps[point] = largest - next_largest;
    }
}

void orc_top2(int64_t rows, int k, const float* point_norms, const float* centroid_norms,
              const float* dots, int* nearest, float* first_out, float* second_out) {
    for (int64_t row = 0; row < rows; ++row) {
        float first = INFINITY, second = INFINITY;
        int best = 0x7fffffff;
        for (int c = 0; c < k; ++c) {
            const float dist = fmaf(-2.0f, dots[(size_t)row * k + c], point_norms[row] + centroid_norms[c]);
            insert_distance(dist, c, &first, &second, &best);
        }
        nearest[row] = best;
        first_out[row] = first;
        second_out[row] = second;
    }
}

/* ------------------------------------------------------------------------- */
/* src/kernels/update.cu:7-61                                                 */

void orc_update_centroids(int64_t n, int d, int k, const float* points, const int* labels,
                          const float* old_centroids, float* centroids, int* counts) {
    memset(centroids, 0, sizeof(float) * (size_t)k * d);
    memset(counts, 0, sizeof(int) * (size_t)k);
    for (int64_t p = 0; p < n; ++p) {
        const int c = labels[p];
        counts[c] += 1;
        for (int f = 0; f < d; ++f) centroids[(size_t)c * d + f] += points[(size_t)p * d + f];
    }
    for (int64_t i = 0; i < (int64_t)k * d; ++i) {
        const int count = counts[i / d];
        /* an empty cluster keeps its previous center (update.cu:26-29) */
        centroids[i] = count ? centroids[i] / (float)count : old_centroids[i];
    }
}

float orc_centroid_shift(int64_t elements, const float* previous, const float* current) {
    float sum = 0.0f;
    for (int64_t i = 0; i < elements; ++i) {
        const float diff = previous[i] - current[i];
        sum += diff * diff;
    }
    return sum;
}

double orc_inertia(int64_t n, int d, const float* points, const float* centroids, const int* labels) {
    double total = 0.0;
    for (int64_t p = 0; p < n; ++p) {
        const float* x = points + (size_t)p * d;
        const float* c = centroids + (size_t)labels[p] * d;
        double s = 0.0;
        for (int f = 0; f < d; ++f) {
            const double diff = (double)x[f] - (double)c[f];
            s += diff * diff;
        }
        total += s;
    }
    return total;
}

/* ------------------------------------------------------------------------- */
/* Lloyd loop of src/kmeans.cu:12-68                                          */

typedef struct {
    int64_t n;
    int d, k;
    const float* x;      /* dequantized or raw point rows */
    const float* c;      /* dequantized or raw centroid rows */
    const float* pn;     /* point norms */
    const float* cn;     /* centroid norms */
    const int* pid;      /* optional row -> point map */
    int* labels;
    float* gaps;
    float gap_init;
    float* dots_out;     /* optional dense product (float) */
} assign_ctx;

/* Fused product + assignment over a row range: the product of one row with all
 * centroids is accumulated in double and rounded to float (the value a GPU
 * GEMM would hand to assign_clusters), then the assignment rule runs. */
static void assign_rows(int64_t begin, int64_t end, void* p) {
    assign_ctx* a = (assign_ctx*)p;
    float* dots = (float*)malloc(sizeof(float) * (size_t)a->k);
    for (int64_t row = begin; row < end; ++row) {
        const float* xr = a->x + (size_t)row * a->d;
        for (int c = 0; c < a->k; ++c) {
            const float* cr = a->c + (size_t)c * a->d;
            double s = 0.0;
            for (int f = 0; f < a->d; ++f) s += (double)xr[f] * (double)cr[f];
            dots[c] = (float)s;
        }
        if (a->dots_out) memcpy(a->dots_out + (size_t)row * a->k, dots, sizeof(float) * (size_t)a->k);
        const int64_t point = a->pid ? a->pid[row] : row;
        float first = INFINITY, second = INFINITY, largest = a->gap_init, next_largest = a->gap_init;
        int best = 0x7fffffff;
        for (int c = 0; c < a->k; ++c) {
            const float dist = fmaf(-2.0f, dots[c], a->pn[point] + a->cn[c]);
            insert_distance(dist, c, &first, &second, &best);
            insert_largest(dist, &largest, &next_largest);
        }
        a->labels[point] = best;
        if (a->gaps) a->gaps[point] = largest - next_largest;
    }
    free(dots);
}

float orc_lloyd_step(int64_t n, int d, int k, const float* points, const float* point_norms,
                     float* centroids, int* labels, float* dots_out, int threads) {
    float* cn = (float*)malloc(sizeof(float) * (size_t)k);
    float* prev = (float*)malloc(sizeof(float) * (size_t)k * d);
    uint8_t* qc = (uint8_t*)malloc((size_t)k * d);
    uint8_t* sc = (uint8_t*)malloc((size_t)k * (d / 32));
    float* cd = (float*)malloc(sizeof(float) * (size_t)k * d);
    uint8_t* qx = (uint8_t*)malloc((size_t)n * d);
    uint8_t* sx = (uint8_t*)malloc((size_t)n * (d / 32));
    float* xd = (float*)malloc(sizeof(float) * (size_t)n * d);
    int* counts = (int*)malloc(sizeof(int) * (size_t)k);
    memcpy(prev, centroids, sizeof(float) * (size_t)k * d);
    orc_l2_norm(k, d, centroids, cn);
    orc_quantize_rows(8, k, d, centroids, NULL, qc, sc, NULL);
    orc_dequantize_rows(8, k, d, qc, sc, cd);
    orc_quantize_rows(8, n, d, points, NULL, qx, sx, NULL);
    orc_dequantize_rows(8, n, d, qx, sx, xd);
    assign_ctx a = {n, d, k, xd, cd, point_norms, cn, NULL, labels, NULL, -1e38f, dots_out};
    parallel_for(n, threads, assign_rows, &a);
    orc_update_centroids(n, d, k, points, labels, prev, centroids, counts);
    const float shift = orc_centroid_shift((int64_t)k * d, prev, centroids);
    free(cn); free(prev); free(qc); free(sc); free(cd); free(qx); free(sx); free(xd); free(counts);
    return shift;
}

int orc_kmeans_mixed(int64_t n, int d, int k, const float* points, float* centroids, int* labels,
                     int max_iterations, int fp32_iterations, float tolerance, int threads) {
    return orc_kmeans_mixed_ex(n, d, k, points, centroids, labels, max_iterations, fp32_iterations, tolerance,
                               threads, 0, NULL);
}

int orc_kmeans_mixed_ex(int64_t n, int d, int k, const float* points, float* centroids, int* labels,
                        int max_iterations, int fp32_iterations, float tolerance, int threads, int policy,
                        int* group_sizes) {
    if (n <= 0 || d <= 0 || k <= 0 || d % 32 || max_iterations <= 0) return -2;
    float* pn = (float*)malloc(sizeof(float) * (size_t)n);
    float* cn = (float*)malloc(sizeof(float) * (size_t)k);
    float* gaps = (float*)calloc((size_t)n, sizeof(float));
    float* upper = (float*)malloc(sizeof(float) * (size_t)((n + 31) / 32) * 96);
    float* prev = (float*)malloc(sizeof(float) * (size_t)k * d);
    float* errors = (float*)malloc(sizeof(float) * (size_t)k);
    int* precision = (int*)malloc(sizeof(int) * (size_t)n);
    int* ids = (int*)malloc(sizeof(int) * (size_t)n);
    int* counts = (int*)malloc(sizeof(int) * (size_t)k);
    uint8_t* qc = (uint8_t*)malloc((size_t)k * d);
    uint8_t* sc = (uint8_t*)malloc((size_t)k * (d / 32));
    float* cd = (float*)malloc(sizeof(float) * (size_t)k * d);
    uint8_t* qx = (uint8_t*)malloc((size_t)n * d);
    uint8_t* sx = (uint8_t*)malloc((size_t)n * (d / 32));
    float* xd = (float*)malloc(sizeof(float) * (size_t)n * d);
    int result = max_iterations;

    orc_l2_norm(n, d, points, pn);                 /* kmeans.cu:24 */
    orc_point_bounds(n, d, points, pn, upper);     /* kmeans.cu:25 */
    for (int it = 0; it < max_iterations; ++it) {  /* kmeans.cu:28 */
        memcpy(prev, centroids, sizeof(float) * (size_t)k * d);
        orc_l2_norm(k, d, centroids, cn);
        if (it < fp32_iterations) { /* kmeans.cu:31-34 */
            assign_ctx a = {n, d, k, points, centroids, pn, cn, NULL, labels, gaps, -1.0f, NULL};
            parallel_for(n, threads, assign_rows, &a);
        } else { /* kmeans.cu:36-57 */
            memset(errors, 0, sizeof(float) * (size_t)k);
            orc_quantize_rows(8, k, d, centroids, NULL, qc, sc, errors);
            orc_dequantize_rows(8, k, d, qc, sc, cd);
            float emax = errors[0], nmax = cn[0];
            for (int c = 1; c < k; ++c) {
                if (errors[c] > emax) emax = errors[c];
                if (cn[c] > nmax) nmax = cn[c];
            }
            const float ec = sqrtf(emax), lc = sqrtf(nmax);
            assign_precisions_policy(n, d, upper, gaps, lc, ec, precision, policy);
            static const int group_bits[3] = {4, 6, 8};
            for (int g = 0; g < 3; ++g) {
                const int bits = group_bits[g];
                int64_t rows = 0;
                for (int64_t p = 0; p < n; ++p)
                    if (precision[p] == bits) ids[rows++] = (int)p; /* thrust::copy_if, stable */
                if (group_sizes) group_sizes[3 * it + g] = (int)rows;
                if (!rows) continue;
                orc_quantize_rows(bits, rows, d, points, ids, qx, sx, NULL);
                orc_dequantize_rows(bits, rows, d, qx, sx, xd);
                assign_ctx a = {rows, d, k, xd, cd, pn, cn, ids, labels, gaps, -1e38f, NULL};
                parallel_for(rows, threads, assign_rows, &a);
            }
        }
        orc_update_centroids(n, d, k, points, labels, prev, centroids, counts); /* kmeans.cu:62 */
        const float shift = orc_centroid_shift((int64_t)k * d, prev, centroids);
        if (!isfinite(shift)) {
            result = -1;
            break;
        }
        if (shift <= tolerance) {
            result = it + 1;
            break;
        }
    }
    free(pn); free(cn); free(gaps); free(upper); free(prev); free(errors); free(precision); free(ids);
    free(counts); free(qc); free(sc); free(cd); free(qx); free(sx); free(xd);
    return result;
}

/* ------------------------------------------------------------------------- */
/* FP32 Lloyd: the multithreaded CPU baseline.  FP32 dot products of the      */
/* unquantized rows (8 partial sums per product, vectorizable), fmaf distance  */
/* with the lowest-index argmin, sums/counts with empty-cluster keep, shift.   */

typedef struct {
    int64_t n;
    int d, k;
    const float *x, *c, *pn, *cn;
    int* labels;
} f32_ctx;

static void f32_rows(int64_t begin, int64_t end, void* p) {
    f32_ctx* a = (f32_ctx*)p;
    for (int64_t row = begin; row < end; ++row) {
        const float* xr = a->x + (size_t)row * a->d;
        float first = INFINITY;
        int best = 0;
        for (int c = 0; c < a->k; ++c) {
            const float* cr = a->c + (size_t)c * a->d;
            float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            int f = 0;
            for (; f + 8 <= a->d; f += 8)
                for (int l = 0; l < 8; ++l) acc[l] = fmaf(xr[f + l], cr[f + l], acc[l]);
            for (; f < a->d; ++f) acc[0] = fmaf(xr[f], cr[f], acc[0]);
            const float dot = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
            const float dist = fmaf(-2.0f, dot, a->pn[row] + a->cn[c]);
            if (dist < first) {
                first = dist;
                best = c;
            }
        }
        a->labels[row] = best;
    }
}

int orc_lloyd_fp32(int64_t n, int d, int k, const float* points, float* centroids, int* labels,
                   int max_iterations, float tolerance, int threads) {
    float* pn = (float*)malloc(sizeof(float) * (size_t)n);
    float* cn = (float*)malloc(sizeof(float) * (size_t)k);
    float* prev = (float*)malloc(sizeof(float) * (size_t)k * d);
    int* counts = (int*)malloc(sizeof(int) * (size_t)k);
    int result = max_iterations;
    orc_l2_norm(n, d, points, pn);
    for (int it = 0; it < max_iterations; ++it) {
        memcpy(prev, centroids, sizeof(float) * (size_t)k * d);
        orc_l2_norm(k, d, centroids, cn);
        f32_ctx a = {n, d, k, points, centroids, pn, cn, labels};
        parallel_for(n, threads, f32_rows, &a);
        orc_update_centroids(n, d, k, points, labels, prev, centroids, counts);
        const float shift = orc_centroid_shift((int64_t)k * d, prev, centroids);
        if (!isfinite(shift)) {
            result = -1;
            break;
        }
        if (shift <= tolerance) {
            result = it + 1;
            break;
        }
    }
    free(pn); free(cn); free(prev); free(counts);
    return result;
}
