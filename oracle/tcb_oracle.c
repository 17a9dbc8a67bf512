/*
 * CPU restatement of the chip-metric probes' arithmetic - TEST INFRASTRUCTURE.
 *
 * This file is the checker, never the thing measured or shipped: only the
 * test suite, the smoke entry point and bench.py's CPU-baseline leg load it.
 * Each function names the reference-suite code (huangyiqun/triton_chip_benchmarks)
 * whose semantics it restates.
 *
 *   oracle_copy        dst = src, split over host threads
 *                      (copy_kernel, bench_bandwidth.py:36-40; host copy baseline)
 *   oracle_chain_f32   x <- fmaf(x, a, b_c) per step       (bench_vector.py:87-91, 269-309)
 *   oracle_chain_f64   x <- fma(x, a, b_c) per step
 *   oracle_chain_h16   fp16 / bf16 state, exact x*a+b then one rounding
 *   oracle_chain_dp4a  x <- dot4(x, a) + b_c on int32 words (bench_vector.py:134-145)
 *   oracle_chain_imad  x <- a*x + b_c mod 2**32
 *   oracle_chain_i8    x <- (a*x + b_c) mod 256, int8 state (bench_vector.py:160-166)
 *   oracle_block_sums  per-block sums in double (read_kernel, bench_bandwidth.py:50-59)
 *
 * Chains use the [8][elements] layout of the probe; coefficients are
 * {a, b_0 .. b_7}.  Half-precision values are passed as their 16-bit
 * patterns.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define CHAINS 8

/* ------------------------------------------------------------- copy */
typedef struct {
  const unsigned char *src;
  unsigned char *dst;
  size_t bytes;
} copy_job;

static void *copy_worker(void *arg) {
  copy_job *job = (copy_job *)arg;
  memcpy(job->dst, job->src, job->bytes);
  return NULL;
}

/* Returns the number of threads used. */
int oracle_copy(const void *src, void *dst, size_t bytes, int threads) {
  if (threads < 1) threads = 1;
  if (threads > 256) threads = 256;
  if (bytes < (size_t)threads * 4096) threads = 1;
  pthread_t tid[256];
  copy_job jobs[256];
  size_t chunk = (bytes / (size_t)threads + 4095) & ~(size_t)4095;
  int used = 0;
  for (int t = 0; t < threads; ++t) {
    size_t off = (size_t)t * chunk;
    if (off >= bytes) break;
    size_t len = bytes - off < chunk ? bytes - off : chunk;
    jobs[t].src = (const unsigned char *)src + off;
    jobs[t].dst = (unsigned char *)dst + off;
    jobs[t].bytes = len;
    if (pthread_create(&tid[t], NULL, copy_worker, &jobs[t]) != 0) {
      copy_worker(&jobs[t]);
      tid[t] = 0;
    }
    used = t + 1;
  }
  for (int t = 0; t < used; ++t)
    if (tid[t]) pthread_join(tid[t], NULL);
  return used;
}

/* ----------------------------------------------------- float chains */
void oracle_chain_f32(const float *in, float *out, long long elements, const float *coeff,
                      int iterations) {
  const float a = coeff[0];
  for (int c = 0; c < CHAINS; ++c) {
    const float b = coeff[1 + c];
    for (long long e = 0; e < elements; ++e) {
      float x = in[c * elements + e];
      for (int i = 0; i < iterations; ++i) x = fmaf(x, a, b);
      out[c * elements + e] = x;
    }
  }
}

void oracle_chain_f64(const double *in, double *out, long long elements, const double *coeff,
                      int iterations) {
  const double a = coeff[0];
  for (int c = 0; c < CHAINS; ++c) {
    const double b = coeff[1 + c];
    for (long long e = 0; e < elements; ++e) {
      double x = in[c * elements + e];
      for (int i = 0; i < iterations; ++i) x = fma(x, a, b);
      out[c * elements + e] = x;
    }
  }
}

/* IEEE binary16 / bfloat16 <-> double, round-to-nearest-even on the way in. */
static double h16_to_double(uint16_t h, int bf16) {
  if (bf16) {
    uint32_t bits = (uint32_t)h << 16;
    float f;
    memcpy(&f, &bits, 4);
    return (double)f;
  }
  int sign = h >> 15, exp = (h >> 10) & 31, man = h & 1023;
  double v;
  if (exp == 0)
    v = ldexp((double)man, -24);
  else if (exp == 31)
    v = man ? NAN : INFINITY;
  else
    v = ldexp((double)(man | 1024), exp - 25);
  return sign ? -v : v;
}

/* Round |v| to `bits` significant bits (nearest-even), quantum >= 2^min_q. */
static double round_significant(double m, int bits, int min_q) {
  if (m == 0.0) return 0.0;
  int e;
  frexp(m, &e); /* m = f * 2^e, f in [0.5, 1) */
  int q = e - bits;
  if (q < min_q) q = min_q;
  return ldexp(nearbyint(ldexp(m, -q)), q); /* scalings by 2^k are exact */
}

static uint16_t double_to_h16(double v, int bf16) {
  uint16_t sign = signbit(v) ? 0x8000 : 0;
  double m = fabs(v);
  if (bf16) {
    if (isnan(m)) return sign | 0x7fc0;
    double r = round_significant(m, 8, -133);
    if (r > ldexp(255.0, 120)) return sign | 0x7f80; /* beyond the largest finite bf16 */
    float f = (float)r;                                /* exact: <= 8 significant bits */
    uint32_t bits;
    memcpy(&bits, &f, 4);
    return sign | (uint16_t)(bits >> 16);
  }
  if (isnan(m)) return sign | 0x7e00;
  double r = round_significant(m, 11, -24);
  if (r > 65504.0) return sign | 0x7c00;
  if (r == 0.0) return sign;
  int e;
  frexp(r, &e);
  if (e - 1 < -14) return sign | (uint16_t)ldexp(r, 24); /* subnormal: r / 2^-24 */
  uint16_t man = (uint16_t)(ldexp(r, 11 - e) - 1024.0);
  return sign | (uint16_t)((e - 1 + 15) << 10) | man;
}

/* Returns 0, or -1 if some step's x*a+b was not exactly representable in
   double (then the single-rounding emulation would not be exact). */
int oracle_chain_h16(const uint16_t *in, uint16_t *out, long long elements,
                     const uint16_t *coeff, int iterations, int bf16) {
  const double a = h16_to_double(coeff[0], bf16);
  int status = 0;
  for (int c = 0; c < CHAINS; ++c) {
    const double b = h16_to_double(coeff[1 + c], bf16);
    for (long long e = 0; e < elements; ++e) {
      uint16_t x = in[c * elements + e];
      for (int i = 0; i < iterations; ++i) {
        double p = h16_to_double(x, bf16) * a; /* exact: <= 22 significant bits */
        double s = p + b;
        if ((s - p) - b != 0.0 || fma(1.0, p, b) != s) status = -1;
        x = double_to_h16(s, bf16);
      }
      out[c * elements + e] = x;
    }
  }
  return status;
}

/* ------------------------------------------------------- int chains */
static int32_t dot4(int32_t x, int32_t w) {
  int32_t s = 0;
  for (int k = 0; k < 4; ++k) {
    int8_t xb = (int8_t)((uint32_t)x >> (8 * k));
    int8_t wb = (int8_t)((uint32_t)w >> (8 * k));
    s += (int32_t)xb * (int32_t)wb;
  }
  return s;
}

void oracle_chain_dp4a(const int32_t *in, int32_t *out, long long elements, const int32_t *coeff,
                       int iterations) {
  for (int c = 0; c < CHAINS; ++c) {
    const uint32_t b = (uint32_t)coeff[1 + c];
    for (long long e = 0; e < elements; ++e) {
      int32_t x = in[c * elements + e];
      for (int i = 0; i < iterations; ++i) x = (int32_t)((uint32_t)dot4(x, coeff[0]) + b);
      out[c * elements + e] = x;
    }
  }
}

void oracle_chain_imad(const int32_t *in, int32_t *out, long long elements, const int32_t *coeff,
                       int iterations) {
  const uint32_t a = (uint32_t)coeff[0];
  for (int c = 0; c < CHAINS; ++c) {
    const uint32_t b = (uint32_t)coeff[1 + c];
    for (long long e = 0; e < elements; ++e) {
      uint32_t x = (uint32_t)in[c * elements + e];
      for (int i = 0; i < iterations; ++i) x = x * a + b;
      out[c * elements + e] = (int32_t)x;
    }
  }
}

void oracle_chain_i8(const int8_t *in, int8_t *out, long long elements, const int8_t *coeff,
                     int iterations) {
  const int32_t a = coeff[0];
  for (int c = 0; c < CHAINS; ++c) {
    const int32_t b = coeff[1 + c];
    for (long long e = 0; e < elements; ++e) {
      int32_t x = in[c * elements + e];
      for (int i = 0; i < iterations; ++i) x = (int8_t)(uint8_t)(x * a + b);
      out[c * elements + e] = (int8_t)x;
    }
  }
}

/* ------------------------------------------------------- block sums */
void oracle_block_sums(const float *src, long long elements, int block, double *sums,
                       double *abs_sums) {
  long long blocks = (elements + block - 1) / block;
  for (long long i = 0; i < blocks; ++i) {
    double s = 0.0, a = 0.0;
    long long end = (i + 1) * block < elements ? (i + 1) * block : elements;
    for (long long e = i * block; e < end; ++e) {
      s += src[e];
      a += fabs(src[e]);
    }
    sums[i] = s;
    abs_sums[i] = a;
  }
}
