/*
 * efo.c - CPU oracle (test infrastructure only) for the EdgeForge quantized
 * matrix-product path. A plain-C restatement of the reference algorithm; every
 * function names the reference file:line it follows. Build flags must keep
 * the reference's numerics: -O2 -ffp-contract=off, no -ffast-math.
 *
 * Never linked into the product library; see efo.h.
 */
#include "efo.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

static uint32_t bits_of(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

static float float_of(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* ------------------------------------------------------------------ fp16 / bf16 */

/* include/ef/fp16.h:28-30: a bf16 is the top half of an f32. */
float efo_bf16_to_f32(uint16_t h) { return float_of((uint32_t)h << 16); }

/* include/ef/fp16.h:32-40: round to nearest even; NaN stays a quiet NaN. */
uint16_t efo_f32_to_bf16(float f) {
  uint32_t u = bits_of(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((u >> 16) | 0x0040u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* include/ef/fp16.h:44-66: exact binary16 -> binary32. A subnormal half m is
 * m * 2^-24, which is exact in single precision. */
float efo_fp16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1Fu;
  const uint32_t m = h & 0x3FFu;
  if (e == 0) {
    const float mag = (float)m * 5.9604644775390625e-08f; /* 2^-24 */
    return float_of(bits_of(mag) | sign);
  }
  if (e == 31) return float_of(sign | 0x7F800000u | (m << 13));
  return float_of(sign | ((e + 112u) << 23) | (m << 13));
}

/* include/ef/fp16.h:69-92: binary32 -> binary16, round to nearest even,
 * |x| >= 65520 -> inf, NaN -> quiet NaN keeping the top payload bits. */
uint16_t efo_f32_to_fp16(float f) {
  const uint32_t u = bits_of(f);
  const uint16_t sign = (uint16_t)((u >> 16) & 0x8000u);
  const uint32_t a = u & 0x7FFFFFFFu;
  if (a > 0x7F800000u) return (uint16_t)(sign | 0x7E00u | ((a >> 13) & 0x3FFu));
  if (a >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);
  if (a < 0x38800000u) {
    /* Below the smallest normal half: the result is a multiple of 2^-24.
     * Scaling by 2^24 is exact, and nearbyintf rounds ties to even. */
    const float q = nearbyintf(float_of(a) * 16777216.0f);
    return (uint16_t)(sign | (uint16_t)q);
  }
  const uint32_t x = a - 0x38000000u; /* exponent bias 127 -> 15 */
  uint32_t r = x >> 13;
  const uint32_t dropped = x & 0x1FFFu;
  if (dropped > 0x1000u || (dropped == 0x1000u && (r & 1u))) ++r;
  return (uint16_t)(sign | r);
}

/* ------------------------------------------------------------------ blocks */

#define QK 32
#define FP16_MAX 65504.0f

static float fp16_round(float d) { return efo_fp16_to_f32(efo_f32_to_fp16(d)); }

static int clamp_i(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

static float clamp_f(float v, float lo, float hi) { return v < lo ? lo : (hi < v ? hi : v); }

static double clamp_d(double v, double lo, double hi) { return v < lo ? lo : (hi < v ? hi : v); }

/* static_cast<int>(std::nearbyint(v)) as the reference build executes it on
 * x86-64: round to nearest even, then truncating conversion, which yields
 * INT_MIN ("integer indefinite") for NaN and for values outside int range. */
static int round_to_int(float v) {
  const float r = nearbyintf(v);
  if (!(r >= -2147483648.0f && r < 2147483648.0f)) return (int)0x80000000u;
  return (int)r;
}

uint64_t efo_row_bytes(int qtype, uint64_t cols, int* ok) {
  /* src/quant.cpp:136-149 */
  if (ok) *ok = 1;
  switch (qtype) {
    case EFO_F32: return cols * 4;
    case EFO_F16:
    case EFO_BF16: return cols * 2;
    case EFO_Q8_0:
    case EFO_Q4_0:
      if (cols % QK != 0) {
        if (ok) *ok = 0;
        return 0;
      }
      return cols / QK * (qtype == EFO_Q8_0 ? 34u : 18u);
    default:
      if (ok) *ok = 0;
      return 0;
  }
}

/* Squared reconstruction error of one candidate scale over n values, codes
 * into q (src/quant.cpp:52-58 and :79-85: double accumulation in j order). */
static double q4_try(const float* x, size_t n, float d, uint8_t* q) {
  const float inv = 1.0f / d;
  double err = 0.0;
  for (size_t j = 0; j < n; ++j) {
    const int c = clamp_i(round_to_int(x[j] * inv) + 8, 0, 15);
    q[j] = (uint8_t)c;
    const float w = (float)(c - 8) * d;
    const double e = (double)x[j] - (double)w;
    err += e * e;
  }
  return err;
}

/* src/quant.cpp:26-99 (q4_group): amax/signed-max scan, up to six candidate
 * scales rounded to fp16 before use, strict-less-than selection, then two
 * least-squares refinement rounds. Returns the fp16-exact scale. */
static float q4_group(const float* x, size_t n, int search, uint8_t* q) {
  float amax = 0.0f, smax = 0.0f;
  for (size_t j = 0; j < n; ++j) {
    const float a = fabsf(x[j]);
    if (a > amax) {
      amax = a;
      smax = x[j];
    }
  }
  if (!(amax > 0.0f) || !isfinite(amax)) {
    for (size_t j = 0; j < n; ++j) q[j] = 8;
    return 0.0f;
  }
  float cand[6];
  int nc = 0;
  cand[nc++] = smax / -8.0f;
  if (search) {
    static const float div[5] = {7.0f, 7.25f, 7.5f, 7.75f, 8.0f};
    for (int k = 0; k < 5; ++k) cand[nc++] = amax / div[k];
  }
  uint8_t trial[256];
  float best_d = 0.0f;
  double best = -1.0;
  for (int c = 0; c < nc; ++c) {
    const float d = fp16_round(clamp_f(cand[c], -FP16_MAX, FP16_MAX));
    if (d == 0.0f) continue;
    const double err = q4_try(x, n, d, trial);
    if (best < 0.0 || err < best) {
      best = err;
      best_d = d;
      memcpy(q, trial, n);
    }
  }
  if (best < 0.0) {
    for (size_t j = 0; j < n; ++j) q[j] = 8;
    return 0.0f;
  }
  if (search) {
    for (int round = 0; round < 2; ++round) {
      double sxc = 0.0, scc = 0.0;
      for (size_t j = 0; j < n; ++j) {
        const double c = (double)((int)q[j] - 8);
        sxc += (double)x[j] * c;
        scc += c * c;
      }
      if (scc == 0.0) break;
      const float d = fp16_round((float)clamp_d(sxc / scc, -65504.0, 65504.0));
      if (d == 0.0f || d == best_d) break;
      const double err = q4_try(x, n, d, trial);
      if (!(err < best)) break;
      best = err;
      best_d = d;
      memcpy(q, trial, n);
    }
  }
  return best_d;
}

/* src/quant.cpp:151-156: scale at bytes 0-1 (little-endian fp16), then byte j
 * holds code j in its low nibble and code j+16 in its high nibble. */
void efo_quantize_block_q4_0(const float* x, uint8_t out[18], int search) {
  uint8_t q[QK];
  const uint16_t h = efo_f32_to_fp16(q4_group(x, QK, search, q));
  out[0] = (uint8_t)(h & 0xFF);
  out[1] = (uint8_t)(h >> 8);
  for (int j = 0; j < 16; ++j) out[2 + j] = (uint8_t)(q[j] | (q[j + 16] << 4));
}

/* src/quant.cpp:243-248: q4_group on the first min(n, 256) values, written back as
 * float(code - 8) * d. */
void efo_fake_quant_q4_group(const float* x, size_t n, float* out, int search) {
  uint8_t q[256];
  const size_t m = n < 256 ? n : 256;
  const float d = q4_group(x, m, search, q);
  for (size_t j = 0; j < m; ++j) out[j] = (float)((int)q[j] - 8) * d;
}

/* src/quant.cpp:158-164 */
void efo_dequantize_block_q4_0(const uint8_t in[18], float* out) {
  const float d = efo_fp16_to_f32((uint16_t)(in[0] | (in[1] << 8)));
  for (int j = 0; j < 16; ++j) {
    out[j] = (float)((in[2 + j] & 0x0F) - 8) * d;
    out[j + 16] = (float)((in[2 + j] >> 4) - 8) * d;
  }
}

/* src/quant.cpp:166-175: d = fp16(min(amax/127, 65504)), codes clamp to +-127. */
void efo_quantize_block_q8_0(const float* x, uint8_t out[34]) {
  float amax = 0.0f;
  for (int j = 0; j < QK; ++j) {
    const float a = fabsf(x[j]);
    amax = amax < a ? a : amax; /* std::max(amax, a) keeps amax on ties and NaN */
  }
  float d = 0.0f;
  if (amax > 0.0f && isfinite(amax)) {
    const float s = amax / 127.0f;
    d = fp16_round(FP16_MAX < s ? FP16_MAX : s);
  }
  const uint16_t h = efo_f32_to_fp16(d);
  out[0] = (uint8_t)(h & 0xFF);
  out[1] = (uint8_t)(h >> 8);
  const float inv = d != 0.0f ? 1.0f / d : 0.0f;
  for (int j = 0; j < QK; ++j) out[2 + j] = (uint8_t)(int8_t)clamp_i(round_to_int(x[j] * inv), -127, 127);
}

/* src/quant.cpp:177-180 */
void efo_dequantize_block_q8_0(const uint8_t in[34], float* out) {
  const float d = efo_fp16_to_f32((uint16_t)(in[0] | (in[1] << 8)));
  for (int j = 0; j < QK; ++j) out[j] = (float)(int8_t)in[2 + j] * d;
}

/* src/quant.cpp:182-218 */
int efo_quantize_row(int qtype, const float* x, size_t n, void* out, int search) {
  uint8_t* o = (uint8_t*)out;
  switch (qtype) {
    case EFO_F32: memcpy(o, x, n * 4); return 0;
    case EFO_F16:
    case EFO_BF16:
      for (size_t i = 0; i < n; ++i) {
        const uint16_t h = qtype == EFO_F16 ? efo_f32_to_fp16(x[i]) : efo_f32_to_bf16(x[i]);
        o[2 * i] = (uint8_t)(h & 0xFF);
        o[2 * i + 1] = (uint8_t)(h >> 8);
      }
      return 0;
    case EFO_Q8_0:
    case EFO_Q4_0:
      if (n % QK != 0) return -1;
      for (size_t b = 0; b < n / QK; ++b) {
        if (qtype == EFO_Q4_0) efo_quantize_block_q4_0(x + b * QK, o + b * 18, search);
        else efo_quantize_block_q8_0(x + b * QK, o + b * 34);
      }
      return 0;
    default: return -1;
  }
}

/* src/quant.cpp:220-249 */
int efo_dequantize_row(int qtype, const void* in, size_t n, float* out) {
  const uint8_t* p = (const uint8_t*)in;
  switch (qtype) {
    case EFO_F32: memcpy(out, p, n * 4); return 0;
    case EFO_F16:
    case EFO_BF16:
      for (size_t i = 0; i < n; ++i) {
        const uint16_t h = (uint16_t)(p[2 * i] | (p[2 * i + 1] << 8));
        out[i] = qtype == EFO_F16 ? efo_fp16_to_f32(h) : efo_bf16_to_f32(h);
      }
      return 0;
    case EFO_Q8_0:
    case EFO_Q4_0:
      if (n % QK != 0) return -1;
      for (size_t b = 0; b < n / QK; ++b) {
        if (qtype == EFO_Q4_0) efo_dequantize_block_q4_0(p + b * 18, out + b * QK);
        else efo_dequantize_block_q8_0(p + b * 34, out + b * QK);
      }
      return 0;
    default: return -1;
  }
}

/* ------------------------------------------------------------------ threads */

/* Contiguous chunk c of n items split in `chunks` (include/ef/threadpool.h:52-54). */
static size_t chunk_begin(size_t n, size_t chunks, size_t c) {
  return (size_t)((unsigned long long)n * c / chunks);
}

typedef void (*range_fn)(void* ctx, size_t b, size_t e);

typedef struct {
  range_fn fn;
  void* ctx;
  size_t b, e;
} range_job;

static void* range_thread(void* p) {
  range_job* j = (range_job*)p;
  j->fn(j->ctx, j->b, j->e);
  return NULL;
}

static void parallel_rows(size_t n, int threads, range_fn fn, void* ctx) {
  size_t T = threads > 1 ? (size_t)threads : 1;
  if (T > n) T = n ? n : 1;
  if (T <= 1) {
    fn(ctx, 0, n);
    return;
  }
  pthread_t* th = (pthread_t*)malloc(T * sizeof(pthread_t));
  range_job* jobs = (range_job*)malloc(T * sizeof(range_job));
  for (size_t c = 0; c < T; ++c) {
    jobs[c].fn = fn;
    jobs[c].ctx = ctx;
    jobs[c].b = chunk_begin(n, T, c);
    jobs[c].e = chunk_begin(n, T, c + 1);
  }
  for (size_t c = 1; c < T; ++c) pthread_create(&th[c], NULL, range_thread, &jobs[c]);
  range_thread(&jobs[0]);
  for (size_t c = 1; c < T; ++c) pthread_join(th[c], NULL);
  free(th);
  free(jobs);
}

typedef struct {
  int qtype, search;
  const float* x;
  float* fx;
  const uint8_t* in;
  uint8_t* out;
  size_t cols, rb;
} rows_ctx;

static void quant_range(void* p, size_t b, size_t e) {
  rows_ctx* c = (rows_ctx*)p;
  for (size_t r = b; r < e; ++r) efo_quantize_row(c->qtype, c->x + r * c->cols, c->cols, c->out + r * c->rb, c->search);
}

static void dequant_range(void* p, size_t b, size_t e) {
  rows_ctx* c = (rows_ctx*)p;
  for (size_t r = b; r < e; ++r) efo_dequantize_row(c->qtype, c->in + r * c->rb, c->cols, c->fx + r * c->cols);
}

int efo_quantize_rows(int qtype, const float* x, size_t rows, size_t cols, void* out, int search, int threads) {
  int ok = 0;
  const uint64_t rb = efo_row_bytes(qtype, cols, &ok);
  if (!ok) return -1;
  rows_ctx c = {qtype, search, x, NULL, NULL, (uint8_t*)out, cols, (size_t)rb};
  parallel_rows(rows, threads, quant_range, &c);
  return 0;
}

int efo_dequantize_rows(int qtype, const void* in, size_t rows, size_t cols, float* out, int threads) {
  int ok = 0;
  const uint64_t rb = efo_row_bytes(qtype, cols, &ok);
  if (!ok) return -1;
  rows_ctx c = {qtype, 0, NULL, out, (const uint8_t*)in, NULL, cols, (size_t)rb};
  parallel_rows(rows, threads, dequant_range, &c);
  return 0;
}

/* ------------------------------------------------------------------ packed dots */

/* src/qkernels.cpp:28-32: fixed pairwise reduction of 32 lane sums. */
static float sum32(const float* a, const float* b) {
  float s[8];
  for (int j = 0; j < 8; ++j) s[j] = (a[j] + a[j + 8]) + (b[j] + b[j + 8]);
  return ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
}

/* src/qkernels.cpp:39-51: lane j accumulates weight j of every block (low
 * nibbles into lo[], high nibbles into hi[]), d * (code * x) per weight. */
float efo_dot_q4_0(const uint8_t* row, const float* x, size_t n) {
  float lo[16] = {0}, hi[16] = {0};
  for (size_t b = 0; b < n / QK; ++b, row += 18, x += QK) {
    const float d = efo_fp16_to_f32((uint16_t)(row[0] | (row[1] << 8)));
    for (int j = 0; j < 16; ++j) {
      const uint8_t byte = row[2 + j];
      lo[j] += d * ((float)((byte & 0x0F) - 8) * x[j]);
      hi[j] += d * ((float)((byte >> 4) - 8) * x[j + 16]);
    }
  }
  return sum32(lo, hi);
}

/* src/qkernels.cpp:53-65 */
float efo_dot_q8_0(const uint8_t* row, const float* x, size_t n) {
  float lo[16] = {0}, hi[16] = {0};
  for (size_t b = 0; b < n / QK; ++b, row += 34, x += QK) {
    const float d = efo_fp16_to_f32((uint16_t)(row[0] | (row[1] << 8)));
    const int8_t* q = (const int8_t*)(row + 2);
    for (int j = 0; j < 16; ++j) {
      lo[j] += d * ((float)q[j] * x[j]);
      hi[j] += d * ((float)q[j + 16] * x[j + 16]);
    }
  }
  return sum32(lo, hi);
}

/* src/qkernels.cpp:67-75 */
void efo_matvec_q4_0(float* y, const uint8_t* W, const float* x, size_t rows, size_t cols) {
  const size_t rb = cols / QK * 18;
  for (size_t r = 0; r < rows; ++r) y[r] = efo_dot_q4_0(W + r * rb, x, cols);
}

void efo_matvec_q8_0(float* y, const uint8_t* W, const float* x, size_t rows, size_t cols) {
  const size_t rb = cols / QK * 34;
  for (size_t r = 0; r < rows; ++r) y[r] = efo_dot_q8_0(W + r * rb, x, cols);
}

/* ------------------------------------------------------------------ FP32 ops */

/* src/kernels.cpp:28-43 (dot_row): 8 partial sums, pairwise combine. */
static float dot_any(int type, const uint8_t* w, const float* x, size_t n) {
  float a[8] = {0};
  size_t i = 0;
  if (type == EFO_F32) {
    const float* f = (const float*)w;
    for (; i + 8 <= n; i += 8)
      for (int k = 0; k < 8; ++k) a[k] += f[i + k] * x[i + k];
    for (; i < n; ++i) a[0] += f[i] * x[i];
  } else { /* BF16 */
    for (; i + 8 <= n; i += 8)
      for (int k = 0; k < 8; ++k) {
        const size_t o = 2 * (i + k);
        a[k] += efo_bf16_to_f32((uint16_t)(w[o] | (w[o + 1] << 8))) * x[i + k];
      }
    for (; i < n; ++i) a[0] += efo_bf16_to_f32((uint16_t)(w[2 * i] | (w[2 * i + 1] << 8))) * x[i];
  }
  return ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
}

float efo_dot_f32(const float* a, const float* b, size_t n) { return dot_any(EFO_F32, (const uint8_t*)a, b, n); }

/* Scalar-backend row dispatch (src/qkernels.cpp:243-268). */
static float dot_row_typed(const efo_weight* W, size_t r, const float* x) {
  int ok = 0;
  const size_t rb = (size_t)efo_row_bytes(W->type, W->cols, &ok);
  const uint8_t* row = W->data + r * rb;
  switch (W->type) {
    case EFO_Q4_0: return efo_dot_q4_0(row, x, W->cols);
    case EFO_Q8_0: return efo_dot_q8_0(row, x, W->cols);
    case EFO_F32:
    case EFO_BF16: return dot_any(W->type, row, x, W->cols);
    default: { /* F16: sequential accumulation */
      float acc = 0.0f;
      for (size_t c = 0; c < W->cols; ++c) acc += efo_fp16_to_f32((uint16_t)(row[2 * c] | (row[2 * c + 1] << 8))) * x[c];
      return acc;
    }
  }
}

typedef struct {
  const efo_weight* W;
  const float* x;
  float* y;
} mv_ctx;

static void mv_range(void* p, size_t b, size_t e) {
  mv_ctx* c = (mv_ctx*)p;
  for (size_t r = b; r < e; ++r) c->y[r] = dot_row_typed(c->W, r, c->x);
}

static void matvec_typed(float* y, const efo_weight* W, const float* x, int threads) {
  mv_ctx c = {W, x, y};
  parallel_rows(W->rows, threads, mv_range, &c);
}

void efo_matvec_mt(int qtype, float* y, const uint8_t* W, const float* x, size_t rows, size_t cols, int threads) {
  const efo_weight w = {qtype, W, rows, cols};
  matvec_typed(y, &w, x, threads);
}

void efo_exact_dot(int qtype, const uint8_t* row, const float* x, size_t n, double* exact, double* mag) {
  float* w = (float*)malloc(n * sizeof(float));
  efo_dequantize_row(qtype, row, n, w);
  double s = 0.0, m = 0.0;
  for (size_t i = 0; i < n; ++i) {
    const double p = (double)w[i] * (double)x[i];
    s += p;
    m += fabs(p);
  }
  free(w);
  *exact = s;
  *mag = m;
}

typedef struct {
  int qtype;
  const uint8_t* W;
  const float* x;
  size_t cols, rb;
  double *exact, *mag;
} exact_ctx;

static void exact_range(void* vc, size_t b, size_t e) {
  const exact_ctx* c = (const exact_ctx*)vc;
  for (size_t r = b; r < e; ++r) efo_exact_dot(c->qtype, c->W + r * c->rb, c->x, c->cols, &c->exact[r], &c->mag[r]);
}

int efo_exact_dots(int qtype, const uint8_t* W, const float* x, size_t rows, size_t cols, double* exact, double* mag,
                   int threads) {
  int ok = 0;
  const uint64_t rb = efo_row_bytes(qtype, cols, &ok);
  if (!ok) return -1;
  exact_ctx c = {qtype, W, x, cols, (size_t)rb, exact, mag};
  parallel_rows(rows, threads, exact_range, &c);
  return 0;
}

double efo_rel_dot_error(int qtype, const uint8_t* row, const float* x, size_t n, float got) {
  double exact, mag;
  efo_exact_dot(qtype, row, x, n, &exact, &mag);
  return fabs((double)got - exact) / (mag > 1e-30 ? mag : 1e-30);
}

/* src/kernels.cpp:69-75: double sum of squares; out = w * (x * inv). */
void efo_rmsnorm(float* out, const float* x, const float* w, size_t n, float eps) {
  double ss = 0.0;
  for (size_t i = 0; i < n; ++i) ss += (double)x[i] * (double)x[i];
  const double mean = n ? ss / (double)n : 0.0;
  const float inv = (float)(1.0 / sqrt(mean + (double)eps));
  for (size_t i = 0; i < n; ++i) out[i] = w[i] * (x[i] * inv);
}

/* src/kernels.cpp:77-92 */
void efo_softmax_inplace(float* x, size_t n) {
  if (n == 0) return;
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) mx = x[i] > mx ? x[i] : mx;
  if (mx == -INFINITY) {
    for (size_t i = 0; i < n; ++i) x[i] = 0.0f;
    return;
  }
  double sum = 0.0;
  for (size_t i = 0; i < n; ++i) {
    x[i] = expf(x[i] - mx);
    sum += (double)x[i];
  }
  const float inv = (float)(1.0 / sum);
  for (size_t i = 0; i < n; ++i) x[i] *= inv;
}

/* src/kernels.cpp:94-99 */
void efo_swiglu(float* out, const float* gate, const float* up, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    const float g = gate[i];
    out[i] = g / (1.0f + expf(-g)) * up[i];
  }
}

/* src/kernels.cpp:105-111: first index of the maximum. */
size_t efo_argmax(const float* x, size_t n) {
  size_t best = 0;
  for (size_t i = 1; i < n; ++i)
    if (x[i] > x[best]) best = i;
  return best;
}

/* src/kernels.cpp:113-131: inv_freq[i] = 1 / theta^(2i/hd) in float;
 * angle = float(pos) * inv_freq[i]. */
void efo_rope_table(float* cos_out, float* sin_out, size_t max_pos, size_t head_dim, float theta) {
  const size_t half = head_dim / 2;
  float* inv = (float*)malloc((half ? half : 1) * sizeof(float));
  for (size_t i = 0; i < half; ++i) inv[i] = 1.0f / powf(theta, (float)(2 * i) / (float)head_dim);
  for (size_t p = 0; p < max_pos; ++p)
    for (size_t i = 0; i < half; ++i) {
      const float ang = (float)p * inv[i];
      cos_out[p * half + i] = cosf(ang);
      sin_out[p * half + i] = sinf(ang);
    }
  free(inv);
}

/* src/kernels.cpp:133-146: half-split rotation, dim i pairs with i + hd/2. */
void efo_rope_apply(float* x, size_t n_heads, size_t head_dim, const float* c, const float* s) {
  const size_t half = head_dim / 2;
  for (size_t h = 0; h < n_heads; ++h) {
    float* v = x + h * head_dim;
    for (size_t i = 0; i < half; ++i) {
      const float a = v[i], b = v[i + half];
      v[i] = a * c[i] - b * s[i];
      v[i + half] = b * c[i] + a * s[i];
    }
  }
}

/* src/kernels.cpp:153-174 */
void efo_attention(float* out, const float* q, const float* kc, const float* vc, size_t n_pos, size_t H,
                   size_t KV, size_t hd, float* scores) {
  const size_t group = H / KV, kvd = KV * hd;
  const float scale = (float)(1.0 / sqrt((double)hd));
  for (size_t h = 0; h < H; ++h) {
    const size_t kv = h / group;
    const float* qh = q + h * hd;
    for (size_t t = 0; t < n_pos; ++t) scores[t] = efo_dot_f32(qh, kc + t * kvd + kv * hd, hd) * scale;
    efo_softmax_inplace(scores, n_pos);
    float* oh = out + h * hd;
    memset(oh, 0, hd * sizeof(float));
    for (size_t t = 0; t < n_pos; ++t) {
      const float p = scores[t];
      const float* vt = vc + t * kvd + kv * hd;
      for (size_t d = 0; d < hd; ++d) oh[d] += p * vt[d];
    }
  }
}

/* src/qkernels.cpp:299-305 + src/kernels.cpp:100-103 */
void efo_row_f32(float* out, const efo_weight* w, size_t r) {
  int ok = 0;
  const size_t rb = (size_t)efo_row_bytes(w->type, w->cols, &ok);
  efo_dequantize_row(w->type, w->data + r * rb, w->cols, out);
}

/* ------------------------------------------------------------------ decode forward */

struct efo_state {
  const efo_model* m;
  size_t cached;
  float *k_cache, *v_cache, *rope_cos, *rope_sin;
  float *x, *h, *q, *ctx, *o, *gate, *up, *scores;
};

efo_state* efo_state_new(const efo_model* m) {
  efo_state* s = (efo_state*)calloc(1, sizeof(efo_state));
  const size_t kvd = m->KV * m->hd;
  s->m = m;
  s->k_cache = (float*)calloc(m->L * m->max_seq * kvd, sizeof(float));
  s->v_cache = (float*)calloc(m->L * m->max_seq * kvd, sizeof(float));
  s->rope_cos = (float*)malloc(m->max_seq * (m->hd / 2) * sizeof(float));
  s->rope_sin = (float*)malloc(m->max_seq * (m->hd / 2) * sizeof(float));
  efo_rope_table(s->rope_cos, s->rope_sin, m->max_seq, m->hd, m->rope_theta);
  s->x = (float*)malloc(m->D * sizeof(float));
  s->h = (float*)malloc(m->D * sizeof(float));
  s->q = (float*)malloc(m->D * sizeof(float));
  s->ctx = (float*)malloc(m->D * sizeof(float));
  s->o = (float*)malloc(m->D * sizeof(float));
  s->gate = (float*)malloc(m->F * sizeof(float));
  s->up = (float*)malloc(m->F * sizeof(float));
  s->scores = (float*)malloc(m->max_seq * sizeof(float));
  return s;
}

void efo_state_free(efo_state* s) {
  if (!s) return;
  free(s->k_cache);
  free(s->v_cache);
  free(s->rope_cos);
  free(s->rope_sin);
  free(s->x);
  free(s->h);
  free(s->q);
  free(s->ctx);
  free(s->o);
  free(s->gate);
  free(s->up);
  free(s->scores);
  free(s);
}

/* src/model.cpp:184-276, one token through every layer. */
int efo_forward(efo_state* s, int32_t token, size_t pos, float* logits, int threads) {
  const efo_model* m = s->m;
  if (token < 0 || (size_t)token >= m->V || pos >= m->max_seq || pos > s->cached) return -1;
  const size_t D = m->D, kvd = m->KV * m->hd, half = m->hd / 2;
  efo_row_f32(s->x, &m->embed, (size_t)token);
  const float* c = s->rope_cos + pos * half;
  const float* sn = s->rope_sin + pos * half;
  for (size_t l = 0; l < m->L; ++l) {
    const efo_layer* w = &m->layers[l];
    float* k_layer = s->k_cache + l * m->max_seq * kvd;
    float* v_layer = s->v_cache + l * m->max_seq * kvd;
    float* k_pos = k_layer + pos * kvd;
    float* v_pos = v_layer + pos * kvd;
    efo_rmsnorm(s->h, s->x, w->attn_norm, D, m->eps);
    matvec_typed(s->q, &w->wq, s->h, threads);
    matvec_typed(k_pos, &w->wk, s->h, threads);
    matvec_typed(v_pos, &w->wv, s->h, threads);
    efo_rope_apply(s->q, m->H, m->hd, c, sn);
    efo_rope_apply(k_pos, m->KV, m->hd, c, sn);
    efo_attention(s->ctx, s->q, k_layer, v_layer, pos + 1, m->H, m->KV, m->hd, s->scores);
    matvec_typed(s->o, &w->wo, s->ctx, threads);
    for (size_t i = 0; i < D; ++i) s->x[i] += s->o[i];
    efo_rmsnorm(s->h, s->x, w->ffn_norm, D, m->eps);
    matvec_typed(s->gate, &w->w_gate, s->h, threads);
    matvec_typed(s->up, &w->w_up, s->h, threads);
    efo_swiglu(s->gate, s->gate, s->up, m->F);
    matvec_typed(s->o, &w->w_down, s->gate, threads);
    for (size_t i = 0; i < D; ++i) s->x[i] += s->o[i];
  }
  s->cached = pos + 1;
  efo_rmsnorm(s->h, s->x, m->final_norm, D, m->eps);
  if (logits) matvec_typed(logits, &m->lm_head, s->h, threads);
  return 0;
}
