/*
 * efo.h - CPU oracle for the EdgeForge quantized matrix-product path.
 *
 * TEST INFRASTRUCTURE ONLY. This is a plain-C restatement of the reference
 * algorithm (MG782469/EdgeForge, C++20), used by tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg as the checker. The product path (the CUDA
 * library under edgeforge_b200/) never links, loads or calls this code.
 *
 * Parity is pinned two ways: (1) against the reference itself, compiled from
 * its own sources into oracle/_ref/ by oracle/Makefile (same seeded inputs,
 * bit-for-bit comparison in tests/test_oracle.py), and (2) against the
 * reference's own known-answer tests (tests/test_quant.cpp, test_qinfer.cpp,
 * test_fp16.cpp), restated in tests/test_oracle.py, plus committed golden
 * vectors under tests/golden/.
 *
 * Numerics follow the reference build: -ffp-contract=off (no a*b+c -> fma),
 * round-to-nearest-even, no fast-math.
 */
#ifndef EFO_H
#define EFO_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Storage types, same numbering as ef::QType (include/ef/quant.h:35). */
enum { EFO_F32 = 0, EFO_F16 = 1, EFO_BF16 = 2, EFO_Q8_0 = 3, EFO_Q4_0 = 4 };

/* ---- 16-bit floats (include/ef/fp16.h:28-92) ---------------------------- */
float efo_bf16_to_f32(uint16_t h);
uint16_t efo_f32_to_bf16(float f);
float efo_fp16_to_f32(uint16_t h);
uint16_t efo_f32_to_fp16(float f);

/* ---- blocks (src/quant.cpp:26-180) -------------------------------------- */
/* Row bytes for `cols` weights; returns 0 (and sets *ok = 0) when a block type
 * is given a length that is not a multiple of 32 (quant.cpp:136-149 throws). */
uint64_t efo_row_bytes(int qtype, uint64_t cols, int* ok);
void efo_quantize_block_q4_0(const float* x, uint8_t out[18], int search);
void efo_quantize_block_q8_0(const float* x, uint8_t out[34]);
void efo_dequantize_block_q4_0(const uint8_t in[18], float* out);
/* quant.cpp:243-248: Q4 quantize -> dequantize of one group (first min(n, 256) values). */
void efo_fake_quant_q4_group(const float* x, size_t n, float* out, int search);
void efo_dequantize_block_q8_0(const uint8_t in[34], float* out);
/* Rows (quant.cpp:182-249). Return 0 on success, -1 if n is not a multiple of 32
 * for a block type. */
int efo_quantize_row(int qtype, const float* x, size_t n, void* out, int search);
int efo_dequantize_row(int qtype, const void* in, size_t n, float* out);
/* Many rows in one call (row-major [rows][cols]); threads > 1 splits rows in
 * contiguous chunks like quantizer.cpp:37-51 (results do not depend on it). */
int efo_quantize_rows(int qtype, const float* x, size_t rows, size_t cols, void* out, int search, int threads);
int efo_dequantize_rows(int qtype, const void* in, size_t rows, size_t cols, float* out, int threads);

/* ---- packed dots, scalar reference backend (src/qkernels.cpp:28-75) ------ */
float efo_dot_q4_0(const uint8_t* row, const float* x, size_t n);
float efo_dot_q8_0(const uint8_t* row, const float* x, size_t n);
void efo_matvec_q4_0(float* y, const uint8_t* W, const float* x, size_t rows, size_t cols);
void efo_matvec_q8_0(float* y, const uint8_t* W, const float* x, size_t rows, size_t cols);
/* Same as efo_matvec_q*_0 split over `threads` POSIX threads (rows in
 * contiguous chunks, threadpool.h:52-54); bit-identical for any thread count. */
void efo_matvec_mt(int qtype, float* y, const uint8_t* W, const float* x, size_t rows, size_t cols, int threads);
/* The reference's error metric (tests/test_qinfer.cpp:58-67): |got - exact| /
 * sum|w_i x_i| with the dequantized weights and double accumulation. */
double efo_rel_dot_error(int qtype, const uint8_t* row, const float* x, size_t n, float got);
/* Exact (double) dot of a dequantized row with x and its magnitude sum|w x|. */
void efo_exact_dot(int qtype, const uint8_t* row, const float* x, size_t n, double* exact, double* mag);
/* efo_exact_dot for every row of a packed [rows][cols] matrix, rows split over `threads`
 * POSIX threads. Returns -1 when cols is not a multiple of 32. */
int efo_exact_dots(int qtype, const uint8_t* W, const float* x, size_t rows, size_t cols, double* exact, double* mag,
                   int threads);

/* ---- FP32 transformer ops (src/kernels.cpp) ----------------------------- */
float efo_dot_f32(const float* a, const float* b, size_t n);                             /* :28-47 */
void efo_rmsnorm(float* out, const float* x, const float* w, size_t n, float eps);       /* :69-75 */
void efo_softmax_inplace(float* x, size_t n);                                              /* :77-92 */
void efo_swiglu(float* out, const float* gate, const float* up, size_t n);               /* :94-99 */
size_t efo_argmax(const float* x, size_t n);                                              /* :105-111 */
/* RoPE table [max_pos][head_dim/2] (kernels.cpp:113-131). */
void efo_rope_table(float* cos_out, float* sin_out, size_t max_pos, size_t head_dim, float theta);
void efo_rope_apply(float* x, size_t n_heads, size_t head_dim, const float* cos_row, const float* sin_row); /* :133-146 */
/* Single-query GQA attention (kernels.cpp:153-174); scores: n_pos floats scratch. */
void efo_attention(float* out, const float* q, const float* k_cache, const float* v_cache, size_t n_pos,
                   size_t n_heads, size_t n_kv_heads, size_t head_dim, float* scores);

/* ---- one decode forward (src/model.cpp:184-276) -------------------------- */
typedef struct {
  int type;            /* EFO_* storage type */
  const uint8_t* data; /* row-major packed rows */
  size_t rows, cols;
} efo_weight;

typedef struct {
  efo_weight wq, wk, wv, wo, w_gate, w_up, w_down;
  const float* attn_norm; /* [D] */
  const float* ffn_norm;  /* [D] */
} efo_layer;

typedef struct {
  size_t D, F, H, KV, hd, V, L, max_seq;
  float eps, rope_theta;
  efo_weight embed;   /* BF16 or a block type [V][D] */
  efo_weight lm_head; /* [V][D] */
  const float* final_norm;
  const efo_layer* layers;
} efo_model;

/* Opaque decode state: KV caches, RoPE table, activations. */
typedef struct efo_state efo_state;
efo_state* efo_state_new(const efo_model* m);
void efo_state_free(efo_state* s);
/* Runs `token` at `pos` (pos <= cached); writes logits[V] when logits != NULL.
 * Uses `threads` threads for the matvecs. Returns 0, or -1 on a bad token/pos. */
int efo_forward(efo_state* s, int32_t token, size_t pos, float* logits, int threads);

/* Generic row lookup as float (qkernels.cpp:299-305). */
void efo_row_f32(float* out, const efo_weight* w, size_t r);

#ifdef __cplusplus
}
#endif
#endif /* EFO_H */
