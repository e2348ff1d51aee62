/*
 * pllm_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * A scalar C restatement of the reference's quantized forward kernels (takano32/pyodide-llm, the .ts files of kernels/), kept in
 * the reference's own lane order and float32 rounding order so that its results are the reference's to the bit.
 * It is the checker for the CUDA library and the timed CPU baseline; no product code path may call it.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU legs load it.
 *
 * Every pointer is a host pointer. Byte strides (os, frame) are in bytes, as in the reference.
 * Each function cites the reference file:line it restates.
 */
#ifndef PLLM_ORACLE_H
#define PLLM_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- numeric helpers (kernels/kernel/math.ts, kernels/kernel/halves.ts) */
float or_fexp(float x);                 /* math.ts:28-43: table-free exp, one value */
float or_vexp(float x);                 /* math.ts:46-58: the same, four-lane form (clamps below -87) */
float or_half(uint16_t h);              /* halves.ts:21-23: float16 -> float32 as the kernels widen it */

/* ---- activations (kernels/kernel/quantize.ts, kernels/kernel/matmul.ts) */
void or_quantize_x(uint8_t *xq, float *xs, const float *x, int32_t n, int32_t bias);  /* quantize.ts:124-151 */
void or_int8_sums(int32_t *out, const int8_t *w, int32_t groups);                       /* matmul.ts:50-58 */
void or_six_sums(int32_t *out, const uint8_t *w, int32_t groups);                       /* matmul.ts:38-46 */
void or_interleave(uint8_t *xq, float *xs, int32_t n);                                  /* matmul.ts:129-146 */
void or_widen6(int8_t *out, const uint8_t *group24);                                    /* six.ts:16-31 */

/* ---- products (int32 group sums exact, float32 in the reference's lane order) */
void or_matmul_q8(float *xout, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                  int32_t n, int32_t r0, int32_t r1);                                   /* matmul.ts:77-104 */
void or_matmul_q8r(float *xout, const uint8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                   const int32_t *wc, int32_t n, int32_t r0, int32_t r1);               /* relaxed/int8.ts:17-50 */
void or_matmul_q8r_tile(float *xout, const uint8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                        const int32_t *wc, int32_t n, int32_t r0, int32_t r1, int32_t count, int32_t os,
                        int32_t frame);                                                 /* relaxed/int8.ts:147-166 */
void or_matmul_q6(float *xout, const int8_t *xq, const float *xs, const uint8_t *wq, const float *ws,
                  int32_t n, int32_t r0, int32_t r1);                                   /* matmul.ts:227-244 */
void or_matmul_q6r(float *xout, const uint8_t *xq, const float *xs, const uint8_t *wq, const float *ws,
                   const int32_t *wc, int32_t n, int32_t r0, int32_t r1);               /* relaxed/six.ts:16-39 */
/* ternary (binary = 0) or binary (binary = 1) weights against interleaved activations; code is the mask the
 * reference passes (3 for ternary, 2 for binary) */
void or_matmul_signs(float *xout, const uint8_t *xq, const float *xs, const uint8_t *wq, const uint16_t *ws,
                     int32_t n, int32_t r0, int32_t r1, int32_t code, int32_t binary); /* matmul.ts:183-224, relaxed/signs.ts:28-127 */
void or_matmul_signs_tile(float *xout, const uint8_t *xq, const float *xs, const uint8_t *wq, const uint16_t *ws,
                          int32_t n, int32_t r0, int32_t r1, int32_t count, int32_t os, int32_t frame,
                          int32_t code, int32_t binary);                                /* relaxed/signs.ts:77-114 */
void or_matmul_f32(float *xout, const float *x, const float *w, int32_t n, int32_t r0, int32_t r1); /* matmul.ts:13-33 */

/* exact int32 sums of every (row, group of 32): the accumulators the products scale (q8/q6 plain: signed acts;
 * q8r/q6r: acts biased by 64, the correction applied; signs: interleaved acts and their sums) */
void or_group_sums_q8(int32_t *out, const uint8_t *xq, const int8_t *wq, int32_t n, int32_t r0, int32_t r1, int32_t bias);
void or_group_sums_q6(int32_t *out, const uint8_t *xq, const uint8_t *wq, int32_t n, int32_t r0, int32_t r1, int32_t bias);
void or_group_sums_signs(int32_t *out, const uint8_t *xq, const float *xs, const uint8_t *wq, int32_t n, int32_t r0,
                         int32_t r1, int32_t code, int32_t binary);

/* ---- attention and rope (kernels/kernel/attention.ts) */
void or_rope(float *v, const float *fcr, const float *fci, int32_t nh, int32_t hs, int32_t rot); /* attention.ts:7-20 */
/* half: 0 float32 cache, 1 float16 cache; cap: 0 for none */
void or_attention(float *out, const float *q, const void *kc, const void *vc, float *att, int32_t pos, int32_t nh,
                  int32_t nkv, int32_t hs, int32_t h0, int32_t h1, int32_t half, float cap); /* attention.ts:87-211 */

/* ---- float16 (kernels/kernel/halves.ts) */
int32_t or_to_f16(uint16_t *out, const float *x, int32_t n);    /* halves.ts:35-67 */
void or_from_f16(float *out, const uint16_t *x, int32_t n);     /* halves.ts:72-76 */
int32_t or_finite_f16(const uint16_t *x, int32_t n);            /* halves.ts:82-94 */

/* ---- vector glue (kernels/kernel/activations.ts) and stateful layers (kernels/kernel/stateful.ts) */
void or_rmsnorm(float *out, const float *x, const float *w, int32_t n, float eps);        /* activations.ts:8-20 */
void or_swiglu(float *out, const float *h1, const float *h3, int32_t n);                  /* activations.ts:77-90 */
void or_add_inplace(float *x, const float *y, int32_t n);                                 /* activations.ts:156-158 */
int32_t or_argmax(const float *x, int32_t n);                                             /* sample.ts:6-10 */
void or_penalize(float *logits, const int32_t *tokens, int32_t count, float penalty, float presence); /* sample.ts:16-30 */
int32_t or_sb_size(int32_t type);
int32_t or_sb_tables(uint8_t *area, const uint8_t *codebooks);                          /* blocks/types.ts:294-322 */
void or_sums_x(float *xs, const int8_t *xq, int32_t n);                                /* blocks/token.ts:158-172 */
void or_matmul_sb(float *out, const int8_t *xq, const float *xs, const uint8_t *w, const uint8_t *tab, int32_t n,
                  int32_t r0, int32_t r1, int32_t type);                                /* blocks/token.ts:130-141 */
void or_sb_row(float *out, const uint8_t *w, const uint8_t *tab, int32_t n, int32_t type); /* blocks/row.ts:21-72 */
int32_t or_sample(const float *logits, int32_t n, float temperature, float topp, double random, int32_t topk,
                  float minp);                                                          /* sample.ts:248-337 */
void or_gate(float *out, const float *x, const float *g, int32_t n);                      /* stateful.ts:12-23 */
void or_convolve(float *out, const float *taps, const float *rows, int32_t n, int32_t count); /* stateful.ts:49-63 */
void or_short_conv(float *out, const float *taps, float *rows, const float *b, int32_t n, int32_t count); /* stateful.ts:70-86 */
void or_delta_rule(float *out, const float *state, float *next, const float *c, float *work, int32_t kh, int32_t kd,
                   int32_t vd, int32_t vh, int32_t h0, int32_t h1);                      /* stateful.ts:96-151 */

/* ---- a decoder forward pass over these kernels (forward/engine.ts:421-475 run(); attention layer
 * forward/attention.ts:171-197; gated FFN forward/ffn.ts:25-35), threaded over rows and heads as
 * forward/threads.ts shares them. One token, batch 1. Weights in the reference's int8 group-of-32 format. */
typedef struct {
  int32_t dim, hidden, layers, heads, kv_heads, head_size, vocab, seq_len;
  int32_t qk_norm;      /* Qwen3's per-head RMSNorm of q and k */
  int32_t relaxed;      /* 1: matmul_q8r arithmetic (bias 64), 0: matmul_q8 (bias 0) */
  int32_t half_kv;      /* 1: float16 cache (to_f16 / attention_f16) */
  float eps;
} or_config;

typedef struct {
  const int8_t *wq, *wk, *wv, *wo, *w1, *w2, *w3;   /* [layers][rows][cols] int8 */
  const float *sq, *sk, *sv, *so, *s1, *s2, *s3;    /* [layers][rows][cols/32] */
  const int32_t *cq, *ck, *cv, *co, *c1, *c2, *c3;  /* corrections (relaxed only; may be NULL otherwise) */
  const int8_t *emb; const float *emb_s;            /* [vocab][dim] int8 + [vocab][dim/32] */
  const int8_t *cls; const float *cls_s; const int32_t *cls_c;
  const float *att_norm, *ffn_norm, *final_norm;    /* [layers][dim], [layers][dim], [dim] */
  const float *q_norm, *k_norm;                     /* [layers][head_size] (qk_norm only) */
  const float *cos_t, *sin_t;                       /* [seq_len][head_size/2] */
  void *kc, *vc;                                    /* [layers][seq_len][kv_heads*head_size], f32 or f16 */
} or_weights;

/* one decode step at pos: logits (vocab floats); returns 0, or -1 on a bad argument. threads <= 0: all */
int32_t or_forward(const or_config *c, const or_weights *w, int32_t token, int32_t pos, float *logits, int32_t threads);
/* the number of threads the OpenMP runtime would use (the CPU baseline reports it) */
int32_t or_threads(void);

#ifdef __cplusplus
}
#endif
#endif
