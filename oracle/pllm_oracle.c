/*
 * pllm_oracle.c -- TEST INFRASTRUCTURE ONLY: the CPU restatement of the reference's kernels that the CUDA library
 * is checked against (and that bench.py times as the CPU baseline). Nothing in the product links it.
 *
 * Restated from takano32/pyodide-llm's AssemblyScript kernels, function by function (file:line beside each). Each
 * keeps the reference's order of float32 operations: the reference's int8 results depend on the order of its adds,
 * and its own tests (tests/int8-check.ts:65-91) hold the kernels to written-out models in exactly that order.
 * Built with -ffp-contract=off: WASM SIMD has no fused multiply-add, so neither may this.
 */
#include "pllm_oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <float.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define GS 32

static inline float bits_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* WASM's f32 max/min: a NaN in either operand gives NaN (the lanes of f32x4.max and f32.max alike) */
static inline float wmax(float a, float b) {
  if (a != a || b != b) return NAN;
  if (a == 0.0f && b == 0.0f) return signbit(a) ? b : a;
  return a > b ? a : b;
}
static inline float wmin(float a, float b) {
  if (a != a || b != b) return NAN;
  if (a == 0.0f && b == 0.0f) return signbit(a) ? a : b;
  return a < b ? a : b;
}
/* i32.trunc_sat_f32_s */
static inline int32_t trunc_sat(float v) {
  if (v != v) return 0;
  if (v >= 2147483648.0f) return INT32_MAX;
  if (v <= -2147483648.0f) return INT32_MIN;
  return (int32_t)v;
}
static inline int32_t sat8(int32_t v) { return v < -128 ? -128 : v > 127 ? 127 : v; }

/* ---------------------------------------------------------------------------------------------------------------
 * exp: the reference's table-free exponential (kernels/kernel/math.ts:28-58) is the Cephes single-precision expf
 * (S. L. Moshier, Cephes Math Library, expf.c): x = k ln2 + r with ln2 split in two parts, and a degree-5
 * polynomial in r. Restated from that published method. */
#define LOG2E 1.44269504088896341f
#define LN2_HI 0.693359375f
#define LN2_LO -2.12194440e-4f
static inline float exp_poly(float x, float k) {
  const float r = (x - k * LN2_HI) - k * LN2_LO;
  float p = 1.9875691500e-4f;
  p = p * r + 1.3981999507e-3f;
  p = p * r + 8.3334519073e-3f;
  p = p * r + 4.1665795894e-2f;
  p = p * r + 1.6666665459e-1f;
  p = p * r + 5.0000001201e-1f;
  return (p * (r * r) + r) + 1.0f;
}
float or_fexp(float x) {
  if (x < -87.0f) return 0.0f;
  if (x > 88.0f) x = 88.0f;
  const float k = rintf(x * LOG2E);
  const float e = exp_poly(x, k);
  return e * bits_f((uint32_t)((int32_t)k + 127) << 23);
}
float or_vexp(float x) {
  x = wmin(wmax(x, -87.0f), 88.0f);
  const float k = rintf(x * LOG2E);
  const float e = exp_poly(x, k);
  return e * bits_f((uint32_t)(trunc_sat(k) + 127) << 23);
}

/* halves.ts:12-23: the half's bits sign-extended, shifted by 13, the three copies of the sign cleared, times 2^112 */
float or_half(uint16_t h) {
  const int32_t s = (int32_t)(int16_t)h;
  return bits_f((uint32_t)(s << 13) & 0x8fffffffu) * 5.192296858534828e33f;
}

/* ---------------------------------------------------------------------------------------------------------------
 * quantize_x (kernels/kernel/quantize.ts:124-151; groupMax :8-19): per group of 32, the largest |x| lane by lane
 * (lane l holds values 4i + l), the lanes compared in order, scale = amax / qmax, q = sat8(trunc_sat(rne(x / s)) + bias) */
void or_quantize_x(uint8_t *xq, float *xs, const float *x, int32_t n, int32_t bias) {
  const float qmax = bias == 0 ? 127.0f : 63.0f;
  for (int32_t g = 0; g < n; g += GS) {
    const float *p = x + g;
    float m[4];
    for (int l = 0; l < 4; l++) {
      float a = wmax(wmax(wmax(fabsf(p[l]), fabsf(p[4 + l])), wmax(fabsf(p[8 + l]), fabsf(p[12 + l]))),
                     wmax(wmax(fabsf(p[16 + l]), fabsf(p[20 + l])), wmax(fabsf(p[24 + l]), fabsf(p[28 + l]))));
      m[l] = a;
    }
    float amax = m[0];
    if (m[1] > amax) amax = m[1];
    if (m[2] > amax) amax = m[2];
    if (m[3] > amax) amax = m[3];
    const float scale = amax / qmax;
    xs[g / GS] = scale;
    const float inv = scale > 0 ? 1.0f / scale : 0.0f;
    for (int j = 0; j < GS; j++) {
      const int32_t q = (int32_t)((uint32_t)trunc_sat(rintf(p[j] * inv)) + (uint32_t)bias);  /* wraps, as i32x4.add */
      xq[g + j] = (uint8_t)(int8_t)sat8(q);
    }
  }
}

/* matmul.ts:50-58: -64 times the sum of each group of 32 int8 weights */
void or_int8_sums(int32_t *out, const int8_t *w, int32_t groups) {
  for (int32_t g = 0; g < groups; g++) {
    int32_t s = 0;
    for (int j = 0; j < GS; j++) s += w[g * GS + j];
    out[g] = -64 * s;
  }
}

/* six.ts:16-31 (the layout of engine/packing.py:56-63 pack6): value v's low four bits are the low nibble of byte v
 * (v < 16) or the high nibble of byte v - 16; its top two bits are bits 2 (v / 8) of byte 16 + v % 8; the int8 is
 * (top << 6 | low << 2) */
void or_widen6(int8_t *out, const uint8_t *b) {
  for (int v = 0; v < 32; v++) {
    const uint32_t low = v < 16 ? (b[v] & 15u) : (uint32_t)(b[v - 16] >> 4);
    const uint32_t top = (b[16 + (v & 7)] >> (2 * (v >> 3))) & 3u;
    out[v] = (int8_t)(uint8_t)((top << 6) | (low << 2));
  }
}

/* matmul.ts:38-46 */
void or_six_sums(int32_t *out, const uint8_t *w, int32_t groups) {
  int8_t v[32];
  for (int32_t g = 0; g < groups; g++) {
    or_widen6(v, w + (size_t)g * 24);
    int32_t s = 0;
    for (int j = 0; j < GS; j++) s += v[j];
    out[g] = -64 * s;
  }
}

/* matmul.ts:129-146: per block of 64, byte 16 p + c <- activation 4 c + p; after the n / 32 scales, an int32 a group:
 * minus the sum of its 32 activations */
void or_interleave(uint8_t *xq, float *xs, int32_t n) {
  int32_t *sums = (int32_t *)(xs + n / 32);
  uint8_t blk[64];
  for (int32_t b = 0; b < n; b += 64) {
    int32_t s0 = 0, s1 = 0;
    for (int j = 0; j < 32; j++) s0 += (int8_t)xq[b + j];
    for (int j = 32; j < 64; j++) s1 += (int8_t)xq[b + j];
    sums[b / 32] = -s0;
    sums[b / 32 + 1] = -s1;
    for (int a = 0; a < 64; a++) blk[16 * (a & 3) + (a >> 2)] = xq[b + a];
    memcpy(xq + b, blk, 64);
  }
}

/* ---------------------------------------------------------------------------------------------------------------
 * int8 products */

/* dot32 (matmul.ts:68-72): lane k holds products 2k, 2k+1, 2k+8, 2k+9 of each half of the group; two products are
 * added in int16 (wrapping) before the widening */
static inline void dot32_lanes(const int8_t *w, const int8_t *a, int32_t lanes[4]) {
  for (int k = 0; k < 4; k++) lanes[k] = 0;
  for (int h = 0; h < 32; h += 16) {
    int16_t t[8];
    for (int j = 0; j < 8; j++) t[j] = (int16_t)((int32_t)w[h + j] * a[h + j] + (int32_t)w[h + j + 8] * a[h + j + 8]);
    for (int k = 0; k < 4; k++) lanes[k] += (int32_t)t[2 * k] + (int32_t)t[2 * k + 1];
  }
}

/* matmul.ts:77-104: lane k of every group, times the product of the two scales, into float32 lane k; the four lanes
 * added in order at the end */
static float row_q8(const int8_t *row, const int8_t *xq, const float *srow, const float *xs, int32_t ng) {
  float facc[4] = {0, 0, 0, 0};
  int32_t lanes[4];
  for (int32_t g = 0; g < ng; g++) {
    const float s = srow[g] * xs[g];
    dot32_lanes(row + (size_t)g * GS, xq + (size_t)g * GS, lanes);
    for (int k = 0; k < 4; k++) facc[k] = facc[k] + (float)lanes[k] * s;
  }
  return ((facc[0] + facc[1]) + facc[2]) + facc[3];
}

void or_matmul_q8(float *xout, const int8_t *xq, const float *xs, const int8_t *wq, const float *ws, int32_t n,
                  int32_t r0, int32_t r1) {
  const int32_t ng = n / GS;
  for (int32_t i = r0; i < r1; i++)
    xout[i] = row_q8(wq + (size_t)i * n, xq, ws + (size_t)i * ng, xs, ng);
}

/* the exact integer dot(w, q - 64) of a group (relaxed_dot_i8x16_i7x16 on 0..127 activations, plus the correction
 * -64 sum(w)): computed directly; the correction array, when given, must be int8_sums' (it is added instead) */
static inline int32_t group_q8r(const int8_t *w, const uint8_t *q, const int32_t *wc) {
  int32_t s = 0;
  if (wc) {
    for (int j = 0; j < GS; j++) s += (int32_t)w[j] * (int32_t)q[j];
    return s + *wc;
  }
  for (int j = 0; j < GS; j++) s += (int32_t)w[j] * ((int32_t)q[j] - 64);
  return s;
}

/* relaxed/int8.ts:17-50: lane g % 4 adds the groups of the first ng & ~3 in order; the lanes added in order; then the
 * groups past the fours one at a time */
static float row_q8r(const int8_t *row, const uint8_t *xq, const float *srow, const int32_t *crow, const float *xs,
                     int32_t ng) {
  const int32_t ng4 = ng & ~3;
  float facc[4] = {0, 0, 0, 0};
  int32_t g = 0;
  for (; g < ng4; g++) {
    const int32_t G = group_q8r(row + (size_t)g * GS, xq + (size_t)g * GS, crow ? crow + g : NULL);
    facc[g & 3] = facc[g & 3] + (float)G * (srow[g] * xs[g]);
  }
  float sum = ((facc[0] + facc[1]) + facc[2]) + facc[3];
  for (; g < ng; g++) {
    const int32_t G = group_q8r(row + (size_t)g * GS, xq + (size_t)g * GS, crow ? crow + g : NULL);
    sum = sum + (float)G * (srow[g] * xs[g]);
  }
  return sum;
}

void or_matmul_q8r(float *xout, const uint8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                   const int32_t *wc, int32_t n, int32_t r0, int32_t r1) {
  const int32_t ng = n / GS;
  for (int32_t i = r0; i < r1; i++)
    xout[i] = row_q8r(wq + (size_t)i * n, xq, ws + (size_t)i * ng, wc ? wc + (size_t)i * ng : NULL, xs, ng);
}

/* relaxed/int8.ts:147-166: every (row, token) is matmul_q8r's number; token t at xq + t frame, xs + t frame (bytes),
 * its outputs at xout + t os (bytes) */
void or_matmul_q8r_tile(float *xout, const uint8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                        const int32_t *wc, int32_t n, int32_t r0, int32_t r1, int32_t count, int32_t os,
                        int32_t frame) {
  for (int32_t t = 0; t < count; t++)
    or_matmul_q8r((float *)((char *)xout + (size_t)t * os), xq + (size_t)t * frame,
                  (const float *)((const char *)xs + (size_t)t * frame), wq, ws, wc, n, r0, r1);
}

/* matmul.ts:227-244: matmul_q8 on the widened int6 groups (24 bytes a group) */
void or_matmul_q6(float *xout, const int8_t *xq, const float *xs, const uint8_t *wq, const float *ws, int32_t n,
                  int32_t r0, int32_t r1) {
  const int32_t ng = n / GS;
  int8_t *row = (int8_t *)malloc((size_t)n);
  for (int32_t i = r0; i < r1; i++) {
    for (int32_t g = 0; g < ng; g++) or_widen6(row + (size_t)g * GS, wq + ((size_t)i * ng + g) * 24);
    xout[i] = row_q8(row, xq, ws + (size_t)i * ng, xs, ng);
  }
  free(row);
}

/* relaxed/six.ts:16-39: matmul_q8r on the widened groups */
void or_matmul_q6r(float *xout, const uint8_t *xq, const float *xs, const uint8_t *wq, const float *ws,
                   const int32_t *wc, int32_t n, int32_t r0, int32_t r1) {
  const int32_t ng = n / GS;
  int8_t *row = (int8_t *)malloc((size_t)n);
  for (int32_t i = r0; i < r1; i++) {
    for (int32_t g = 0; g < ng; g++) or_widen6(row + (size_t)g * GS, wq + ((size_t)i * ng + g) * 24);
    xout[i] = row_q8r(row, xq, ws + (size_t)i * ng, wc ? wc + (size_t)i * ng : NULL, xs, ng);
  }
  free(row);
}

/* ---------------------------------------------------------------------------------------------------------------
 * ternary and binary products (matmul.ts:148-224 plain, relaxed/signs.ts:17-127 relaxed: the same numbers).
 * A group of 128 weights; sub-group s (0..3) is its s-th 32 activations. Its exact integer is
 *   whole_s = sum code_j a_j + sums[4g + s]   (= sum (code_j - 1) a_j: the weights -1, 0, 1)
 * with a_j read from the interleaved activations (block 64 (j / 64), byte 16 (j & 3) + (j % 64) / 4); ternary's code of
 * weight j is bits 2 (j & 3) of byte j / 4 (ternary.ts:25-27), binary's is twice bit 4 (j / 64) + (j & 3) of byte
 * (j % 64) / 4 (binary.ts:20-22). Lane s += float32(whole_s) * xs[4g + s] * d, d the group's float16 scale. */
static inline int32_t signs_code(const uint8_t *grp, int j, int32_t code, int32_t binary) {
  if (!binary) return (grp[j >> 2] >> (2 * (j & 3))) & code;
  const int bit = 4 * (j >> 6) + (j & 3);
  return ((grp[(j & 63) >> 2] >> bit) & 1) ? (code & 2) : 0;
}
static inline int8_t signs_act(const uint8_t *xg, int j) {  /* xg: the group's 128 interleaved activations */
  const int a = j & 63;
  return (int8_t)xg[64 * (j >> 6) + 16 * (a & 3) + (a >> 2)];
}
static inline int32_t signs_whole(const uint8_t *grp, const uint8_t *xg, const int32_t *sums, int s, int32_t code,
                                  int32_t binary) {
  int32_t acc = 0;
  for (int j = 32 * s; j < 32 * s + 32; j++) acc += signs_code(grp, j, code, binary) * (int32_t)signs_act(xg, j);
  return acc + sums[s];
}
static float row_signs(const uint8_t *row, const uint16_t *srow, const uint8_t *xq, const float *xs,
                       const int32_t *sums, int32_t groups, int32_t code, int32_t binary) {
  const int bytes = binary ? 16 : 32;
  float facc[4] = {0, 0, 0, 0};
  for (int32_t g = 0; g < groups; g++) {
    const float d = or_half(srow[g]);
    for (int s = 0; s < 4; s++) {
      const int32_t whole = signs_whole(row + (size_t)g * bytes, xq + (size_t)g * 128, sums + 4 * g, s, code, binary);
      facc[s] = facc[s] + ((float)whole * xs[4 * g + s]) * d;
    }
  }
  return ((facc[0] + facc[1]) + facc[2]) + facc[3];
}
void or_matmul_signs(float *xout, const uint8_t *xq, const float *xs, const uint8_t *wq, const uint16_t *ws,
                     int32_t n, int32_t r0, int32_t r1, int32_t code, int32_t binary) {
  const int32_t groups = n >> 7;
  const size_t rb = binary ? (size_t)(n >> 3) : (size_t)(n >> 2);
  const int32_t *sums = (const int32_t *)(xs + (n >> 5));
  for (int32_t i = r0; i < r1; i++)
    xout[i] = row_signs(wq + (size_t)i * rb, ws + (size_t)i * groups, xq, xs, sums, groups, code, binary);
}
/* relaxed/signs.ts:77-114: a row against count tokens, each (row, token) the token kernel's number */
void or_matmul_signs_tile(float *xout, const uint8_t *xq, const float *xs, const uint8_t *wq, const uint16_t *ws,
                          int32_t n, int32_t r0, int32_t r1, int32_t count, int32_t os, int32_t frame,
                          int32_t code, int32_t binary) {
  for (int32_t t = 0; t < count; t++)
    or_matmul_signs((float *)((char *)xout + (size_t)t * os), xq + (size_t)t * frame,
                    (const float *)((const char *)xs + (size_t)t * frame), wq, ws, n, r0, r1, code, binary);
}

/* ---- the exact group sums (the accumulators every product scales) */
void or_group_sums_q8(int32_t *out, const uint8_t *xq, const int8_t *wq, int32_t n, int32_t r0, int32_t r1,
                      int32_t bias) {
  const int32_t ng = n / GS;
  for (int32_t i = r0; i < r1; i++)
    for (int32_t g = 0; g < ng; g++) {
      int32_t s = 0;
      for (int j = 0; j < GS; j++)
        s += (int32_t)wq[(size_t)i * n + g * GS + j] *
             (bias ? (int32_t)xq[g * GS + j] - bias : (int32_t)(int8_t)xq[g * GS + j]);
      out[(size_t)(i - r0) * ng + g] = s;
    }
}
void or_group_sums_q6(int32_t *out, const uint8_t *xq, const uint8_t *wq, int32_t n, int32_t r0, int32_t r1,
                      int32_t bias) {
  const int32_t ng = n / GS;
  int8_t v[32];
  for (int32_t i = r0; i < r1; i++)
    for (int32_t g = 0; g < ng; g++) {
      or_widen6(v, wq + ((size_t)i * ng + g) * 24);
      int32_t s = 0;
      for (int j = 0; j < GS; j++)
        s += (int32_t)v[j] * (bias ? (int32_t)xq[g * GS + j] - bias : (int32_t)(int8_t)xq[g * GS + j]);
      out[(size_t)(i - r0) * ng + g] = s;
    }
}
void or_group_sums_signs(int32_t *out, const uint8_t *xq, const float *xs, const uint8_t *wq, int32_t n, int32_t r0,
                         int32_t r1, int32_t code, int32_t binary) {
  const int32_t groups = n >> 7, bytes = binary ? 16 : 32;
  const size_t rb = (size_t)groups * bytes;
  const int32_t *sums = (const int32_t *)(xs + (n >> 5));
  for (int32_t i = r0; i < r1; i++)
    for (int32_t g = 0; g < groups; g++)
      for (int s = 0; s < 4; s++)
        out[(size_t)(i - r0) * (n >> 5) + 4 * g + s] =
            signs_whole(wq + (size_t)i * rb + (size_t)g * bytes, xq + (size_t)g * 128, sums + 4 * g, s, code, binary);
}

/* matmul.ts:13-33: four accumulators of four lanes over 16 values a step, lane-wise sums (a0+a1)+(a2+a3), hsum, then
 * the values past the sixteens one at a time */
void or_matmul_f32(float *xout, const float *x, const float *w, int32_t n, int32_t r0, int32_t r1) {
  const int32_t n16 = n & ~15;
  for (int32_t i = r0; i < r1; i++) {
    const float *row = w + (size_t)i * n;
    float a[4][4] = {{0}};
    int32_t j = 0;
    for (; j < n16; j += 16)
      for (int v = 0; v < 4; v++)
        for (int l = 0; l < 4; l++) a[v][l] = a[v][l] + row[j + 4 * v + l] * x[j + 4 * v + l];
    float t[4];
    for (int l = 0; l < 4; l++) t[l] = (a[0][l] + a[1][l]) + (a[2][l] + a[3][l]);
    float val = ((t[0] + t[1]) + t[2]) + t[3];
    for (; j < n; j++) val = val + row[j] * x[j];
    xout[i] = val;
  }
}

/* ---------------------------------------------------------------------------------------------------------------
 * rope (attention.ts:7-20): pairs (v0, v1) of the first rot values of every head turned by the tables' (c, s) */
void or_rope(float *v, const float *fcr, const float *fci, int32_t nh, int32_t hs, int32_t rot) {
  const int32_t turned = rot > 0 && rot < hs ? rot : hs;
  for (int32_t h = 0; h < nh; h++) {
    float *base = v + (size_t)h * hs;
    for (int32_t i = 0; i < turned; i += 2) {
      const float c = fcr[i >> 1], s = fci[i >> 1];
      const float v0 = base[i], v1 = base[i + 1];
      base[i] = v0 * c - v1 * s;
      base[i + 1] = v0 * s + v1 * c;
    }
  }
}

static inline float kv_at(const void *p, size_t i, int half) {
  return half ? or_half(((const uint16_t *)p)[i]) : ((const float *)p)[i];
}

/* attention.ts:87-211 (attentionOf). Scores four positions at a time (each a four-lane accumulator over the head's
 * fours, sums4's order (l0 + l2) + (l1 + l3), then the values past the fours), a last position or three alone in
 * the same order; softmax with the largest score, vexp on the fours and fexp after them, the sum of four lanes then
 * the rest; the weighted values four positions at a time ((w0 v0 + w1 v1) + (w2 v2 + w3 v3) added to out). */
void or_attention(float *out, const float *q, const void *kc, const void *vc, float *att, int32_t pos, int32_t nh,
                  int32_t nkv, int32_t hs, int32_t h0, int32_t h1, int32_t half, float cap) {
  const int32_t kvDim = nkv * hs, kvMul = nh / nkv, hs4 = hs & ~3;
  const int32_t count = pos + 1, count4 = count & ~3;
  const float isq = 1.0f / sqrtf((float)hs);
  int32_t t = 0;
  for (; t < count4; t += 4) {
    for (int32_t h = h0; h < h1; h++) {
      const float *qh = q + (size_t)h * hs;
      const size_t k0 = (size_t)t * kvDim + (size_t)(h / kvMul) * hs;
      float a[4][4] = {{0}};
      int32_t j = 0;
      for (; j < hs4; j += 4)
        for (int i = 0; i < 4; i++)
          for (int l = 0; l < 4; l++)
            a[i][l] = a[i][l] + qh[j + l] * kv_at(kc, k0 + (size_t)i * kvDim + j + l, half);
      float sc[4];
      for (int i = 0; i < 4; i++) sc[i] = (a[i][0] + a[i][2]) + (a[i][1] + a[i][3]);
      for (; j < hs; j++)
        for (int i = 0; i < 4; i++) sc[i] = sc[i] + qh[j] * kv_at(kc, k0 + (size_t)i * kvDim + j, half);
      for (int i = 0; i < 4; i++) att[(size_t)h * count + t + i] = sc[i] * isq;
    }
  }
  for (; t < count; t++) {
    for (int32_t h = h0; h < h1; h++) {
      const float *qh = q + (size_t)h * hs;
      const size_t kt = (size_t)t * kvDim + (size_t)(h / kvMul) * hs;
      float a[4] = {0, 0, 0, 0};
      int32_t j = 0;
      for (; j < hs4; j += 4)
        for (int l = 0; l < 4; l++) a[l] = a[l] + qh[j + l] * kv_at(kc, kt + j + l, half);
      float sc = (a[0] + a[2]) + (a[1] + a[3]);
      for (; j < hs; j++) sc = sc + qh[j] * kv_at(kc, kt + j, half);
      att[(size_t)h * count + t] = sc * isq;
    }
  }
  for (int32_t h = h0; h < h1; h++) {
    float *scores = att + (size_t)h * count;
    if (cap > 0) {
      const float twice = 2.0f / cap;
      int32_t c = 0;
      for (; c < count4; c++) scores[c] = cap * (1.0f - 2.0f / (or_vexp(scores[c] * twice) + 1.0f));
      for (; c < count; c++) scores[c] = cap * (1.0f - 2.0f / (or_fexp(scores[c] * twice) + 1.0f));
    }
    float mx = -FLT_MAX;  /* math.ts:67-89 largest: a NaN anywhere makes it NaN */
    for (int32_t c = 0; c < count; c++) mx = wmax(mx, scores[c]);
    float sums[4] = {0, 0, 0, 0};
    int32_t u = 0;
    for (; u < count4; u++) {
      const float e = or_vexp(scores[u] - mx);
      scores[u] = e;
      sums[u & 3] = sums[u & 3] + e;
    }
    float sum = ((sums[0] + sums[1]) + sums[2]) + sums[3];
    for (; u < count; u++) {
      const float e = or_fexp(scores[u] - mx);
      scores[u] = e;
      sum = sum + e;
    }
    const float inv = 1.0f / sum;
    for (u = 0; u < count; u++) scores[u] = scores[u] * inv;
  }
  for (int32_t j = h0 * hs; j < h1 * hs; j++) out[j] = 0.0f;
  for (t = 0; t < count4; t += 4) {
    for (int32_t h = h0; h < h1; h++) {
      const float *wt = att + (size_t)h * count + t;
      float *oh = out + (size_t)h * hs;
      const size_t v0 = (size_t)t * kvDim + (size_t)(h / kvMul) * hs;
      int32_t j = 0;
      for (; j < hs4; j++) {
        const float pair0 = wt[0] * kv_at(vc, v0 + j, half) + wt[1] * kv_at(vc, v0 + kvDim + j, half);
        const float pair1 = wt[2] * kv_at(vc, v0 + 2 * (size_t)kvDim + j, half) + wt[3] * kv_at(vc, v0 + 3 * (size_t)kvDim + j, half);
        oh[j] = oh[j] + (pair0 + pair1);
      }
      for (; j < hs; j++)
        oh[j] = (((oh[j] + wt[0] * kv_at(vc, v0 + j, half)) + wt[1] * kv_at(vc, v0 + kvDim + j, half)) +
                 wt[2] * kv_at(vc, v0 + 2 * (size_t)kvDim + j, half)) + wt[3] * kv_at(vc, v0 + 3 * (size_t)kvDim + j, half);
    }
  }
  for (; t < count; t++) {
    for (int32_t h = h0; h < h1; h++) {
      const float weight = att[(size_t)h * count + t];
      float *oh = out + (size_t)h * hs;
      const size_t vt = (size_t)t * kvDim + (size_t)(h / kvMul) * hs;
      for (int32_t j = 0; j < hs; j++) oh[j] = oh[j] + weight * kv_at(vc, vt + j, half);
    }
  }
}

/* ---------------------------------------------------------------------------------------------------------------
 * float16 (halves.ts:35-94): round to nearest even, too large to infinity, counting the inputs that were not finite */
int32_t or_to_f16(uint16_t *out, const float *x, int32_t n) {
  int32_t bad = 0;
  for (int32_t i = 0; i < n; i++) {
    const uint32_t bits = f_bits(x[i]);
    const uint32_t sign = (bits >> 16) & 0x8000u;
    const int32_t exponent = (int32_t)((bits >> 23) & 0xff) - 112;
    uint32_t mantissa = bits & 0x7fffffu, result;
    if (exponent >= 31) {
      result = sign | 0x7c00u;
      if (exponent == 143) bad++;
    } else if (exponent <= 0) {
      if (exponent < -10) {
        result = sign;
      } else {
        mantissa |= 0x800000u;
        const uint32_t shift = (uint32_t)(14 - exponent);
        const uint32_t rest = mantissa & ((1u << shift) - 1), middle = 1u << (shift - 1);
        uint32_t value = mantissa >> shift;
        if (rest > middle || (rest == middle && (value & 1))) value++;
        result = sign | value;
      }
    } else {
      const uint32_t rest = mantissa & 0x1fffu;
      uint32_t value = ((uint32_t)exponent << 10) | (mantissa >> 13);
      if (rest > 0x1000u || (rest == 0x1000u && (value & 1))) value++;
      result = sign | value;
    }
    out[i] = (uint16_t)result;
  }
  return bad;
}
void or_from_f16(float *out, const uint16_t *x, int32_t n) {
  for (int32_t i = 0; i < n; i++) out[i] = or_half(x[i]);
}
int32_t or_finite_f16(const uint16_t *x, int32_t n) {
  for (int32_t i = 0; i < n; i++)
    if ((x[i] & 0x7c00u) == 0x7c00u) return 0;
  return 1;
}

/* ---------------------------------------------------------------------------------------------------------------
 * glue (activations.ts, stateful.ts). The four-lane kernels use vexp for the values of whole fours and fexp past
 * them; for these functions the two give the same numbers (1 + exp(-87) is 1), so one exp serves. */
void or_rmsnorm(float *out, const float *x, const float *w, int32_t n, float eps) {  /* activations.ts:8-20 */
  float acc[4] = {0, 0, 0, 0};
  const int32_t n4 = n & ~3;
  int32_t j = 0;
  for (; j < n4; j++) acc[j & 3] = acc[j & 3] + x[j] * x[j];
  float ss = ((acc[0] + acc[1]) + acc[2]) + acc[3];
  for (; j < n; j++) ss = ss + x[j] * x[j];
  const float s = 1.0f / sqrtf(ss / (float)n + eps);
  for (j = 0; j < n; j++) out[j] = w[j] * (s * x[j]);
}
void or_swiglu(float *out, const float *h1, const float *h3, int32_t n) {  /* activations.ts:77-90 */
  for (int32_t j = 0; j < n; j++) {
    const float v = h1[j];
    out[j] = (v / (1.0f + or_fexp(-v))) * h3[j];
  }
}
void or_add_inplace(float *x, const float *y, int32_t n) {  /* activations.ts:156-158 */
  for (int32_t j = 0; j < n; j++) x[j] = x[j] + y[j];
}
void or_gate(float *out, const float *x, const float *g, int32_t n) {  /* stateful.ts:12-23 */
  for (int32_t j = 0; j < n; j++) out[j] = x[j] / (1.0f + or_fexp(-g[j]));
}
static inline float taps_of(const float *taps, const float *rows, int32_t c, int32_t n, int32_t count) {
  float acc = taps[c] * rows[c];  /* stateful.ts:27-44: oldest first */
  for (int32_t j = 1; j < count; j++) acc = acc + taps[(size_t)j * n + c] * rows[(size_t)j * n + c];
  return acc;
}
void or_convolve(float *out, const float *taps, const float *rows, int32_t n, int32_t count) {  /* stateful.ts:49-63 */
  for (int32_t c = 0; c < n; c++) {
    const float acc = taps_of(taps, rows, c, n, count);
    out[c] = acc / (1.0f + or_fexp(-acc));
  }
}
void or_short_conv(float *out, const float *taps, float *rows, const float *b, int32_t n, int32_t count) {  /* stateful.ts:70-86 */
  float *newest = rows + (size_t)(count - 1) * n;
  const float *gate = b + n, *z = b + 2 * (size_t)n;
  for (int32_t c = 0; c < n; c++) {
    newest[c] = b[c] * z[c];
    out[c] = gate[c] * taps_of(taps, rows, c, n, count);
  }
}
void or_delta_rule(float *out, const float *state, float *next, const float *c, float *work, int32_t kh, int32_t kd,
                   int32_t vd, int32_t vh, int32_t h0, int32_t h1) {  /* stateful.ts:96-151 */
  const int32_t each = vh / kh;
  for (int32_t h = h0; h < h1; h++) {
    const int32_t key = h / each;
    const float *q = c + (size_t)key * kd, *k = c + (size_t)(kh + key) * kd;
    const float *v = c + (size_t)(2 * kh) * kd + (size_t)h * vd;
    const float beta = work[h], decay = work[vh + h];
    float *delta = work + 2 * (size_t)vh + (size_t)h * vd;
    const float *from = state + (size_t)h * kd * vd;
    float *to = next + (size_t)h * kd * vd, *o = out + (size_t)h * vd;
    for (int32_t j = 0; j < vd; j++) delta[j] = 0.0f;
    for (int32_t i = 0; i < kd; i++) {
      const float ki = k[i];
      for (int32_t j = 0; j < vd; j++) delta[j] = delta[j] + ki * (from[(size_t)i * vd + j] * decay);
    }
    for (int32_t j = 0; j < vd; j++) {
      delta[j] = (v[j] - delta[j]) * beta;
      o[j] = 0.0f;
    }
    for (int32_t i = 0; i < kd; i++) {
      const float ki = k[i], qi = q[i];
      for (int32_t j = 0; j < vd; j++) {
        const float s = from[(size_t)i * vd + j] * decay + ki * delta[j];
        to[(size_t)i * vd + j] = s;
        o[j] = o[j] + qi * s;
      }
    }
  }
}

/* ---------------------------------------------------------------------------------------------------------------
 * a decode step of a Llama / Qwen3-shaped int8 decoder, one token (forward/engine.ts:421-475; attention layer
 * forward/attention.ts:171-197; FFN forward/ffn.ts:25-35), the rows of every product and the heads of the attention
 * shared among OpenMP threads as forward/threads.ts shares them among software threads (the numbers do not depend on
 * how: every row and head is computed alone). */
int32_t or_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

static void product(const or_config *c, const int8_t *w, const float *s, const int32_t *corr, const uint8_t *xq,
                    const float *xs, float *out, int32_t rows, int32_t n) {
  const int32_t ng = n / GS;
#pragma omp parallel for schedule(static)
  for (int32_t i = 0; i < rows; i++) {
    if (c->relaxed)
      out[i] = row_q8r(w + (size_t)i * n, xq, s + (size_t)i * ng, corr ? corr + (size_t)i * ng : NULL, xs, ng);
    else
      out[i] = row_q8(w + (size_t)i * n, (const int8_t *)xq, s + (size_t)i * ng, xs, ng);
  }
}

int32_t or_forward(const or_config *c, const or_weights *w, int32_t token, int32_t pos, float *logits,
                   int32_t threads) {
  if (!c || !w || !logits || pos < 0 || pos >= c->seq_len || token < 0 || token >= c->vocab) return -1;
  if (c->dim % GS || c->hidden % GS || c->heads % c->kv_heads) return -1;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
  const int32_t dim = c->dim, hid = c->hidden, hs = c->head_size, nh = c->heads, nkv = c->kv_heads;
  const int32_t qdim = nh * hs, kvdim = nkv * hs, bias = c->relaxed ? 64 : 0, big = hid > qdim ? hid : qdim;
  const int32_t wide = big > dim ? big : dim;
  float *x = malloc(sizeof(float) * dim), *xb = malloc(sizeof(float) * wide), *xb2 = malloc(sizeof(float) * dim);
  float *q = malloc(sizeof(float) * qdim), *k = malloc(sizeof(float) * kvdim), *v = malloc(sizeof(float) * kvdim);
  float *hb = malloc(sizeof(float) * hid), *hb2 = malloc(sizeof(float) * hid);
  float *att = malloc(sizeof(float) * (size_t)nh * (pos + 1));
  uint8_t *xq = malloc((size_t)wide);
  float *xs = malloc(sizeof(float) * (wide / GS));
  const size_t E = c->half_kv ? 2 : 4;
  /* embed (forward/tensors.ts:154-160): the int8 value times its group's scale */
  for (int32_t i = 0; i < dim; i++)
    x[i] = (float)w->emb[(size_t)token * dim + i] * w->emb_s[((size_t)token * dim + i) / GS];
  for (int32_t l = 0; l < c->layers; l++) {
    const size_t lq = (size_t)l * qdim * dim, lk = (size_t)l * kvdim * dim, lo = (size_t)l * dim * qdim;
    const size_t l1 = (size_t)l * hid * dim, l2 = (size_t)l * dim * hid;
    or_rmsnorm(xb, x, w->att_norm + (size_t)l * dim, dim, c->eps);
    or_quantize_x(xq, xs, xb, dim, bias);
    product(c, w->wq + lq, w->sq + lq / GS, w->cq ? w->cq + lq / GS : NULL, xq, xs, q, qdim, dim);
    product(c, w->wk + lk, w->sk + lk / GS, w->ck ? w->ck + lk / GS : NULL, xq, xs, k, kvdim, dim);
    product(c, w->wv + lk, w->sv + lk / GS, w->cv ? w->cv + lk / GS : NULL, xq, xs, v, kvdim, dim);
    if (c->qk_norm) {
      for (int32_t h = 0; h < nh; h++) or_rmsnorm(q + h * hs, q + h * hs, w->q_norm + (size_t)l * hs, hs, c->eps);
      for (int32_t h = 0; h < nkv; h++) or_rmsnorm(k + h * hs, k + h * hs, w->k_norm + (size_t)l * hs, hs, c->eps);
    }
    or_rope(q, w->cos_t + (size_t)pos * (hs / 2), w->sin_t + (size_t)pos * (hs / 2), nh, hs, 0);
    or_rope(k, w->cos_t + (size_t)pos * (hs / 2), w->sin_t + (size_t)pos * (hs / 2), nkv, hs, 0);
    char *kl = (char *)w->kc + (size_t)l * c->seq_len * kvdim * E, *vl = (char *)w->vc + (size_t)l * c->seq_len * kvdim * E;
    if (c->half_kv) {
      or_to_f16((uint16_t *)(kl + (size_t)pos * kvdim * E), k, kvdim);
      or_to_f16((uint16_t *)(vl + (size_t)pos * kvdim * E), v, kvdim);
    } else {
      memcpy(kl + (size_t)pos * kvdim * E, k, sizeof(float) * kvdim);
      memcpy(vl + (size_t)pos * kvdim * E, v, sizeof(float) * kvdim);
    }
#pragma omp parallel for schedule(static)
    for (int32_t h = 0; h < nh; h++) or_attention(xb, q, kl, vl, att, pos, nh, nkv, hs, h, h + 1, c->half_kv, 0.0f);
    or_quantize_x(xq, xs, xb, qdim, bias);
    product(c, w->wo + lo, w->so + lo / GS, w->co ? w->co + lo / GS : NULL, xq, xs, xb2, dim, qdim);
    or_add_inplace(x, xb2, dim);
    or_rmsnorm(xb, x, w->ffn_norm + (size_t)l * dim, dim, c->eps);
    or_quantize_x(xq, xs, xb, dim, bias);
    product(c, w->w1 + l1, w->s1 + l1 / GS, w->c1 ? w->c1 + l1 / GS : NULL, xq, xs, hb, hid, dim);
    product(c, w->w3 + l1, w->s3 + l1 / GS, w->c3 ? w->c3 + l1 / GS : NULL, xq, xs, hb2, hid, dim);
    or_swiglu(hb, hb, hb2, hid);
    or_quantize_x(xq, xs, hb, hid, bias);
    product(c, w->w2 + l2, w->s2 + l2 / GS, w->c2 ? w->c2 + l2 / GS : NULL, xq, xs, xb2, dim, hid);
    or_add_inplace(x, xb2, dim);
  }
  or_rmsnorm(xb, x, w->final_norm, dim, c->eps);
  or_quantize_x(xq, xs, xb, dim, bias);
  product(c, w->cls, w->cls_s, w->cls_c, xq, xs, logits, c->vocab, dim);
  free(x); free(xb); free(xb2); free(q); free(k); free(v); free(hb); free(hb2); free(att); free(xq); free(xs);
  return 0;
}

/* sample.ts:6-10: the walk from the first element, a later one taking over only when strictly greater */
int32_t or_argmax(const float *x, int32_t n) {
  int32_t mi = 0;
  float mv = x[0];
  for (int32_t j = 1; j < n; j++)
    if (x[j] > mv) {
      mv = x[j];
      mi = j;
    }
  return mi;
}

/* sample.ts:16-30: each token once (its first occurrence), divided or multiplied by penalty, less presence */
void or_penalize(float *logits, const int32_t *tokens, int32_t count, float penalty, float presence) {
  const float less = presence > 0 ? presence : 0;
  for (int32_t i = 0; i < count; i++) {
    const int32_t token = tokens[i];
    int seen = 0;
    for (int32_t j = 0; j < i; j++)
      if (tokens[j] == token) {
        seen = 1;
        break;
      }
    if (seen) continue;
    const float value = logits[token];
    logits[token] = (value > 0 ? value / penalty : value * penalty) - less;
  }
}

/* sample.ts:248-337: a token drawn from softmax(logits / temperature), as the reference's kernel walks it.
 *  - best = the largest logit (a NaN anywhere, or an infinity: -1);
 *  - a nucleus (0 < topp < 1) leaves out what is below best - 16.118095 temperature (a ten millionth of the best's
 *    probability); the others, in token order, become exp((v - best) / temperature): the first 4 (count / 4) by
 *    vexp of the product with 1 / temperature, the rest by fexp of the quotient (sample.ts:274-282);
 *  - total (double) and top; top-k (0 < topk < count) keeps the topk largest by (probability, the lower token) and
 *    sums them again; least = min(minp, 1) top where minp > 0;
 *  - with a nucleus or a top-k: the kept at or above the cutoff ((1 - topp) / (count - 1) total, at most top) and at
 *    or above least, sorted by (probability, the lower token) descending, taken until their sum reaches topp total
 *    (every one without a nucleus); else with minp: those at or above least in token order; else all in token order;
 *  - the first whose cumulative sum (double) passes random x their sum, else the last.
 * The reference sums top-k's survivors in its partition's order; this sums them in the sorted order (the double's
 * last bits may differ). Scratch is allocated here. */
typedef struct {
  float p;
  int32_t t;
} or_place;
static int or_ahead(const void *a, const void *b) {
  const or_place *x = (const or_place *)a, *y = (const or_place *)b;
  if (x->p != y->p) return x->p > y->p ? -1 : 1;
  return x->t < y->t ? -1 : (x->t > y->t);
}
int32_t or_sample(const float *logits, int32_t n, float temperature, float topp, double random, int32_t topk,
                  float minp) {
  float best = logits[0];
  for (int32_t i = 1; i < n; i++) best = wmax(best, logits[i]);
  if (!isfinite(best)) return -1;
  const int nucleus = topp > 0 && topp < 1;
  const float floor_ = nucleus ? best - temperature * 16.118095f : -FLT_MAX;
  or_place *c = (or_place *)malloc(sizeof(or_place) * (size_t)n);
  int32_t count = 0;
  for (int32_t i = 0; i < n; i++)
    if (logits[i] >= floor_) {
      c[count].p = logits[i] - best;
      c[count].t = i;
      count++;
    }
  const float inverse = 1.0f / temperature;
  const int32_t fours = count / 4 * 4;
  for (int32_t i = 0; i < count; i++) c[i].p = i < fours ? or_vexp(c[i].p * inverse) : or_fexp(c[i].p / temperature);
  double total = 0;
  float top = 0;
  for (int32_t i = 0; i < count; i++) {
    total += c[i].p;
    top = top > c[i].p ? top : c[i].p;
  }
  const int narrowed = topk > 0 && topk < count;
  if (narrowed) {
    qsort(c, (size_t)count, sizeof(or_place), or_ahead);
    count = topk;
    total = 0;
    for (int32_t i = 0; i < count; i++) total += c[i].p;
  }
  const float least = minp > 0 ? (minp < 1.0f ? minp : 1.0f) * top : 0.0f;
  int32_t last = count - 1;
  double mass = total;
  if (nucleus || narrowed) {
    const double cutoff0 = (1.0 - (double)topp) / (double)(count > 1 ? count - 1 : 1) * total;
    const double cutoff = nucleus ? (cutoff0 < (double)top ? cutoff0 : (double)top) : 0;
    int32_t likely = 0;
    for (int32_t k = 0; k < count; k++)
      if ((double)c[k].p >= cutoff && c[k].p >= least) c[likely++] = c[k];
    qsort(c, (size_t)likely, sizeof(or_place), or_ahead);
    const double limit = nucleus ? (double)topp * total : INFINITY;
    mass = 0;
    last = likely - 1;
    for (int32_t k = 0; k < likely; k++) {
      mass += c[k].p;
      if (mass >= limit) {
        last = k;
        break;
      }
    }
  } else if (minp > 0) {
    int32_t likely = 0;
    mass = 0;
    for (int32_t k = 0; k < count; k++)
      if (c[k].p >= least) {
        mass += c[k].p;
        c[likely++] = c[k];
      }
    last = likely - 1;
  }
  const double target = random * mass;
  double cumulative = 0;
  int32_t token = last >= 0 ? c[last].t : -1;
  for (int32_t k = 0; k <= last; k++) {
    cumulative += c[k].p;
    if (cumulative > target) {
      token = c[k].t;
      break;
    }
  }
  free(c);
  return token;
}

/* ---------------------------------------------------------------------------------------------------------------
 * llama.cpp's blocks of 256 weights (kernels/blocks/types.ts): the ten types' reading, a unit of 16 weights at a time,
 * as signed integers W with the integer S of their unit and, for the K types, the integer minimum m; F and Fm of the
 * block; then the token's arithmetic of types.ts:66-83 (G[k] = sum over group k's 32 of S W a, exact;
 * lane k & 3 += ((G[k] xs[k] + G[k + 4] xs[k + 4]) F) - ((M[k] xs[k] + M[k + 4] xs[k + 4]) Fm); the lanes added in
 * order at the row's end). The tables are sb_tables' (types.ts:294-322): the grids, then the 7-bit signs' table, then
 * IQ4_XS's values, from the checkpoint's codebooks row. */
#define SB_T_IQ2XS 2048
#define SB_T_IQ2S 6144
#define SB_T_IQ3XXS 14336
#define SB_T_IQ3S 15360
#define SB_T_IQ1S 17408
#define SB_T_SIGNS 33792
#define SB_T_IQ4 34816
#define SB_T_VECTORS 34864
#define SB_GRIDS 33792
#define SB_TABLES 34992

static inline uint32_t rd16(const uint8_t *p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }
static inline uint32_t rd32(const uint8_t *p) { return rd16(p) | (rd16(p + 2) << 16); }

int32_t or_sb_size(int32_t type) {
  switch (type) {
    case 10: return 84;  case 12: return 144; case 16: return 66;  case 17: return 74;  case 18: return 98;
    case 19: return 50;  case 21: return 110; case 22: return 82;  case 23: return 136; case 29: return 56;
    default: return 0;
  }
}

/* sb_tables (types.ts:294-322): the grids as the codebooks hold them (IQ1_S's grid plus 1: codes 0, 1, 2), the signs
 * of 8 weights by a 7-bit index (the eighth makes the number of minuses even), IQ4_XS's values / magnitudes / minus
 * masks, and the small vectors */
int32_t or_sb_tables(uint8_t *area, const uint8_t *codebooks) {
  for (int i = 0; i < SB_GRIDS; i++) area[i] = (uint8_t)(codebooks[i] + (i >= SB_T_IQ1S ? 1 : 0));
  for (uint32_t i = 0; i < 128; i++) {
    uint32_t ones = 0;
    for (int j = 0; j < 7; j++) ones += (i >> j) & 1;
    const uint32_t held = i | ((ones & 1) << 7);
    for (int j = 0; j < 8; j++) area[SB_T_SIGNS + i * 8 + j] = ((held >> j) & 1) ? 255 : 0;
  }
  for (int i = 0; i < 16; i++) {
    const int8_t v = (int8_t)codebooks[SB_GRIDS + i];
    area[SB_T_IQ4 + i] = (uint8_t)v;
    area[SB_T_IQ4 + 16 + i] = (uint8_t)(v < 0 ? -v : v);
    area[SB_T_IQ4 + 32 + i] = v < 0 ? 255 : 0;
  }
  uint8_t *vec = area + SB_T_VECTORS;
  for (int j = 0; j < 16; j++) {
    vec[0 + j] = (uint8_t)(1u << (j & 7));
    vec[16 + j] = (uint8_t)(j >> 3);
    vec[32 + j] = 3;
    vec[48 + j] = 15;
    vec[80 + j] = 7;
    vec[96 + j] = 1;
  }
  for (int j = 0; j < 4; j++) {
    const int32_t p3 = 512 >> (j * 3), p4 = 4096 >> (j * 4);
    memcpy(vec + 64 + 4 * j, &p3, 4);
    memcpy(vec + 112 + 4 * j, &p4, 4);
  }
  return SB_TABLES;
}

static inline int sb_minus(const uint8_t *tab, uint32_t idx7, int j) { return tab[SB_T_SIGNS + (idx7 & 127) * 8 + j] != 0; }

/* unit u (16 weights) of the block at p: W[16] (IQ1: 8 g + 1, or 8 g - 1 where the shift is down), S, m */
static void sb_unit(int type, const uint8_t *p, int u, const uint8_t *tab, int32_t *W, int32_t *S, int32_t *m) {
  const int g = u >> 1;
  *m = 0;
  switch (type) {
    case 10: {  /* Q2_K: bits 2 s, 2 s + 1 of byte b of a half's 32 are weight 32 s + b of the half */
      const int half = u >> 3, s = (u & 7) >> 1;
      const uint8_t *q = p + 16 + 32 * half + 16 * (u & 1);
      for (int j = 0; j < 16; j++) W[j] = (q[j] >> (2 * s)) & 3;
      *S = p[u] & 15;
      *m = p[u] >> 4;
      return;
    }
    case 12: {  /* Q4_K: of every 32 bytes the low halves are 32 weights, the high halves the next 32 */
      const uint8_t *q = p + 16 + 32 * (g >> 1) + 16 * (u & 1), *sc = p + 4;
      for (int j = 0; j < 16; j++) W[j] = (g & 1) ? q[j] >> 4 : q[j] & 15;
      *S = g < 4 ? sc[g] & 63 : (sc[g + 4] & 15) | ((sc[g - 4] >> 6) << 4);
      *m = g < 4 ? sc[g + 4] & 63 : (sc[g + 4] >> 4) | ((sc[g] >> 6) << 4);
      return;
    }
    case 23: {  /* IQ4_XS: of a group's 16 bytes the low halves are its first 16 weights */
      const uint8_t *q = p + 8 + 16 * g;
      for (int j = 0; j < 16; j++) W[j] = (int8_t)tab[SB_T_IQ4 + ((u & 1) ? q[j] >> 4 : q[j] & 15)];
      *S = (int32_t)(((p[4 + (g >> 1)] >> (4 * (g & 1))) & 15) | (((rd16(p + 2) >> (2 * g)) & 3) << 4)) - 32;
      return;
    }
    case 16: {  /* IQ2_XXS: 8 bytes a group: four grid indices, then a word of four 7-bit sign indices and s */
      const uint8_t *q = p + 2 + 8 * g;
      const uint32_t aux = rd32(q + 4), sh = 14 * (u & 1);
      for (int e = 0; e < 2; e++) {
        const uint8_t *entry = tab + q[2 * (u & 1) + e] * 8;
        const uint32_t sg = aux >> (sh + 7 * e);
        for (int j = 0; j < 8; j++) W[8 * e + j] = sb_minus(tab, sg, j) ? -(int32_t)entry[j] : entry[j];
      }
      *S = (int32_t)(2 * (aux >> 28) + 1);
      return;
    }
    case 17: {  /* IQ2_XS: a 16-bit word for 8 weights: 9 bits of index, 7 of signs */
      for (int e = 0; e < 2; e++) {
        const uint32_t q = rd16(p + 2 + 4 * u + 2 * e);
        const uint8_t *entry = tab + SB_T_IQ2XS + (q & 511) * 8;
        for (int j = 0; j < 8; j++) W[8 * e + j] = sb_minus(tab, q >> 9, j) ? -(int32_t)entry[j] : entry[j];
      }
      *S = (int32_t)(2 * ((p[66 + g] >> (4 * (u & 1))) & 15) + 1);
      return;
    }
    case 22: {  /* IQ2_S: 10-bit indices (qs, and 2 bits of qh), a byte of signs for each 8 */
      const uint32_t hi = p[66 + g] >> (4 * (u & 1)), signs = rd16(p + 34 + 2 * u);
      const uint32_t idx[2] = {p[2 + 2 * u] | ((hi & 3) << 8), p[3 + 2 * u] | ((hi & 12) << 6)};
      for (int e = 0; e < 2; e++)
        for (int j = 0; j < 8; j++) {
          const int32_t v = tab[SB_T_IQ2S + idx[e] * 8 + j];
          W[8 * e + j] = ((signs >> (8 * e + j)) & 1) ? -v : v;
        }
      *S = (int32_t)(2 * ((p[74 + g] >> (4 * (u & 1))) & 15) + 1);
      return;
    }
    case 18: {  /* IQ3_XXS: a byte an index of 4 weights; a word a group: its signs and s */
      const uint32_t aux = rd32(p + 66 + 4 * g), sh = 14 * (u & 1);
      for (int i = 0; i < 4; i++) {
        const uint8_t *entry = tab + SB_T_IQ3XXS + p[2 + 4 * u + i] * 4;
        for (int j = 0; j < 4; j++) {
          const int w = 4 * i + j;
          W[w] = sb_minus(tab, aux >> (sh + 7 * (w >> 3)), w & 7) ? -(int32_t)entry[j] : entry[j];
        }
      }
      *S = (int32_t)(2 * (aux >> 28) + 1);
      return;
    }
    case 21: {  /* IQ3_S: 9-bit indices (qs and a bit of qh each), 16 bits of signs, 4-bit scales a 32 */
      const uint32_t hi = p[66 + g] >> (4 * (u & 1)), signs = rd16(p + 74 + 2 * u);
      for (int i = 0; i < 4; i++) {
        const uint32_t idx = p[2 + 4 * u + i] | (((hi >> i) & 1) << 8);
        for (int j = 0; j < 4; j++) {
          const int w = 4 * i + j;
          const int32_t v = tab[SB_T_IQ3S + idx * 4 + j];
          W[w] = ((signs >> w) & 1) ? -v : v;
        }
      }
      *S = (int32_t)(2 * ((p[106 + (u >> 2)] >> (4 * ((u >> 1) & 1))) & 15) + 1);
      return;
    }
    case 19: {  /* IQ1_S: 11-bit indices (qs and 3 bits of the group's word), the word's top bit the shift's sign */
      const uint32_t qh = rd16(p + 34 + 2 * g), hi = qh >> (6 * (u & 1)), down = qh >> 15;
      const uint32_t idx[2] = {p[2 + 2 * u] | ((hi & 7) << 8), p[3 + 2 * u] | ((hi & 56) << 5)};
      for (int e = 0; e < 2; e++)
        for (int j = 0; j < 8; j++) {
          const int32_t code = tab[SB_T_IQ1S + idx[e] * 8 + j];  /* 0, 1, 2 */
          W[8 * e + j] = 8 * (code - 1) + (down ? -1 : 1);
        }
      *S = (int32_t)(2 * ((qh >> 12) & 7) + 1);
      return;
    }
    case 29: {  /* IQ1_M: a byte of qh a unit: 3 bits of each index and the shifts' signs (bits 3 and 7) */
      const uint32_t hq = p[32 + u];
      const uint32_t idx[2] = {p[2 * u] | ((hq & 7) << 8), p[2 * u + 1] | ((hq & 0x70) << 4)};
      const uint32_t down[2] = {(hq >> 3) & 1, hq >> 7};
      for (int e = 0; e < 2; e++)
        for (int j = 0; j < 8; j++) {
          const int32_t code = tab[SB_T_IQ1S + idx[e] * 8 + j];
          W[8 * e + j] = 8 * (code - 1) + (down[e] ? -1 : 1);
        }
      *S = (int32_t)(2 * ((rd16(p + 48 + 2 * (u >> 2)) >> (3 * (u & 3))) & 7) + 1);
      return;
    }
  }
}

/* IQ1_M's d: the top four bits of its four scale words, the first word's the lowest (types.ts:283-287) */
static float sb_whole(const uint8_t *p) {
  const uint32_t w0 = rd16(p + 48), w1 = rd16(p + 50), w2 = rd16(p + 52), w3 = rd16(p + 54);
  return or_half((uint16_t)((w0 >> 12) | ((w1 >> 8) & 0xf0) | ((w2 >> 4) & 0xf00) | (w3 & 0xf000)));
}
static float sb_F(int type, const uint8_t *p) {
  switch (type) {
    case 16: case 17: case 22: case 19: return or_half((uint16_t)rd16(p)) * 0.125f;
    case 18: return or_half((uint16_t)rd16(p)) * 0.25f;
    case 29: return sb_whole(p) * 0.125f;
    case 10: return or_half((uint16_t)rd16(p + 80));
    default: return or_half((uint16_t)rd16(p));
  }
}
static float sb_Fm(int type, const uint8_t *p) {
  return type == 10 ? or_half((uint16_t)rd16(p + 82)) : or_half((uint16_t)rd16(p + 2));
}

/* sums_x (token.ts:158-172): after the n / 32 scales at xs, the int16 sums of each 16 of xq, then of each 8 */
void or_sums_x(float *xs, const int8_t *xq, int32_t n) {
  int16_t *s16 = (int16_t *)(xs + n / 32), *s8 = s16 + n / 16;
  for (int32_t i = 0; i < n / 16; i++) {
    int32_t s = 0;
    for (int j = 0; j < 16; j++) s += xq[16 * i + j];
    s16[i] = (int16_t)s;
  }
  for (int32_t i = 0; i < n / 8; i++) {
    int32_t s = 0;
    for (int j = 0; j < 8; j++) s += xq[8 * i + j];
    s8[i] = (int16_t)s;
  }
}

/* matmul_sb (token.ts:130-141) on one token: out[i] for rows r0..r1 of n weights in blocks of type */
void or_matmul_sb(float *out, const int8_t *xq, const float *xs, const uint8_t *w, const uint8_t *tab, int32_t n,
                  int32_t r0, int32_t r1, int32_t type) {
  const int size = or_sb_size(type), blocks = n / 256, kq = type == 10 || type == 12;
  for (int32_t i = r0; i < r1; i++) {
    const uint8_t *row = w + (size_t)i * blocks * size;
    float facc[4] = {0, 0, 0, 0};
    for (int b = 0; b < blocks; b++) {
      const uint8_t *p = row + (size_t)b * size;
      const int8_t *x = xq + 256 * b;
      int32_t G[8] = {0}, M[8] = {0};
      for (int u = 0; u < 16; u++) {
        int32_t W[16], S, m;
        sb_unit(type, p, u, tab, W, &S, &m);
        int32_t d = 0, s16 = 0;
        for (int j = 0; j < 16; j++) {
          d += W[j] * x[16 * u + j];
          s16 += x[16 * u + j];
        }
        G[u >> 1] += S * d;
        M[u >> 1] += m * s16;
      }
      const float *s = xs + 8 * b, F = sb_F(type, p);
      for (int j = 0; j < 4; j++) {
        float part = ((float)G[j] * s[j] + (float)G[j + 4] * s[j + 4]) * F;
        if (kq) part = part - ((float)M[j] * s[j] + (float)M[j + 4] * s[j + 4]) * sb_Fm(type, p);
        facc[j] += part;
      }
    }
    out[i] = ((facc[0] + facc[1]) + facc[2]) + facc[3];
  }
}

/* sb_row (row.ts): a row of n weights as float32, each as the reference's reader makes it: the unit's float scale
 * (row.ts:11-19) times W (IQ1: the grid's value plus or minus 1/8), less the block's Fm m for the K types */
void or_sb_row(float *out, const uint8_t *w, const uint8_t *tab, int32_t n, int32_t type) {
  const int size = or_sb_size(type);
  for (int b = 0; b < n / 256; b++) {
    const uint8_t *p = w + (size_t)b * size;
    for (int u = 0; u < 16; u++) {
      int32_t W[16], S, m;
      sb_unit(type, p, u, tab, W, &S, &m);
      const float s = (float)(S >> 1);
      float scale;
      switch (type) {
        case 16: case 17: case 22: scale = or_half((uint16_t)rd16(p)) * (0.5f + s) * 0.25f; break;
        case 18: scale = or_half((uint16_t)rd16(p)) * (0.5f + s) * 0.5f; break;
        case 29: scale = sb_whole(p) * (float)S; break;
        case 10: scale = or_half((uint16_t)rd16(p + 80)) * (float)S; break;
        default: scale = or_half((uint16_t)rd16(p)) * (float)S;
      }
      for (int j = 0; j < 16; j++) {
        float v;
        if (type == 19 || type == 29) {  /* (8 g +- 1) / 8 = g +- 1/8, as the reader adds them */
          const int32_t shift = ((W[j] % 8) + 8) % 8 == 1 ? 1 : -1;  /* 8 g + 1 is 1 mod 8, 8 g - 1 is 7 */
          v = (float)((W[j] - shift) / 8) + (shift < 0 ? -0.125f : 0.125f);
        } else {
          v = (float)W[j];
        }
        float o = scale * v;
        if (type == 10 || type == 12) o = o - sb_Fm(type, p) * (float)m;
        out[256 * b + 16 * u + j] = o;
      }
    }
  }
}
