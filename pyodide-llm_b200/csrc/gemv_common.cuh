// gemv_common.cuh: what the two decode-product kernels share (gemv.cu's register-streaming one and gemv_tma.cu's
// bulk-copy pipeline): their arguments, the weight formats, and the activations' prologue (the caller's quantized
// activations, or RMSNorm and quantize_x made from float32).
#pragma once
#include "pllm_common.cuh"
#include "pllm_device.cuh"

namespace gemvk {

enum Fmt { F_Q8 = 0, F_Q6 = 1, F_T2 = 2, F_B1 = 3 };
enum Pro { PRO_Q = 0, PRO_RMS = 1, PRO_QUANT = 2, PRO_RMS_SUM = 3 };
enum Epi { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2, EPI_SEND = 3 };

// A tensor-parallel rank's side of one reduction over NVLink (exchange.cu): the row-parallel product (wo, w2: each
// rank's share of K) sends its rows to every rank's receive region (EPI_SEND), each value in one 8-byte store with
// the reduction's mark beside it; the next product's prologue (PRO_RMS_SUM) reads every rank's slots until their marks
// are this reduction's, makes x + the ranks' partials (in rank order, so every rank gets the same bits), writes that
// to x_out (CTA 0) and takes RMSNorm and quantize_x of it. No fence and no counter: a slot is whole or not there.
constexpr int TP_MAX = 8;
struct Xchg {
  unsigned long long* dst[TP_MAX];  // EPI_SEND: rank p's receive slots of this rank, this parity ([dim] x 8 bytes)
  const unsigned long long* src;    // PRO_RMS_SUM: this rank's receive slots of this parity, [world][dim]
  const unsigned* step;             // this rank's step counter (pllm_tp_step: 1 in the first step)
  float* x_out;                     // PRO_RMS_SUM: x + the partials
  int* status;                      // the device status word (a wait that gives up writes PLLM_ETIMEOUT there)
  int world;
  unsigned per_step, k;             // the reduction's mark: (step - 1) per_step + k + 1
};

__device__ __forceinline__ unsigned xchg_mark(const Xchg& xg) { return (*xg.step - 1u) * xg.per_step + xg.k + 1u; }
__device__ __forceinline__ unsigned long long ld_slot(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_slot(unsigned long long* p, float v, unsigned mark) {
  const unsigned long long s = ((unsigned long long)mark << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(s) : "memory");
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
constexpr unsigned long long XCHG_WAIT_NS = 2000000000ull;  // the wait for the other ranks' partials: 2 s at most

// rank p's four slots from float4 number i: read until all four carry the mark (past 2 s: PLLM_ETIMEOUT recorded,
// and the values as they are)
__device__ __forceinline__ float4 wait_slots(const unsigned long long* s, unsigned mark, int* status) {
  unsigned long long a = ld_slot(s), b = ld_slot(s + 1), c = ld_slot(s + 2), d = ld_slot(s + 3);
  if ((unsigned)(a >> 32) != mark || (unsigned)(b >> 32) != mark || (unsigned)(c >> 32) != mark ||
      (unsigned)(d >> 32) != mark) {
    const unsigned long long t0 = global_ns();
    for (;;) {
      a = ld_slot(s);
      b = ld_slot(s + 1);
      c = ld_slot(s + 2);
      d = ld_slot(s + 3);
      if ((unsigned)(a >> 32) == mark && (unsigned)(b >> 32) == mark && (unsigned)(c >> 32) == mark &&
          (unsigned)(d >> 32) == mark)
        break;
      if (global_ns() - t0 > XCHG_WAIT_NS) {
        atomicExch(status, PLLM_ETIMEOUT);
        break;
      }
    }
  }
  return make_float4(__uint_as_float((unsigned)a), __uint_as_float((unsigned)b), __uint_as_float((unsigned)c),
                     __uint_as_float((unsigned)d));
}

struct GemvArgs {
  float* out;              // out + t * out_stride (floats) + row
  long long out_stride;
  const uint8_t* xq;       // PRO_Q: quantized activations, token t at xq + t * xq_stride (bytes)
  const float* xs;         // PRO_Q: scales (and, for ternary / binary, the interleave's minus-sums after them)
  long long xq_stride, xs_stride;  // bytes
  const float* x;          // PRO_RMS / PRO_QUANT: float32 activations, token t at x + t * x_stride (floats)
  long long x_stride;
  const float* norm;       // PRO_RMS: the RMSNorm weight
  float eps;
  int bias;                // 0: signed int8 activations; 64: biased (relaxed) activations
  const uint8_t* wq;
  const void* ws;          // float32 (int8, int6) or float16 bits (ternary, binary) scales
  int K, r0, r1, count;
  long long pair;          // EPI_SWIGLU: the row of the gate's partner (row + pair)
};

template <int FMT> struct FmtInfo;
template <> struct FmtInfo<F_Q8> { static constexpr int GK = 32, UB = 32; };
template <> struct FmtInfo<F_Q6> { static constexpr int GK = 32, UB = 24; };
template <> struct FmtInfo<F_T2> { static constexpr int GK = 128, UB = 32; };
template <> struct FmtInfo<F_B1> { static constexpr int GK = 128, UB = 16; };

constexpr int THREADS = 256, WARPS = THREADS / 32, UNROLL = 4;

// shared memory: MT tokens of K signed int8 activations, their K / 32 scales, and (ternary / binary) the K / 32
// minus-sums of their groups of 32
template <int FMT>
__host__ __device__ constexpr size_t smem_bytes(int K, int MT) {
  return (size_t)MT * K + (size_t)MT * (K / 32) * 4 + (FMT >= F_T2 ? (size_t)MT * (K / 32) * 4 : 0);
}

// The activations of MT tokens into shared memory, signed. PRO_Q copies the caller's (taking the bias of relaxed
// activations off); PRO_RMS / PRO_QUANT make them here from float32: RMSNorm (optional), then quantize_x's steps.
// One group of 32 held by a pair of threads (h: the lower or upper 16 values, as float4 x 4): RMSNorm's scaling
// (PRO_RMS: w * (rs * x), activations.ts:19), quantize.ts:8-19's largest |x| a SIMD lane (value j in lane j % 4;
// a NaN makes its lane NaN) and the lanes compared in order, then quantize_x's steps; the 16 signed bytes into sq and
// the scale into ss. g past the groups: the pair computes on zeros and stores nothing (every thread of the warp
// takes the shuffle).
template <int PRO>
__device__ __forceinline__ void quantize_pair(const GemvArgs& a, const float4* xv, const float4* wv, float rs, int g,
                                              int h, int t, int8_t* sq, float* ss, size_t sq_stride) {
  const int K = a.K, ng = K / 32;
  float u[16];
#pragma unroll
  for (int k = 0; k < 4; k++) {
    u[4 * k] = xv[k].x;
    u[4 * k + 1] = xv[k].y;
    u[4 * k + 2] = xv[k].z;
    u[4 * k + 3] = xv[k].w;
    if (PRO == PRO_RMS) {
      u[4 * k] = wv[k].x * (rs * u[4 * k]);
      u[4 * k + 1] = wv[k].y * (rs * u[4 * k + 1]);
      u[4 * k + 2] = wv[k].z * (rs * u[4 * k + 2]);
      u[4 * k + 3] = wv[k].w * (rs * u[4 * k + 3]);
    }
  }
  float m[4];
#pragma unroll
  for (int l = 0; l < 4; l++)
    m[l] = wasm_max(wasm_max(fabsf(u[l]), fabsf(u[l + 4])), wasm_max(fabsf(u[l + 8]), fabsf(u[l + 12])));
#pragma unroll
  for (int l = 0; l < 4; l++) m[l] = wasm_max(m[l], __shfl_xor_sync(0xffffffffu, m[l], 1));
  float amax = m[0];
  if (m[1] > amax) amax = m[1];
  if (m[2] > amax) amax = m[2];
  if (m[3] > amax) amax = m[3];
  const float scale = __fdiv_rn(amax, a.bias == 0 ? 127.0f : 63.0f);
  const float inv = scale > 0.0f ? __fdiv_rn(1.0f, scale) : 0.0f;
  if (g >= ng) return;
  uint32_t packed[4];
#pragma unroll
  for (int k = 0; k < 4; k++) {
    uint32_t word = 0;
#pragma unroll
    for (int b = 0; b < 4; b++) {
      const int8_t q = (int8_t)(quantize_one(u[4 * k + b], inv, a.bias) - (int8_t)a.bias);  // signed
      word |= (uint32_t)(uint8_t)q << (8 * b);
    }
    packed[k] = word;
  }
  *reinterpret_cast<int4*>(sq + (size_t)t * sq_stride + 32 * g + 16 * h) =
      make_int4((int)packed[0], (int)packed[1], (int)packed[2], (int)packed[3]);
  if (h == 0) ss[t * ng + g] = scale;
}

// The activations of MT tokens into shared memory by THREADS threads (the whole CTA, or the consumer warps of a
// warp-specialized one: SYNC is their barrier).
struct CtaSync {
  __device__ __forceinline__ void operator()() const { __syncthreads(); }
};
// out += v where a launch adds to each output once: red.global.add.f32, the same rounded sum as a load and a store
// without the consumer warp waiting on the load (measured on the Qwen3-8B decode step: 2.009 -> 1.965 ms); the add
// flushes a subnormal sum to zero
__device__ __forceinline__ void add_once(float* o, float v) { atomicAdd(o, v); }

// x's float4 number i of token t: PRO_RMS_SUM adds the ranks' partials in rank order (waiting for their slots) and
// CTA 0 stores the sum to x_out
template <int PRO>
__device__ __forceinline__ float4 x_vec(const GemvArgs& a, const Xchg* xg, int t, int i) {
  // from L2 (.cg): x was written by the kernel ahead of this one (its CTAs on other SMs)
  float4 v = __ldcg(reinterpret_cast<const float4*>(a.x + t * a.x_stride) + i);
  if constexpr (PRO == PRO_RMS_SUM) {
    const unsigned mark = xchg_mark(*xg);
    for (int p = 0; p < xg->world; p++) {
      const float4 r = wait_slots(xg->src + (size_t)p * a.K + 4 * (size_t)i, mark, xg->status);
      v.x += r.x;
      v.y += r.y;
      v.z += r.z;
      v.w += r.w;
    }
    if (blockIdx.x == 0) reinterpret_cast<float4*>(xg->x_out)[i] = v;
  }
  return v;
}

// sq_stride: bytes from a token's activations to the next's (0: K; the batched tensor-core product pads its rows)
template <int FMT, int MT, int PRO, class SYNC = CtaSync>
__device__ __forceinline__ void load_activations(const GemvArgs& a, int8_t* sq, float* ss, int32_t* sm,
                                                 const Xchg* xg = nullptr, size_t sq_stride = 0) {
  const SYNC sync;
  const int K = a.K, ng = K / 32;
  const size_t SQ = sq_stride ? sq_stride : (size_t)K;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (PRO == PRO_Q) {
    for (int t = 0; t < MT; t++) {
      if (t >= a.count) break;
      const int4* src = reinterpret_cast<const int4*>(a.xq + t * a.xq_stride);
      int4* dst = reinterpret_cast<int4*>(sq + (size_t)t * SQ);
      const int bias4 = a.bias ? 0x40404040 : 0;
      for (int i = threadIdx.x; i < K / 16; i += THREADS) {
        int4 v = src[i];
        if (bias4) {  // q - 64 byte by byte: the bytes are 0..127, so no borrow crosses a byte
          v.x = (int)__vsub4((unsigned)v.x, (unsigned)bias4);
          v.y = (int)__vsub4((unsigned)v.y, (unsigned)bias4);
          v.z = (int)__vsub4((unsigned)v.z, (unsigned)bias4);
          v.w = (int)__vsub4((unsigned)v.w, (unsigned)bias4);
        }
        dst[i] = v;
      }
      const float* xs = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(a.xs) + t * a.xs_stride);
      for (int i = threadIdx.x; i < ng; i += THREADS) ss[t * ng + i] = xs[i];
      if (FMT >= F_T2) {
        const int32_t* sums = reinterpret_cast<const int32_t*>(xs + ng);
        for (int i = threadIdx.x; i < ng; i += THREADS) sm[t * ng + i] = sums[i];
      }
    }
  } else {
    // A pair of threads a group of 32 (the lower thread its values 0..15, the upper 16..31), the groups taken 128 at a
    // time: every float32 load of a token (and of the norm's weights) issued before any is used, held in registers.
    __shared__ float red[WARPS];
    constexpr int RMAX = 3;  // rounds of 128 groups held in registers (K <= 12288); past them read again
    const int pair = threadIdx.x >> 1, h = threadIdx.x & 1;
    const int rounds = (ng + 127) / 128;
    constexpr bool NORM = PRO == PRO_RMS || PRO == PRO_RMS_SUM;
    for (int t = 0; t < MT; t++) {
      if (t >= a.count) break;
      const float4* n4 = reinterpret_cast<const float4*>(a.norm);
      float4 v[RMAX][4], w[RMAX][4];
#pragma unroll
      for (int r = 0; r < RMAX; r++) {
        const int g = pair + 128 * r;
        const bool in = r < rounds && g < ng;
#pragma unroll
        for (int k = 0; k < 4; k++) {
          v[r][k] = in ? x_vec<PRO>(a, xg, t, (32 * g + 16 * h) / 4 + k) : make_float4(0.f, 0.f, 0.f, 0.f);
          w[r][k] = (NORM && in) ? __ldg(n4 + (32 * g + 16 * h) / 4 + k) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      float rs = 1.0f;
      if (NORM) {
        float s = 0.0f;
#pragma unroll
        for (int r = 0; r < RMAX; r++) {
#pragma unroll
            for (int k = 0; k < 4; k++)
              s = fmaf(v[r][k].x, v[r][k].x, fmaf(v[r][k].y, v[r][k].y, fmaf(v[r][k].z, v[r][k].z, fmaf(v[r][k].w, v[r][k].w, s))));
        }
        for (int r = RMAX; r < rounds; r++) {
          const int g = pair + 128 * r;
          if (g < ng)
            for (int k = 0; k < 4; k++) {
              const float4 u = x_vec<PRO>(a, xg, t, (32 * g + 16 * h) / 4 + k);
              s = fmaf(u.x, u.x, fmaf(u.y, u.y, fmaf(u.z, u.z, fmaf(u.w, u.w, s))));
            }
        }
        s = warp_sum(s);
        if (lane == 0) red[warp] = s;
        sync();
        float tot = 0.0f;
#pragma unroll
        for (int i = 0; i < WARPS; i++) tot += red[i];
        rs = 1.0f / sqrtf(tot / (float)K + a.eps);
        sync();
      }
      constexpr int QP = NORM ? PRO_RMS : PRO;
#pragma unroll
      for (int r = 0; r < RMAX; r++) {
        if (r < rounds) quantize_pair<QP>(a, v[r], w[r], rs, pair + 128 * r, h, t, sq, ss, SQ);
      }
      for (int r = RMAX; r < rounds; r++) {
        const int g = pair + 128 * r;
        float4 xv[4], wv[4];
        for (int k = 0; k < 4; k++) {
          xv[k] = g < ng ? x_vec<PRO>(a, xg, t, (32 * g + 16 * h) / 4 + k) : make_float4(0.f, 0.f, 0.f, 0.f);
          wv[k] = (NORM && g < ng) ? __ldg(n4 + (32 * g + 16 * h) / 4 + k) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        quantize_pair<QP>(a, xv, wv, rs, g, h, t, sq, ss, SQ);
      }
    }
  }
  for (int t = a.count; t < MT; t++) {  // tokens past count: zeros (their outputs are not written)
    for (int i = threadIdx.x; i < K; i += THREADS) sq[(size_t)t * SQ + i] = 0;
    for (int i = threadIdx.x; i < ng; i += THREADS) ss[t * ng + i] = 0.0f;
  }
}


// gemv_tma.cu: the bulk-copy pipeline for int8 at 1 or 2 tokens; false where it does not apply (xg: the exchange of
// PRO_RMS_SUM / EPI_SEND, which only this kernel takes)
bool gemv_tma(const GemvArgs& a, int fmt, int pro, int epi, bool pdl, const Xchg* xg = nullptr);
// the device status word's address on the current device (looked up on the first call a device: make that before any
// stream capture; pllm_tp_open does)
int* status_word();
// the CTAs gemv_tma launches for rows r0..r1 (one an SM at most: the tiles of 8 rows are dealt among them)
int gemv_tma_grid(long long rows, int epi);
extern int g_gemv_mode;
extern int g_tma_budget;

}  // namespace gemvk
