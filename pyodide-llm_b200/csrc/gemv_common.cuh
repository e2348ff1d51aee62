// gemv_common.cuh: what the two decode-product kernels share (gemv.cu's register-streaming one and gemv_tma.cu's
// bulk-copy pipeline): their arguments, the weight formats, and the activations' prologue (the caller's quantized
// activations, or RMSNorm and quantize_x made from float32).
#pragma once
#include "pllm_common.cuh"
#include "pllm_device.cuh"

namespace gemvk {

enum Fmt { F_Q8 = 0, F_Q6 = 1, F_T2 = 2, F_B1 = 3 };
enum Pro { PRO_Q = 0, PRO_RMS = 1, PRO_QUANT = 2 };
enum Epi { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2 };

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
// The activations of MT tokens into shared memory by THREADS threads (the whole CTA, or the consumer warps of a
// warp-specialized one: SYNC is their barrier).
struct CtaSync {
  __device__ __forceinline__ void operator()() const { __syncthreads(); }
};
template <int FMT, int MT, int PRO, class SYNC = CtaSync>
__device__ __forceinline__ void load_activations(const GemvArgs& a, int8_t* sq, float* ss, int32_t* sm) {
  const SYNC sync;
  const int K = a.K, ng = K / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (PRO == PRO_Q) {
    for (int t = 0; t < MT; t++) {
      if (t >= a.count) break;
      const int4* src = reinterpret_cast<const int4*>(a.xq + t * a.xq_stride);
      int4* dst = reinterpret_cast<int4*>(sq + (size_t)t * K);
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
    __shared__ float red[WARPS];
    for (int t = 0; t < MT; t++) {
      if (t >= a.count) break;
      const float* x = a.x + t * a.x_stride;
      float rs = 1.0f;
      if (PRO == PRO_RMS) {
        float s = 0.0f;
        for (int i = threadIdx.x; i < K; i += THREADS) s = fmaf(x[i], x[i], s);
        s = warp_sum(s);
        if (lane == 0) red[warp] = s;
        sync();
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < WARPS; w++) tot += red[w];
        rs = 1.0f / sqrtf(tot / (float)K + a.eps);
        sync();
      }
      for (int g = warp; g < ng; g += WARPS) {
        float v = x[g * 32 + lane];
        if (PRO == PRO_RMS) v = a.norm[g * 32 + lane] * (rs * v);
        float scale;
        const int8_t q = quantize_group_warp(v, lane, a.bias, &scale);
        sq[(size_t)t * K + g * 32 + lane] = (int8_t)(q - (int8_t)a.bias);  // signed, as the products take it
        if (lane == 0) ss[t * ng + g] = scale;
      }
    }
  }
  for (int t = a.count; t < MT; t++) {  // tokens past count: zeros (their outputs are not written)
    for (int i = threadIdx.x; i < K; i += THREADS) sq[(size_t)t * K + i] = 0;
    for (int i = threadIdx.x; i < ng; i += THREADS) ss[t * ng + i] = 0.0f;
  }
}


// gemv_tma.cu: the bulk-copy pipeline for int8 at 1 or 2 tokens; false where it does not apply
bool gemv_tma(const GemvArgs& a, int fmt, int pro, int epi, bool pdl);
extern int g_gemv_mode;
extern int g_tma_budget;

}  // namespace gemvk
