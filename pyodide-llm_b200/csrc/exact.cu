// exact.cu: a decode step in the reference's own order of float32 operations, so that the device's logits are the
// reference kernels' to the bit (the default kernels sum in other orders and agree within rounding, which a random
// 36-layer net amplifies through quantize_x's rounding boundaries). Every float operation here is rounded alone
// (__f*_rn: nothing contracted into a fused multiply-add, as WASM SIMD has none) and runs in the order of:
//   pllm_exact_prepare        rmsnorm, activations.ts:8-20 (four lanes over the values, then ((l0+l1)+l2)+l3);
//                             swiglu, activations.ts:77-90; then quantize_x, quantize.ts:124-151
//   pllm_exact_product        matmul_q8, matmul.ts:77-104 (dot32's four integer lanes of a group each scaled into
//                             its float lane) or matmul_q8r, relaxed/int8.ts:17-50 (a group's exact integer into
//                             lane g % 4 for the groups of whole fours, then the rest one by one)
//   pllm_exact_qk_rope_cache  the q / k head norms (rmsnorm per head, attention.ts:140-143), rope, attention.ts:7-20,
//                             to_f16 of the key and value, halves.ts:35-67
//   pllm_exact_attention      attentionOf, attention.ts:87-211: scores in sums4's order, softmax with largest and
//                             vexp / fexp, the weighted values four positions at a time
// The exponential is the Cephes single-precision expf (S. L. Moshier, Cephes Math Library, expf.c), the published
// method the reference's table-free exp follows (kernels/kernel/math.ts:28-58), restated here; CUDA's expf is not
// used on this path. The work is spread over the GPU wherever the order allows (rows, heads, positions, dimensions);
// a chain of adds the order makes serial stays serial.
#include "pllm_common.cuh"
#include "pllm_device.cuh"
#include <float.h>
#include <algorithm>

namespace {

constexpr unsigned kFull = 0xffffffffu;

// ---- Cephes expf: x = k ln2 + r (ln2 in two parts), e^r by a degree-5 polynomial, times 2^k
constexpr float kLog2e = 1.44269504088896341f;
constexpr float kLn2Hi = 0.693359375f;
constexpr float kLn2Lo = -2.12194440e-4f;

__device__ __forceinline__ float cephes_poly(float x, float k) {
  const float r = __fsub_rn(__fsub_rn(x, __fmul_rn(k, kLn2Hi)), __fmul_rn(k, kLn2Lo));
  float p = 1.9875691500e-4f;
  p = __fadd_rn(__fmul_rn(p, r), 1.3981999507e-3f);
  p = __fadd_rn(__fmul_rn(p, r), 8.3334519073e-3f);
  p = __fadd_rn(__fmul_rn(p, r), 4.1665795894e-2f);
  p = __fadd_rn(__fmul_rn(p, r), 1.6666665459e-1f);
  p = __fadd_rn(__fmul_rn(p, r), 5.0000001201e-1f);
  return __fadd_rn(__fadd_rn(__fmul_rn(p, __fmul_rn(r, r)), r), 1.0f);
}

__device__ __forceinline__ float wasm_min(float a, float b) {
  return (a != a || b != b) ? __int_as_float(0x7fc00000) : fminf(a, b);
}

// math.ts's scalar exp (fexp): 0 below -87, the argument held at 88 above
__device__ __forceinline__ float ref_fexp(float x) {
  if (x < -87.0f) return 0.0f;
  if (x > 88.0f) x = 88.0f;
  const float k = rintf(__fmul_rn(x, kLog2e));
  return __fmul_rn(cephes_poly(x, k), __int_as_float((__float2int_rz(k) + 127) << 23));
}

// math.ts's four-lane exp (vexp): the argument clamped to [-87, 88] (a NaN stays NaN)
__device__ __forceinline__ float ref_vexp(float x) {
  x = wasm_min(wasm_max(x, -87.0f), 88.0f);
  const float k = rintf(__fmul_rn(x, kLog2e));
  return __fmul_rn(cephes_poly(x, k), __int_as_float((__float2int_rz(k) + 127) << 23));
}

// the four lanes' sum of squares of v[0..n) (lane l: the values 4 i + l in order), then the values past the fours:
// activations.ts:8-20's ss. Run by one thread per lane (lane < 4), the combine by lane 0 of the caller.
__device__ __forceinline__ float lane_squares(const float* v, int n, int lane) {
  float a = 0.0f;
  const int n4 = n & ~3;
#pragma unroll 8
  for (int j = lane; j < n4; j += 4) a = __fadd_rn(a, __fmul_rn(v[j], v[j]));
  return a;
}
__device__ __forceinline__ float norm_scale(float ss, int n, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
}

// ---- rmsnorm / swiglu / as-is, then quantize_x: one CTA over the whole vector (the sum of squares is one chain)
__global__ void __launch_bounds__(1024) exact_prepare_kernel(uint8_t* __restrict__ xq, float* __restrict__ xs,
                                                             float* __restrict__ out, const float* __restrict__ x,
                                                             const float* __restrict__ w, int n, float eps, int bias,
                                                             int mode) {
  extern __shared__ float y[];  // n floats
  __shared__ float part[4];
  __shared__ float scale;
  const int tid = threadIdx.x;
  if (mode == 2) {  // swiglu(h1 = x[0..n), h3 = x[n..2n)): (v / (1 + exp(-v))) h3
    for (int j = tid; j < n; j += blockDim.x) {
      const float v = x[j];
      y[j] = __fmul_rn(__fdiv_rn(v, __fadd_rn(1.0f, ref_fexp(-v))), x[n + j]);
    }
  } else {
    for (int j = tid; j < n; j += blockDim.x) y[j] = x[j];
  }
  __syncthreads();
  if (mode == 1) {
    if (tid < 4) part[tid] = lane_squares(y, n, tid);
    __syncthreads();
    if (tid == 0) {
      float ss = __fadd_rn(__fadd_rn(__fadd_rn(part[0], part[1]), part[2]), part[3]);
      for (int j = n & ~3; j < n; j++) ss = __fadd_rn(ss, __fmul_rn(y[j], y[j]));
      scale = norm_scale(ss, n, eps);
    }
    __syncthreads();
    const float s = scale;
    for (int j = tid; j < n; j += blockDim.x) y[j] = __fmul_rn(w[j], __fmul_rn(s, y[j]));
    __syncthreads();
  }
  if (out)
    for (int j = tid; j < n; j += blockDim.x) out[j] = y[j];
  const int lane = tid & 31, warp = tid >> 5, warps = blockDim.x >> 5;
  for (int g = warp; g < n / 32; g += warps) {
    float sc;
    const int8_t q = quantize_group_warp(y[g * 32 + lane], lane, bias, &sc);
    xq[g * 32 + lane] = (uint8_t)q;
    if (lane == 0) xs[g] = sc;
  }
}

// ---- the int8 product in the reference's order: a warp a row, the activations in shared memory.
// relaxed: lane L takes group p + L of each pass of 32, its exact dot(w, q - 64) times f32(ws xs) into float lane
// g % 4 (gathered by lanes 0..3 in group order), the four added in order, then the groups past the fours one by one.
// plain: lane L = 4 i + k takes dot32's integer lane k of group p + i of each pass of 8 (the bytes 2k, 2k+1, 2k+8,
// 2k+9 of each half of the group), times f32(ws xs) into float lane k; the four added in order.
template <bool RELAXED>
__global__ void __launch_bounds__(256) exact_product_kernel(float* out, const float* add,
                                                            const uint8_t* __restrict__ xq,
                                                            const float* __restrict__ xs,
                                                            const int8_t* __restrict__ wq,
                                                            const float* __restrict__ ws, int n, int rows) {
  extern __shared__ __align__(16) uint8_t sm[];
  uint8_t* sq = sm;
  float* sxs = reinterpret_cast<float*>(sm + n);
  const int ng = n / 32;
  for (int i = threadIdx.x; i < n / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(sq)[i] = reinterpret_cast<const uint4*>(xq)[i];
  for (int i = threadIdx.x; i < ng; i += blockDim.x) sxs[i] = xs[i];
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, c = lane & 3;
  for (int r = blockIdx.x * 8 + warp; r < rows; r += gridDim.x * 8) {
    const int8_t* row = wq + (size_t)r * n;
    const float* srow = ws + (size_t)r * ng;
    float acc = 0.0f, sum;
    if (RELAXED) {
      const int ng4 = ng & ~3;
      float term = 0.0f;
      for (int p = 0; p < ng; p += 32) {
        const int g = p + lane;
        term = 0.0f;
        if (g < ng) {
          const uint4 w0 = __ldg(reinterpret_cast<const uint4*>(row + (size_t)g * 32));
          const uint4 w1 = __ldg(reinterpret_cast<const uint4*>(row + (size_t)g * 32 + 16));
          const uint4 a0 = reinterpret_cast<const uint4*>(sq + g * 32)[0];
          const uint4 a1 = reinterpret_cast<const uint4*>(sq + g * 32)[1];
          int d = __dp4a((int)w0.x, (int)a0.x, 0);
          d = __dp4a((int)w0.y, (int)a0.y, d);
          d = __dp4a((int)w0.z, (int)a0.z, d);
          d = __dp4a((int)w0.w, (int)a0.w, d);
          d = __dp4a((int)w1.x, (int)a1.x, d);
          d = __dp4a((int)w1.y, (int)a1.y, d);
          d = __dp4a((int)w1.z, (int)a1.z, d);
          d = __dp4a((int)w1.w, (int)a1.w, d);
          const int one = 0x01010101;
          int sw = __dp4a((int)w0.x, one, 0);
          sw = __dp4a((int)w0.y, one, sw);
          sw = __dp4a((int)w0.z, one, sw);
          sw = __dp4a((int)w0.w, one, sw);
          sw = __dp4a((int)w1.x, one, sw);
          sw = __dp4a((int)w1.y, one, sw);
          sw = __dp4a((int)w1.z, one, sw);
          sw = __dp4a((int)w1.w, one, sw);
          const int G = d - 64 * sw;  // dot(w, q - 64): the stored activations are q + 64 in 0..127
          term = __fmul_rn(__int2float_rn(G), __fmul_rn(srow[g], sxs[g]));
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const int src = 4 * i + c;
          const float t = __shfl_sync(kFull, term, src);
          if (p + src < ng4) acc = __fadd_rn(acc, t);
        }
      }
      const float l1 = __shfl_sync(kFull, acc, 1), l2 = __shfl_sync(kFull, acc, 2), l3 = __shfl_sync(kFull, acc, 3);
      sum = __fadd_rn(__fadd_rn(__fadd_rn(acc, l1), l2), l3);
      for (int g = ng4; g < ng; g++) sum = __fadd_rn(sum, __shfl_sync(kFull, term, g & 31));  // the last pass's
    } else {
      const int h = c >> 1;
      const unsigned sel = (c & 1) ? 0x7632u : 0x5410u;
      for (int p = 0; p < ng; p += 8) {
        const int g = p + (lane >> 2);
        float term = 0.0f;
        if (g < ng) {
          const uint32_t* wr = reinterpret_cast<const uint32_t*>(row + (size_t)g * 32);
          const uint32_t* ar = reinterpret_cast<const uint32_t*>(sq + g * 32);
          int t = __dp4a((int)__byte_perm(__ldg(wr + h), __ldg(wr + 2 + h), sel),
                         (int)__byte_perm(ar[h], ar[2 + h], sel), 0);
          t = __dp4a((int)__byte_perm(__ldg(wr + 4 + h), __ldg(wr + 6 + h), sel),
                     (int)__byte_perm(ar[4 + h], ar[6 + h], sel), t);
          term = __fmul_rn(__int2float_rn(t), __fmul_rn(srow[g], sxs[g]));
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
          const float t = __shfl_sync(kFull, term, 4 * i + c);
          if (p + i < ng) acc = __fadd_rn(acc, t);
        }
      }
      const float l1 = __shfl_sync(kFull, acc, 1), l2 = __shfl_sync(kFull, acc, 2), l3 = __shfl_sync(kFull, acc, 3);
      sum = __fadd_rn(__fadd_rn(__fadd_rn(acc, l1), l2), l3);
    }
    if (lane == 0) out[r] = add ? __fadd_rn(add[r], sum) : sum;
  }
}

// ---- the q / k head norms, rope and the cache write: a warp a head (q heads, then k heads, then v heads)
__global__ void __launch_bounds__(32) exact_qk_rope_cache_kernel(float* qkv, const float* __restrict__ qn,
                                                                 const float* __restrict__ kn,
                                                                 const float* __restrict__ cos_t,
                                                                 const float* __restrict__ sin_t,
                                                                 const int* __restrict__ pos_dev, int pos_host,
                                                                 uint8_t* kc, uint8_t* vc, int nh, int nkv, int hs,
                                                                 float eps, int half, int* bad) {
  __shared__ float hv[512];
  const int hb = blockIdx.x, lane = threadIdx.x;
  const int pos = pos_dev ? *pos_dev : pos_host;
  float* v = qkv + (size_t)hb * hs;
  const int kind = hb < nh ? 0 : (hb < nh + nkv ? 1 : 2);
  for (int j = lane; j < hs; j += 32) hv[j] = v[j];
  __syncwarp();
  if (kind < 2) {
    const float* w = kind == 0 ? qn : kn;
    if (w) {
      const float a = lane < 4 ? lane_squares(hv, hs, lane) : 0.0f;
      const float l1 = __shfl_sync(kFull, a, 1), l2 = __shfl_sync(kFull, a, 2), l3 = __shfl_sync(kFull, a, 3);
      float s = 0.0f;
      if (lane == 0) {
        float ss = __fadd_rn(__fadd_rn(__fadd_rn(a, l1), l2), l3);
        for (int j = hs & ~3; j < hs; j++) ss = __fadd_rn(ss, __fmul_rn(hv[j], hv[j]));
        s = norm_scale(ss, hs, eps);
      }
      s = __shfl_sync(kFull, s, 0);
      for (int j = lane; j < hs; j += 32) hv[j] = __fmul_rn(w[j], __fmul_rn(s, hv[j]));
      __syncwarp();
    }
    const float* cr = cos_t + (size_t)pos * (hs / 2);
    const float* ci = sin_t + (size_t)pos * (hs / 2);
    for (int i = 2 * lane; i < hs; i += 64) {
      const float cc = cr[i >> 1], ss = ci[i >> 1], v0 = hv[i], v1 = hv[i + 1];
      hv[i] = __fsub_rn(__fmul_rn(v0, cc), __fmul_rn(v1, ss));
      hv[i + 1] = __fadd_rn(__fmul_rn(v0, ss), __fmul_rn(v1, cc));
    }
    __syncwarp();
  }
  if (kind == 0) {
    for (int j = lane; j < hs; j += 32) v[j] = hv[j];
    return;
  }
  const int kh = hb - nh - (kind == 2 ? nkv : 0);
  const size_t at = (size_t)pos * nkv * hs + (size_t)kh * hs;
  uint8_t* cache = kind == 1 ? kc : vc;
  int nb = 0;
  for (int j = lane; j < hs; j += 32) {
    if (kind == 1) v[j] = hv[j];
    if (half)
      reinterpret_cast<uint16_t*>(cache)[at + j] = float_to_half_bits(hv[j], &nb);
    else
      reinterpret_cast<float*>(cache)[at + j] = hv[j];
  }
  if (nb && bad) atomicAdd(bad, nb);
}

__device__ __forceinline__ float cache_at(const uint8_t* p, size_t i, int half) {
  return half ? half_bits_to_float(reinterpret_cast<const uint16_t*>(p)[i]) : reinterpret_cast<const float*>(p)[i];
}

// ---- attention, part 1: the scaled scores, a thread a position (all heads of its kv head), att[h][count]
__global__ void __launch_bounds__(128) exact_scores_kernel(float* __restrict__ att, const float* __restrict__ q,
                                                           const uint8_t* __restrict__ kc,
                                                           const int* __restrict__ pos_dev, int pos_host, int nh,
                                                           int nkv, int hs, int half) {
  extern __shared__ float qs[];  // the kv head's q heads
  const int count = (pos_dev ? *pos_dev : pos_host) + 1;
  const int kvh = blockIdx.y, mul = nh / nkv;
  for (int i = threadIdx.x; i < mul * hs; i += blockDim.x) qs[i] = q[(size_t)kvh * mul * hs + i];
  __syncthreads();
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= count) return;
  const float isq = __fdiv_rn(1.0f, __fsqrt_rn((float)hs));
  const size_t k0 = (size_t)t * nkv * hs + (size_t)kvh * hs;
  const int hs4 = hs & ~3;
  for (int i0 = 0; i0 < mul; i0 += 4) {
    float a[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int l = 0; l < 4; l++) a[i][l] = 0.0f;
    for (int j = 0; j < hs4; j += 4) {
      float k[4];
#pragma unroll
      for (int l = 0; l < 4; l++) k[l] = cache_at(kc, k0 + j + l, half);
#pragma unroll
      for (int i = 0; i < 4; i++)
        if (i0 + i < mul)
#pragma unroll
          for (int l = 0; l < 4; l++) a[i][l] = __fadd_rn(a[i][l], __fmul_rn(qs[(i0 + i) * hs + j + l], k[l]));
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
      if (i0 + i >= mul) break;
      float sc = __fadd_rn(__fadd_rn(a[i][0], a[i][2]), __fadd_rn(a[i][1], a[i][3]));
      for (int j = hs4; j < hs; j++) sc = __fadd_rn(sc, __fmul_rn(qs[(i0 + i) * hs + j], cache_at(kc, k0 + j, half)));
      att[(size_t)(kvh * mul + i0 + i) * count + t] = __fmul_rn(sc, isq);
    }
  }
}

constexpr int kDS = 16;    // dimensions a CTA of part 2
constexpr int kCH = 512;   // positions a staged chunk of values

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// a chunk of kCH positions' kDS values of this CTA's slice into shared memory (16-byte copies)
__device__ __forceinline__ void stage_values(uint8_t* buf, const uint8_t* vc, int t0, int count, int nkv, int hs,
                                             int kvh, int d0, int E) {
  const int per = kDS * E / 16;  // copies a position
  const int n = min(kCH, count - t0) * per;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int t = i / per, part = i % per;
    const size_t at = ((size_t)(t0 + t) * nkv * hs + (size_t)kvh * hs + d0) * E + part * 16;
    cp_async16(buf + (size_t)t * kDS * E + part * 16, vc + at);
  }
}

// ---- attention, part 2: softmax (largest, exp, the four lanes' sum then the rest) and the weighted values, a CTA
// a (kv head, kDS dimensions); every CTA of a kv head makes the same probabilities. Shared: the probabilities of
// the kv head's heads (mul x capacity floats) and two chunks of values.
__global__ void __launch_bounds__(256) exact_values_kernel(float* __restrict__ out, const float* __restrict__ att,
                                                           const uint8_t* __restrict__ vc,
                                                           const int* __restrict__ pos_dev, int pos_host, int nh,
                                                           int nkv, int hs, int half, float cap, int capacity) {
  extern __shared__ __align__(16) uint8_t smv[];
  const int E = half ? 2 : 4;
  uint8_t* vbuf = smv;                                                 // 2 x kCH x kDS x E bytes
  float* w = reinterpret_cast<float*>(smv + 2 * kCH * kDS * E);        // mul x count
  __shared__ float red[8], mx[8], inv[8], part[8][4];
  const int count = (pos_dev ? *pos_dev : pos_host) + 1, count4 = count & ~3;
  const int kvh = blockIdx.x, d0 = blockIdx.y * kDS, mul = nh / nkv, tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;
  (void)capacity;
  stage_values(vbuf, vc, 0, count, nkv, hs, kvh, d0, E);
  cp_async_commit();
  for (int i = 0; i < mul; i++)
    for (int u = tid; u < count; u += blockDim.x) {
      float s = att[(size_t)(kvh * mul + i) * count + u];
      if (cap > 0.0f) {
        const float twice = __fdiv_rn(2.0f, cap);
        const float e = u < count4 ? ref_vexp(__fmul_rn(s, twice)) : ref_fexp(__fmul_rn(s, twice));
        s = __fmul_rn(cap, __fsub_rn(1.0f, __fdiv_rn(2.0f, __fadd_rn(e, 1.0f))));
      }
      w[i * count + u] = s;
    }
  __syncthreads();
  for (int i = 0; i < mul; i++) {  // largest (math.ts:67-89): from -FLT_MAX, a NaN anywhere makes it NaN
    float m = -FLT_MAX;
    for (int u = tid; u < count; u += blockDim.x) m = wasm_max(m, w[i * count + u]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = wasm_max(m, __shfl_xor_sync(kFull, m, o));
    if (lane == 0) red[warp] = m;
    __syncthreads();
    if (tid == 0) {
      float r = red[0];
      for (int k = 1; k < (int)(blockDim.x >> 5); k++) r = wasm_max(r, red[k]);
      mx[i] = r;
    }
    __syncthreads();
  }
  for (int i = 0; i < mul; i++)
    for (int u = tid; u < count; u += blockDim.x) {
      const float x = __fsub_rn(w[i * count + u], mx[i]);
      w[i * count + u] = u < count4 ? ref_vexp(x) : ref_fexp(x);
    }
  __syncthreads();
  if (tid < mul * 4) {
    const int i = tid >> 2, l = tid & 3;
    const float* e = w + i * count;
    float a = 0.0f;
#pragma unroll 8
    for (int u = l; u < count4; u += 4) a = __fadd_rn(a, e[u]);
    part[i][l] = a;
  }
  __syncthreads();
  if (tid < mul) {
    const float* e = w + tid * count;
    float sum = __fadd_rn(__fadd_rn(__fadd_rn(part[tid][0], part[tid][1]), part[tid][2]), part[tid][3]);
    for (int u = count4; u < count; u++) sum = __fadd_rn(sum, e[u]);
    inv[tid] = __fdiv_rn(1.0f, sum);
  }
  __syncthreads();
  for (int i = 0; i < mul; i++)
    for (int u = tid; u < count; u += blockDim.x) w[i * count + u] = __fmul_rn(w[i * count + u], inv[i]);
  __syncthreads();
  // the weighted values: thread (i, d) one chain over the positions, four at a time ((w0 v0 + w1 v1) + (w2 v2 +
  // w3 v3) added to the sum), then the positions past the fours one at a time
  const bool chain = tid < mul * kDS;
  const int ci = tid / kDS, cd = tid % kDS;
  const float* wi = w + (chain ? ci : 0) * count;
  float o = 0.0f;
  const int chunks = (count + kCH - 1) / kCH;
  for (int ch = 0; ch < chunks; ch++) {
    if (ch + 1 < chunks) stage_values(vbuf + ((ch + 1) & 1) * kCH * kDS * E, vc, (ch + 1) * kCH, count, nkv, hs, kvh,
                                      d0, E);
    cp_async_commit();
    cp_async_wait1();
    __syncthreads();
    if (chain) {
      const uint8_t* vb = vbuf + (ch & 1) * kCH * kDS * E;
      const int t0 = ch * kCH, t1 = min(count, t0 + kCH), t4 = min(t1, count4);
      int t = t0;
      for (; t < t4; t += 4) {
        const float v0 = cache_at(vb, (size_t)(t - t0) * kDS + cd, half);
        const float v1 = cache_at(vb, (size_t)(t - t0 + 1) * kDS + cd, half);
        const float v2 = cache_at(vb, (size_t)(t - t0 + 2) * kDS + cd, half);
        const float v3 = cache_at(vb, (size_t)(t - t0 + 3) * kDS + cd, half);
        const float p0 = __fadd_rn(__fmul_rn(wi[t], v0), __fmul_rn(wi[t + 1], v1));
        const float p1 = __fadd_rn(__fmul_rn(wi[t + 2], v2), __fmul_rn(wi[t + 3], v3));
        o = __fadd_rn(o, __fadd_rn(p0, p1));
      }
      for (; t < t1; t++) o = __fadd_rn(o, __fmul_rn(wi[t], cache_at(vb, (size_t)(t - t0) * kDS + cd, half)));
    }
    __syncthreads();
  }
  if (chain) out[(size_t)(kvh * mul + ci) * hs + d0 + cd] = o;
}

// a launch whose dynamic and static shared memory pass 48 KB needs the kernel's limit raised first (on this device;
// the kernels here hold at most a few hundred static bytes)
template <typename K>
bool raise_smem(K kernel, size_t smem, const char* name) {
  if (smem <= 40 * 1024) return true;
  const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) pllm_fail(PLLM_ECUDA, "%s: %zu bytes of shared memory: %s", name, smem, cudaGetErrorString(e));
  return e == cudaSuccess;
}

size_t values_smem(int mul, int capacity, int half) {
  return (size_t)2 * kCH * kDS * (half ? 2 : 4) + (size_t)mul * capacity * 4;
}

}  // namespace

// x (n floats; mode 2: h1 then h3, 2 n floats) -> mode 0 as it is, 1 rmsnorm with norm, 2 swiglu; then quantize_x
// into xq / xs; out (optional) gets the float32 vector that was quantized
PLLM_API void pllm_exact_prepare(uint64_t xq, uint64_t xs, uint64_t out, uint64_t x, uint64_t norm, int32_t n,
                                 float eps, int32_t bias, int32_t mode) {
  PLLM_REQUIRE(xq && xs && x && n > 0 && n % 32 == 0 && n <= 49152 && (bias == 0 || bias == 64) && mode >= 0 &&
                   mode <= 2 && (mode != 1 || norm),
               "pllm_exact_prepare: n %d bias %d mode %d", n, bias, mode);
  const size_t smem = (size_t)n * 4;
  if (!raise_smem(exact_prepare_kernel, smem, "pllm_exact_prepare")) return;
  exact_prepare_kernel<<<1, 1024, smem, pllm_stream()>>>(dptr<uint8_t>(xq), dptr<float>(xs), dptr<float>(out),
                                                         dptr<const float>(x), dptr<const float>(norm), n, eps, bias,
                                                         mode);
  PLLM_LAUNCHED("pllm_exact_prepare");
}

// rows 0..rows of an int8 product in matmul_q8's order (relaxed 0: xq signed, bias 0) or matmul_q8r's (relaxed 1:
// xq the bias-64 bytes); add non-null: out[r] = add[r] + the row (add may be out: the residual's x +=)
PLLM_API void pllm_exact_product(uint64_t out, uint64_t add, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws,
                                 int32_t n, int32_t rows, int32_t relaxed) {
  PLLM_REQUIRE(out && xq && xs && wq && ws && n > 0 && n % 32 == 0 && n <= 65536 && rows >= 0 &&
                   (xq % 16) == 0 && (wq % 16) == 0,
               "pllm_exact_product: n %d rows %d", n, rows);
  if (rows == 0) return;
  const size_t smem = (size_t)n + (size_t)n / 8;
  const unsigned grid = std::min(cdiv((unsigned)rows, 8u), (unsigned)pllm_num_sms() * 8);
  if (!raise_smem(exact_product_kernel<true>, smem, "pllm_exact_product") ||
      !raise_smem(exact_product_kernel<false>, smem, "pllm_exact_product"))
    return;
  if (relaxed)
    exact_product_kernel<true><<<grid, 256, smem, pllm_stream()>>>(dptr<float>(out), dptr<const float>(add),
                                                                   dptr<const uint8_t>(xq), dptr<const float>(xs),
                                                                   dptr<const int8_t>(wq), dptr<const float>(ws), n,
                                                                   rows);
  else
    exact_product_kernel<false><<<grid, 256, smem, pllm_stream()>>>(dptr<float>(out), dptr<const float>(add),
                                                                    dptr<const uint8_t>(xq), dptr<const float>(xs),
                                                                    dptr<const int8_t>(wq), dptr<const float>(ws), n,
                                                                    rows);
  PLLM_LAUNCHED("pllm_exact_product");
}

// qkv: nh q heads, nkv k heads, nkv v heads of hs floats; q / k normed (null weights: not) and turned in place, the
// key and value written to the cache at the position (pos_dev: device int32, or pos where pos_dev is 0)
PLLM_API void pllm_exact_qk_rope_cache(uint64_t qkv, uint64_t q_norm, uint64_t k_norm, uint64_t cos_t, uint64_t sin_t,
                                       uint64_t pos_dev, int32_t pos, uint64_t kc, uint64_t vc, int32_t nh,
                                       int32_t nkv, int32_t hs, float eps, int32_t half, uint64_t bad) {
  PLLM_REQUIRE(qkv && cos_t && sin_t && kc && vc && nh > 0 && nkv > 0 && hs > 0 && hs % 2 == 0 && hs <= 512 &&
                   (pos_dev || pos >= 0),
               "pllm_exact_qk_rope_cache: nh %d nkv %d hs %d", nh, nkv, hs);
  exact_qk_rope_cache_kernel<<<nh + 2 * nkv, 32, 0, pllm_stream()>>>(
      dptr<float>(qkv), dptr<const float>(q_norm), dptr<const float>(k_norm), dptr<const float>(cos_t),
      dptr<const float>(sin_t), dptr<const int>(pos_dev), pos, dptr<uint8_t>(kc), dptr<uint8_t>(vc), nh, nkv, hs, eps,
      half, dptr<int>(bad));
  PLLM_LAUNCHED("pllm_exact_qk_rope_cache");
}

// attention of nh heads over positions 0..pos (pos_dev: device int32, or pos) of a cache of capacity positions, in
// attentionOf's order; att: nh x capacity floats of scratch (it holds the scaled scores afterwards); cap > 0: the
// capped scores cap (1 - 2 / (exp(2 s / cap) + 1)) of attention_capped
PLLM_API void pllm_exact_attention(uint64_t out, uint64_t q, uint64_t kc, uint64_t vc, uint64_t att, uint64_t pos_dev,
                                   int32_t pos, int32_t capacity, int32_t nh, int32_t nkv, int32_t hs, int32_t half,
                                   float cap) {
  PLLM_REQUIRE(out && q && kc && vc && att && (vc % 16) == 0 && nh > 0 && nkv > 0 && nh % nkv == 0 && nh / nkv <= 8 && hs > 0 &&
                   hs % kDS == 0 && capacity > 0 && (pos_dev || (pos >= 0 && pos < capacity)),
               "pllm_exact_attention: nh %d nkv %d hs %d capacity %d pos %d", nh, nkv, hs, capacity, pos);
  const int mul = nh / nkv;
  const size_t smem = values_smem(mul, capacity, half);
  PLLM_REQUIRE(smem <= 227 * 1024, "pllm_exact_attention: %d positions of %d heads a kv head exceed shared memory",
               capacity, mul);
  if (!raise_smem(exact_values_kernel, smem, "pllm_exact_attention")) return;
  exact_scores_kernel<<<dim3(cdiv((unsigned)capacity, 128u), nkv), 128, (size_t)mul * hs * 4, pllm_stream()>>>(
      dptr<float>(att), dptr<const float>(q), dptr<const uint8_t>(kc), dptr<const int>(pos_dev), pos, nh, nkv, hs,
      half);
  PLLM_LAUNCHED("pllm_exact_attention (scores)");
  exact_values_kernel<<<dim3(nkv, hs / kDS), 256, smem, pllm_stream()>>>(
      dptr<float>(out), dptr<const float>(att), dptr<const uint8_t>(vc), dptr<const int>(pos_dev), pos, nh, nkv, hs,
      half, cap, capacity);
  PLLM_LAUNCHED("pllm_exact_attention (values)");
}
