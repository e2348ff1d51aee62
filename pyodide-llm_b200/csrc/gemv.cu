// gemv.cu: the decode-shape products (M = 1..16 tokens): weights streamed from HBM once, activations in shared
// memory, integer group sums by dp4a, float32 scaling, warp-shuffle reductions.
//
// The registry's products (the reference's kernel names and arguments):
//   matmul_q8, matmul_q8r, matmul_q8r_tile            kernels/kernel/matmul.ts:77, kernels/relaxed/int8.ts:17,147
//   matmul_q6, matmul_q6r                             kernels/kernel/matmul.ts:227, kernels/relaxed/six.ts:16
//   matmul_t2, matmul_t2r, matmul_t2r_tile            kernels/kernel/matmul.ts:218, kernels/relaxed/signs.ts:117,120
//   matmul_b1, matmul_b1r, matmul_b1r_tile            kernels/kernel/matmul.ts:222, kernels/relaxed/signs.ts:123,126
//   matmul_f32                                        kernels/kernel/matmul.ts:13
// The forward driver's product (pllm_gemv): the same kernel with its input made from float32 activations in its
// prologue (RMSNorm and quantize_x fused) and its output fused with the residual add or the SwiGLU of a row pair.
//
// Every group's integer is exact (int32, dp4a): the accumulators equal the reference's to the bit (pllm_group_sums
// exposes them). The float32 sum over the groups runs in another order than the reference's four SIMD lanes, so
// outputs agree within float32 rounding, not to the bit.
//
// Layout: one warp a row; lane l takes the row's weight units l, l + 32, ... (a unit: 32 bytes of int8 = a group of
// 32; 24 bytes of int6 = a group of 32; 32 bytes of ternary or 16 of binary = a group of 128), four units in flight
// per lane. Consecutive lanes read consecutive units, so a warp's loads cover whole 32-byte sectors.
#include "pllm_common.cuh"
#include "pllm_device.cuh"

#include "gemv_common.cuh"

namespace {

using namespace gemvk;

// one unit's weights, read from HBM
template <int FMT> struct Unit { uint32_t w[8]; float s; };

template <int FMT, bool SCALE = true>
__device__ __forceinline__ void load_unit(const GemvArgs& a, long long row, int u, Unit<FMT>& U) {
  constexpr int UB = FmtInfo<FMT>::UB, GK = FmtInfo<FMT>::GK;
  const int units = a.K / GK;
  const uint8_t* p = a.wq + (row * units + u) * (long long)UB;
  if (FMT == F_Q8 || FMT == F_T2) {
    ldg_stream32(p, U.w);
  } else if (FMT == F_Q6) {
    const uint2 v0 = ldg_stream8(p), v1 = ldg_stream8(p + 8), v2 = ldg_stream8(p + 16);
    U.w[0] = v0.x; U.w[1] = v0.y; U.w[2] = v1.x; U.w[3] = v1.y; U.w[4] = v2.x; U.w[5] = v2.y;
  } else {
    const int4 v0 = ldg_stream(p);
    U.w[0] = v0.x; U.w[1] = v0.y; U.w[2] = v0.z; U.w[3] = v0.w;
  }
  if (!SCALE) U.s = 0.0f;
  else if (FMT <= F_Q6) U.s = __ldg(reinterpret_cast<const float*>(a.ws) + row * units + u);
  else U.s = half_bits_to_float(__ldg(reinterpret_cast<const uint16_t*>(a.ws) + row * units + u));
}

// one unit against MT tokens' activations: acc[t] += its scaled group sums
template <int FMT, int MT>
__device__ __forceinline__ void unit_dot(Unit<FMT>& U, int u, int K, const int8_t* sq, const float* ss,
                                         const int32_t* sm, float acc[MT]) {
  const int ng = K / 32;
  if (FMT == F_Q6) {
    uint32_t w[8];
    widen6_regs(U.w[0], U.w[1], U.w[2], U.w[3], U.w[4], U.w[5], w);
#pragma unroll
    for (int k = 0; k < 8; k++) U.w[k] = w[k];
  }
  if (FMT <= F_Q6) {
#pragma unroll
    for (int t = 0; t < MT; t++) {
      const int4* act = reinterpret_cast<const int4*>(sq + (size_t)t * K + u * 32);
      const int G = dot32_words(U.w, act[0], act[1]);
      acc[t] = fmaf((float)G, __fmul_rn(U.s, ss[t * ng + u]), acc[t]);
    }
  } else {
#pragma unroll
    for (int t = 0; t < MT; t++) {
      const int4* act = reinterpret_cast<const int4*>(sq + (size_t)t * K + u * 128);
      int g4[4] = {0, 0, 0, 0};
      if (FMT == F_T2) ternary_group(U.w, act, g4);
      else binary_group(U.w, act, g4);
      const int4 mins = *reinterpret_cast<const int4*>(sm + t * ng + 4 * u);
      const float4 xs4 = *reinterpret_cast<const float4*>(ss + t * ng + 4 * u);
      // relaxed/signs.ts:47-50: (whole * xs) * d, the four groups of 32 of the group
      float r = __fmul_rn(__fmul_rn((float)(g4[0] + mins.x), xs4.x), U.s);
      r += __fmul_rn(__fmul_rn((float)(g4[1] + mins.y), xs4.y), U.s);
      r += __fmul_rn(__fmul_rn((float)(g4[2] + mins.z), xs4.z), U.s);
      r += __fmul_rn(__fmul_rn((float)(g4[3] + mins.w), xs4.w), U.s);
      acc[t] += r;
    }
  }
}

// one row's MT outputs
template <int FMT, int MT>
__device__ __forceinline__ void row_dot(const GemvArgs& a, long long row, const int8_t* sq, const float* ss,
                                        const int32_t* sm, float acc[MT]) {
  constexpr int GK = FmtInfo<FMT>::GK;
  const int units = a.K / GK, lane = threadIdx.x & 31;
#pragma unroll
  for (int t = 0; t < MT; t++) acc[t] = 0.0f;
  int u0 = 0;
  for (; u0 + 32 * UNROLL <= units; u0 += 32 * UNROLL) {
    Unit<FMT> U[UNROLL];
#pragma unroll
    for (int k = 0; k < UNROLL; k++) load_unit<FMT>(a, row, u0 + lane + 32 * k, U[k]);
#pragma unroll
    for (int k = 0; k < UNROLL; k++) unit_dot<FMT, MT>(U[k], u0 + lane + 32 * k, a.K, sq, ss, sm, acc);
  }
  for (int u = u0 + lane; u < units; u += 32) {
    Unit<FMT> U;
    load_unit<FMT>(a, row, u, U);
    unit_dot<FMT, MT>(U, u, a.K, sq, ss, sm, acc);
  }
#pragma unroll
  for (int t = 0; t < MT; t++) acc[t] = warp_sum(acc[t]);
}

template <int FMT, int MT, int PRO, int EPI>
__global__ void __launch_bounds__(THREADS) gemv_kernel(const GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = a.K, ng = K / 32;
  int8_t* sq = reinterpret_cast<int8_t*>(smem);
  float* ss = reinterpret_cast<float*>(smem + (size_t)MT * K);
  int32_t* sm = reinterpret_cast<int32_t*>(smem + (size_t)MT * K + (size_t)MT * ng * 4);
  pdl_wait();  // the activations may be the previous kernel's output
  load_activations<FMT, MT, PRO>(a, sq, ss, sm);
  __syncthreads();
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * WARPS;
  for (long long row = a.r0 + (long long)blockIdx.x * WARPS + (threadIdx.x >> 5); row < a.r1; row += warps) {
    float acc[MT];
    row_dot<FMT, MT>(a, row, sq, ss, sm, acc);
    if (EPI == EPI_SWIGLU) {
      float acc3[MT];
      row_dot<FMT, MT>(a, row + a.pair, sq, ss, sm, acc3);
#pragma unroll
      for (int t = 0; t < MT; t++) acc[t] = (acc[t] / (1.0f + expf(-acc[t]))) * acc3[t];
    }
    if (lane < MT && lane < a.count) {
      float v = acc[0];
#pragma unroll
      for (int t = 1; t < MT; t++)
        if (lane == t) v = acc[t];
      float* o = a.out + lane * a.out_stride + row;
      if (EPI == EPI_ADD) add_once(o, v);
      else *o = v;
    }
  }
}

// the exact integer of every (row, group of 32) of rows [r0, r1): out[(row - r0) * (K / 32) + g] (one token)
template <int FMT>
__global__ void group_sums_kernel(int32_t* __restrict__ out, const GemvArgs a) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int K = a.K, ng = K / 32;
  constexpr int GK = FmtInfo<FMT>::GK;
  int8_t* sq = reinterpret_cast<int8_t*>(smem);
  float* ss = reinterpret_cast<float*>(smem + (size_t)K);
  int32_t* sm = reinterpret_cast<int32_t*>(smem + (size_t)K + (size_t)ng * 4);
  load_activations<FMT, 1, PRO_Q>(a, sq, ss, sm);
  __syncthreads();
  const int units = K / GK;
  const long long total = (long long)(a.r1 - a.r0) * units;
  for (long long i = (long long)blockIdx.x * THREADS + threadIdx.x; i < total; i += (long long)gridDim.x * THREADS) {
    const long long row = a.r0 + i / units;
    const int u = (int)(i % units);
    Unit<FMT> U;
    load_unit<FMT, false>(a, row, u, U);
    if (FMT <= F_Q6) {
      if (FMT == F_Q6) {
        uint32_t w[8];
        widen6_regs(U.w[0], U.w[1], U.w[2], U.w[3], U.w[4], U.w[5], w);
        for (int k = 0; k < 8; k++) U.w[k] = w[k];
      }
      const int4* act = reinterpret_cast<const int4*>(sq + u * 32);
      out[(row - a.r0) * ng + u] = dot32_words(U.w, act[0], act[1]);
    } else {
      const int4* act = reinterpret_cast<const int4*>(sq + u * 128);
      int g4[4] = {0, 0, 0, 0};
      if (FMT == F_T2) ternary_group(U.w, act, g4);
      else binary_group(U.w, act, g4);
      for (int s = 0; s < 4; s++) out[(row - a.r0) * ng + 4 * u + s] = g4[s] + sm[4 * u + s];
    }
  }
}

// ---- launching

template <int FMT, int MT, int PRO, int EPI>
void launch_one(const GemvArgs& a, bool pdl) {
  const size_t smem = smem_bytes<FMT>(a.K, MT);
  auto kernel = gemv_kernel<FMT, MT, PRO, EPI>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  const long long rows = a.r1 - a.r0;
  int per_sm = smem > 100 * 1024 ? 1 : (smem > 48 * 1024 ? 2 : 4);
  long long blocks = (rows + WARPS - 1) / WARPS;
  const long long most = (long long)pllm_num_sms() * per_sm;
  if (blocks > most) blocks = most;
  if (blocks < 1) blocks = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)blocks);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = pllm_stream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, a);
  if (e != cudaSuccess) pllm_fail(PLLM_ECUDA, "gemv launch (fmt %d, %d tokens): %s", FMT, MT, cudaGetErrorString(e));
}

// tokens in passes of at most MT; a pass reads the rows again (from L2 where they fit)
template <int FMT, int PRO, int EPI>
void launch_tokens(GemvArgs a, bool pdl) {
  const int total = a.count;
  for (int t0 = 0; t0 < total;) {
    GemvArgs b = a;
    const int left = total - t0;
    // the largest MT whose activations fit in shared memory with room to spare
    int mt = left >= 16 ? 16 : left >= 8 ? 8 : left >= 4 ? 4 : left >= 2 ? 2 : 1;
    while (mt > 1 && smem_bytes<FMT>(a.K, mt) > 200 * 1024) mt >>= 1;
    if (left < mt) mt = left;
    b.count = mt;
    b.out = a.out + t0 * a.out_stride;
    if (PRO == PRO_Q) {
      b.xq = a.xq + t0 * a.xq_stride;
      b.xs = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(a.xs) + t0 * a.xs_stride);
    } else {
      b.x = a.x + t0 * a.x_stride;
    }
    switch (mt) {
      case 16: launch_one<FMT, 16, PRO, EPI>(b, pdl); break;
      case 8: launch_one<FMT, 8, PRO, EPI>(b, pdl); break;
      case 4: launch_one<FMT, 4, PRO, EPI>(b, pdl); break;
      case 2: launch_one<FMT, 2, PRO, EPI>(b, pdl); break;
      default: launch_one<FMT, 1, PRO, EPI>(b, pdl); break;
    }
    t0 += mt;
  }
}

template <int PRO, int EPI>
void launch_fmt(int fmt, const GemvArgs& a, bool pdl) {
  if (gemv_tma(a, fmt, PRO, EPI, pdl)) return;
  switch (fmt) {
    case F_Q8: launch_tokens<F_Q8, PRO, EPI>(a, pdl); break;
    case F_Q6: launch_tokens<F_Q6, PRO, EPI>(a, pdl); break;
    default:
      // ternary and binary take interleaved activations, made by the caller; ternary from float32 activations is the
      // bulk-copy form's alone
      if constexpr (PRO == PRO_Q) {
        if (fmt == F_T2) launch_tokens<F_T2, PRO, EPI>(a, pdl);
        else launch_tokens<F_B1, PRO, EPI>(a, pdl);
      } else {
        pllm_fail(PLLM_EINVAL, "pllm_gemv: ternary weights from float32 activations need the bulk-copy form (K %% 128, "
                               "K / 128 a multiple of 8, 16-byte aligned weights and scales)");
      }
      break;
  }
}

bool check_rows(const char* name, int n, int r0, int r1, int group) {
  if (n <= 0 || n % group) {
    pllm_fail(PLLM_EINVAL, "%s: n = %d is not whole groups of %d", name, n, group);
    return false;
  }
  if (r0 < 0 || r1 < r0) {
    pllm_fail(PLLM_EINVAL, "%s: rows %d..%d", name, r0, r1);
    return false;
  }
  return true;
}

void registry_product(const char* name, int fmt, uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws,
                      int n, int r0, int r1, int bias, int count, long long os, long long frame) {
  const int group = fmt >= F_T2 ? 128 : 32;
  if (!check_rows(name, n, r0, r1, group)) return;
  if (r1 == r0 || count <= 0) return;
  if (!xout || !xq || !xs || !wq || !ws) {
    pllm_fail(PLLM_EINVAL, "%s: null address", name);
    return;
  }
  if ((xq & 15) || (xs & 15) || (frame & 15)) {
    pllm_fail(PLLM_EINVAL, "%s: the activations (and their frame) must be 16-byte aligned", name);
    return;
  }
  if (fmt == F_Q8 && (wq & 31)) {
    pllm_fail(PLLM_EINVAL, "%s: int8 weights must be 32-byte aligned", name);
    return;
  }
  if (fmt == F_Q6 && (wq & 7)) {
    pllm_fail(PLLM_EINVAL, "%s: int6 weights must be 8-byte aligned", name);
    return;
  }
  if ((fmt == F_T2 && (wq & 31)) || (fmt == F_B1 && (wq & 15))) {
    pllm_fail(PLLM_EINVAL, "%s: ternary weights must be 32-byte aligned, binary 16", name);
    return;
  }
  if (os % 4) {
    pllm_fail(PLLM_EINVAL, "%s: os = %lld is not whole floats", name, os);
    return;
  }
  GemvArgs a = {};
  a.out = dptr<float>(xout);
  a.out_stride = os / 4;
  a.xq = dptr<const uint8_t>(xq);
  a.xs = dptr<const float>(xs);
  a.xq_stride = frame;
  a.xs_stride = frame;
  a.bias = bias;
  a.wq = dptr<const uint8_t>(wq);
  a.ws = dptr<const void>(ws);
  a.K = n;
  a.r0 = r0;
  a.r1 = r1;
  a.count = count;
  launch_fmt<PRO_Q, EPI_STORE>(fmt, a, false);
}

}  // namespace

// ---- the registry (the reference's names and arguments; the addresses are device pointers)

// matmul.ts:77: int8 weights (wq, rows of n bytes), a float32 scale a group of 32 (ws), activations of
// quantize_x(bias 0)
PLLM_API void matmul_q8(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n, int32_t r0,
                        int32_t r1) {
  registry_product("matmul_q8", F_Q8, xout, xq, xs, wq, ws, n, r0, r1, 0, 1, 0, 0);
}

// relaxed/int8.ts:17: activations of quantize_x(bias 64). wc (int8_sums: -64 times each group's sum) takes the bias
// out in the reference; here the bias is taken off the activations as they are loaded, the same exact integer
// dot(w, q - 64), so wc is not read (it must be int8_sums' of wq, as the reference's callers make it).
PLLM_API void matmul_q8r(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, uint64_t wc, int32_t n,
                         int32_t r0, int32_t r1) {
  (void)wc;
  registry_product("matmul_q8r", F_Q8, xout, xq, xs, wq, ws, n, r0, r1, 64, 1, 0, 0);
}

// relaxed/int8.ts:147: count tokens, token t's activations and scales at xq + t frame and xs + t frame (bytes), its
// outputs at xout + t os (bytes)
PLLM_API void matmul_q8r_tile(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, uint64_t wc,
                              int32_t n, int32_t r0, int32_t r1, int32_t count, int32_t os, int32_t frame) {
  (void)wc;
  registry_product("matmul_q8r_tile", F_Q8, xout, xq, xs, wq, ws, n, r0, r1, 64, count, os, frame);
}

// matmul.ts:227 / relaxed/six.ts:16: int6 weights, 24 bytes a group of 32
PLLM_API void matmul_q6(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n, int32_t r0,
                        int32_t r1) {
  registry_product("matmul_q6", F_Q6, xout, xq, xs, wq, ws, n, r0, r1, 0, 1, 0, 0);
}
PLLM_API void matmul_q6r(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, uint64_t wc, int32_t n,
                         int32_t r0, int32_t r1) {
  (void)wc;
  registry_product("matmul_q6r", F_Q6, xout, xq, xs, wq, ws, n, r0, r1, 64, 1, 0, 0);
}

// matmul.ts:218 / relaxed/signs.ts:117: ternary weights (two bits a weight, a float16 scale a group of 128) against
// the activations interleave() laid out. three: the mask of the codes, 3
PLLM_API void matmul_t2(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n, int32_t r0,
                        int32_t r1, int32_t three) {
  PLLM_REQUIRE(three == 3, "matmul_t2: three = %d (the codes' mask is 3)", three);
  registry_product("matmul_t2", F_T2, xout, xq, xs, wq, ws, n, r0, r1, 0, 1, 0, 0);
}
PLLM_API void matmul_t2r(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n, int32_t r0,
                         int32_t r1, int32_t three) {
  PLLM_REQUIRE(three == 3, "matmul_t2r: three = %d (the codes' mask is 3)", three);
  registry_product("matmul_t2r", F_T2, xout, xq, xs, wq, ws, n, r0, r1, 0, 1, 0, 0);
}
PLLM_API void matmul_t2r_tile(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n,
                              int32_t r0, int32_t r1, int32_t count, int32_t os, int32_t frame, int32_t three) {
  PLLM_REQUIRE(three == 3, "matmul_t2r_tile: three = %d (the codes' mask is 3)", three);
  registry_product("matmul_t2r_tile", F_T2, xout, xq, xs, wq, ws, n, r0, r1, 0, count, os, frame);
}
// matmul.ts:222 / relaxed/signs.ts:123: binary weights (a bit a weight). two: the mask of the codes, 2
PLLM_API void matmul_b1(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n, int32_t r0,
                        int32_t r1, int32_t two) {
  PLLM_REQUIRE(two == 2, "matmul_b1: two = %d (the codes' mask is 2)", two);
  registry_product("matmul_b1", F_B1, xout, xq, xs, wq, ws, n, r0, r1, 0, 1, 0, 0);
}
PLLM_API void matmul_b1r(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n, int32_t r0,
                         int32_t r1, int32_t two) {
  PLLM_REQUIRE(two == 2, "matmul_b1r: two = %d (the codes' mask is 2)", two);
  registry_product("matmul_b1r", F_B1, xout, xq, xs, wq, ws, n, r0, r1, 0, 1, 0, 0);
}
PLLM_API void matmul_b1r_tile(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n,
                              int32_t r0, int32_t r1, int32_t count, int32_t os, int32_t frame, int32_t two) {
  PLLM_REQUIRE(two == 2, "matmul_b1r_tile: two = %d (the codes' mask is 2)", two);
  registry_product("matmul_b1r_tile", F_B1, xout, xq, xs, wq, ws, n, r0, r1, 0, count, os, frame);
}

// the exact int32 group sums of rows [r0, r1) against one token: out[(row - r0) * (n / 32) + g]. fmt: 0 int8,
// 1 int6, 2 ternary, 3 binary; bias: 0 or 64 (int8 and int6); ternary and binary take interleaved activations and
// the minus-sums after their scales, and their groups of 32 are the four of each group of 128
PLLM_API void pllm_group_sums(uint64_t out, uint64_t xq, uint64_t xs, uint64_t wq, int32_t fmt, int32_t n, int32_t r0,
                              int32_t r1, int32_t bias) {
  PLLM_REQUIRE(fmt >= 0 && fmt <= 3, "pllm_group_sums: fmt %d", fmt);
  if (!check_rows("pllm_group_sums", n, r0, r1, fmt >= F_T2 ? 128 : 32) || r0 == r1) return;
  GemvArgs a = {};
  a.xq = dptr<const uint8_t>(xq);
  a.xs = dptr<const float>(xs);
  a.wq = dptr<const uint8_t>(wq);
  a.K = n;
  a.r0 = r0;
  a.r1 = r1;
  a.count = 1;
  a.bias = bias;
  const size_t smem = (size_t)n + (size_t)(n / 32) * 8;
  const unsigned blocks = (unsigned)((((long long)(r1 - r0) * (n / (fmt >= 2 ? 128 : 32))) + THREADS - 1) / THREADS);
  const unsigned grid = blocks > 1024 ? 1024 : blocks;
#define GS_LAUNCH(F)                                                                                     \
  do {                                                                                                   \
    if (smem > 48 * 1024) cudaFuncSetAttribute(group_sums_kernel<F>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    group_sums_kernel<F><<<grid, THREADS, smem, pllm_stream()>>>(dptr<int32_t>(out), a);                  \
  } while (0)
  switch (fmt) {
    case 0: GS_LAUNCH(F_Q8); break;
    case 1: GS_LAUNCH(F_Q6); break;
    case 2: GS_LAUNCH(F_T2); break;
    default: GS_LAUNCH(F_B1); break;
  }
#undef GS_LAUNCH
  PLLM_LAUNCHED("pllm_group_sums");
}

// ---- the forward driver's product
// fmt: 0 int8, 1 int6, 2 ternary, 3 binary. pro: 0 the activations given quantized (xq, xs, token strides xq_stride
// and xs_stride bytes), 1 RMSNorm of x with norm then quantize_x, 2 quantize_x of x (x token stride x_stride floats).
// epi: 0 out = W x, 1 out += W x (the residual), 2 out = silu(W[row] x) * W[row + pair] x (the gated FFN's pair of
// matrices in one, w1's rows then w3's). count: tokens. pdl: 1 launches it as a programmatic dependent of the
// kernel before it on the stream.
PLLM_API void pllm_gemv(uint64_t out, int64_t out_stride, uint64_t xq, uint64_t xs, int64_t xq_stride,
                        int64_t xs_stride, uint64_t x, int64_t x_stride, uint64_t norm, float eps, int32_t bias,
                        uint64_t wq, uint64_t ws, int32_t fmt, int32_t n, int32_t r0, int32_t r1, int32_t count,
                        int32_t pro, int32_t epi, int64_t pair, int32_t pdl) {
  PLLM_REQUIRE(fmt >= 0 && fmt <= 3 && pro >= 0 && pro <= 2 && epi >= 0 && epi <= 2, "pllm_gemv: fmt %d pro %d epi %d",
               fmt, pro, epi);
  if (!check_rows("pllm_gemv", n, r0, r1, fmt >= F_T2 ? 128 : 32) || r0 == r1 || count <= 0) return;
  PLLM_REQUIRE(!(fmt == F_B1 && pro != PRO_Q) && !(fmt == F_T2 && pro != PRO_Q && count != 1),
               "pllm_gemv: binary (and ternary past one token) take interleaved activations (pro 0)");
  PLLM_REQUIRE(bias == 0 || bias == 64, "pllm_gemv: bias %d", bias);
  GemvArgs a = {};
  a.out = dptr<float>(out);
  a.out_stride = out_stride;
  a.xq = dptr<const uint8_t>(xq);
  a.xs = dptr<const float>(xs);
  a.xq_stride = xq_stride;
  a.xs_stride = xs_stride;
  a.x = dptr<const float>(x);
  a.x_stride = x_stride;
  a.norm = dptr<const float>(norm);
  a.eps = eps;
  a.bias = bias;
  a.wq = dptr<const uint8_t>(wq);
  a.ws = dptr<const void>(ws);
  a.K = n;
  a.r0 = r0;
  a.r1 = r1;
  a.count = count;
  a.pair = pair;
  const bool p = pdl != 0;
#define EPI_CASES(PRO)                                   \
  switch (epi) {                                         \
    case EPI_STORE: launch_fmt<PRO, EPI_STORE>(fmt, a, p); break; \
    case EPI_ADD: launch_fmt<PRO, EPI_ADD>(fmt, a, p); break;     \
    default: launch_fmt<PRO, EPI_SWIGLU>(fmt, a, p); break;       \
  }
  switch (pro) {
    case PRO_Q: EPI_CASES(PRO_Q); break;
    case PRO_RMS: EPI_CASES(PRO_RMS); break;
    default: EPI_CASES(PRO_QUANT); break;
  }
#undef EPI_CASES
}

// ---- matmul_f32 (matmul.ts:13): float32 weights, a warp a row
namespace {
__global__ void matmul_f32_kernel(float* __restrict__ out, const float* __restrict__ x, const float* __restrict__ w,
                                  int n, int r0, int r1) {
  const int lane = threadIdx.x & 31;
  for (long long row = r0 + (long long)blockIdx.x * WARPS + (threadIdx.x >> 5); row < r1;
       row += (long long)gridDim.x * WARPS) {
    const float* wr = w + row * n;
    float s = 0.0f;
    for (int j = lane; j < n; j += 32) s = fmaf(wr[j], x[j], s);
    s = warp_sum(s);
    if (lane == 0) out[row] = s;
  }
}
}  // namespace

PLLM_API void matmul_f32(uint64_t xout, uint64_t x, uint64_t w, int32_t n, int32_t r0, int32_t r1) {
  PLLM_REQUIRE(n > 0 && r0 >= 0 && r1 >= r0, "matmul_f32: n %d rows %d..%d", n, r0, r1);
  if (r0 == r1) return;
  long long blocks = (r1 - r0 + WARPS - 1) / WARPS;
  if (blocks > pllm_num_sms() * 8) blocks = pllm_num_sms() * 8;
  matmul_f32_kernel<<<(unsigned)blocks, THREADS, 0, pllm_stream()>>>(dptr<float>(xout), dptr<const float>(x),
                                                                   dptr<const float>(w), n, r0, r1);
  PLLM_LAUNCHED("matmul_f32");
}
