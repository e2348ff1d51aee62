// sample.cu: from the logits to a token on the device (kernels/kernel/sample.ts), so that a decode step returns 4
// bytes instead of the vocabulary's logits.
//   argmax     sample.ts:6-10   the first index of the largest (strictly greater wins: the lowest index of equal ones;
//                               a NaN is never greater, and one at index 0 stays the answer, as the reference's walk)
//   penalize   sample.ts:16-30  each distinct token of the list once: a positive logit divided by penalty, another
//                               multiplied by it, then presence taken off (presence <= 0: nothing)
//
// The argmax is a grid of CTAs, each reducing its elements to one 64-bit key (the value's bits made to order as
// unsigned integers, then the complement of the index, so that the largest key is the largest value at its lowest
// index), combined by atomicMax; the last CTA turns the key into the index and sets the key and count back to zero.
#include "pllm_common.cuh"

namespace {

constexpr int AM_THREADS = 256;

// a float's bits made to order as unsigned: larger value, larger key (-inf lowest of the non-NaN)
__device__ __forceinline__ unsigned ordered(float v) {
  const unsigned b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__global__ void argmax_kernel(const float* __restrict__ x, int n, unsigned long long* key, unsigned* count, int* out) {
  unsigned long long best = 0;  // no element (every one a NaN): key 0
  for (long long i = blockIdx.x * (long long)AM_THREADS + threadIdx.x; i < n; i += (long long)gridDim.x * AM_THREADS) {
    const float v = x[i];
    if (v != v) continue;
    const unsigned long long k = ((unsigned long long)ordered(v) << 32) | (0xFFFFFFFFu - (unsigned)i);
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  __shared__ unsigned long long warps[AM_THREADS / 32];
  __shared__ bool last;
  if ((threadIdx.x & 31) == 0) warps[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < AM_THREADS / 32; w++) best = warps[w] > best ? warps[w] : best;
    atomicMax(key, best);
    __threadfence();
    last = atomicAdd(count, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  const unsigned long long k = atomicExch(key, 0ull);
  int idx = k ? (int)(0xFFFFFFFFu - (unsigned)(k & 0xFFFFFFFFu)) : 0;
  const float x0 = x[0];
  if (x0 != x0) idx = 0;  // the walk starts from a NaN: nothing is greater
  *out = idx;
  *count = 0;
}

__global__ void penalize_kernel(float* logits, const int* tokens, int count, float penalty, float presence) {
  const float less = presence > 0.0f ? presence : 0.0f;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < count; i += gridDim.x * blockDim.x) {
    const int token = tokens[i];
    bool seen = false;
    for (int j = 0; j < i && !seen; j++) seen = tokens[j] == token;
    if (seen) continue;
    const float v = logits[token];
    logits[token] = (v > 0.0f ? v / penalty : v * penalty) - less;
  }
}

int grid_for(int n) {
  int g = (n + AM_THREADS * 8 - 1) / (AM_THREADS * 8);
  const int most = pllm_num_sms();
  return g < 1 ? 1 : (g > most ? most : g);
}

}  // namespace

// The library's own scratch for the registry's argmax (it returns the index, so it waits for it): a key and a count,
// zero between calls; calls that overlap on the GPU race on it.
static __device__ unsigned long long g_argmax_key = 0;
static __device__ unsigned g_argmax_count = 0;
static __device__ int g_argmax_out = 0;

// argmax (sample.ts:6): the first index of the largest of n floats at x
PLLM_API int32_t argmax(uint64_t x, int32_t n) {
  PLLM_REQUIRE_RET(x && n > 0, 0, "argmax: n %d", n);
  void *key = nullptr, *count = nullptr, *out = nullptr;
  if (cudaGetSymbolAddress(&key, g_argmax_key) != cudaSuccess ||
      cudaGetSymbolAddress(&count, g_argmax_count) != cudaSuccess ||
      cudaGetSymbolAddress(&out, g_argmax_out) != cudaSuccess) {
    pllm_fail(PLLM_ECUDA, "argmax: its scratch");
    return 0;
  }
  argmax_kernel<<<grid_for(n), AM_THREADS, 0, pllm_stream()>>>(dptr<const float>(x), n, (unsigned long long*)key,
                                                               (unsigned*)count, (int*)out);
  int idx = 0;
  const cudaError_t e = cudaMemcpyAsync(&idx, out, sizeof idx, cudaMemcpyDeviceToHost, pllm_stream());
  if (e != cudaSuccess || cudaStreamSynchronize(pllm_stream()) != cudaSuccess) {
    pllm_fail(PLLM_ECUDA, "argmax: %s", cudaGetErrorString(e));
    return 0;
  }
  return idx;
}

// the same into device memory, without waiting (the forward driver's greedy step): out one int32; scratch 16 bytes
// of device memory, zero before the first call (every call leaves it at zero)
PLLM_API void pllm_argmax_dev(uint64_t out, uint64_t x, int32_t n, uint64_t scratch) {
  PLLM_REQUIRE(out && x && n > 0 && scratch && !(scratch & 7), "pllm_argmax_dev: n %d", n);
  argmax_kernel<<<grid_for(n), AM_THREADS, 0, pllm_stream()>>>(
      dptr<const float>(x), n, dptr<unsigned long long>(scratch), dptr<unsigned>(scratch + 8), dptr<int>(out));
  PLLM_LAUNCHED("pllm_argmax_dev");
}

// penalize (sample.ts:16): the logits of the distinct tokens of tokens[0..count)
PLLM_API void penalize(uint64_t logits, uint64_t tokens, int32_t count, float penalty, float presence) {
  PLLM_REQUIRE(count >= 0 && (count == 0 || (logits && tokens)), "penalize: count %d", count);
  if (!count) return;
  penalize_kernel<<<(count + 255) / 256, 256, 0, pllm_stream()>>>(dptr<float>(logits), dptr<const int>(tokens), count,
                                                                 penalty, presence);
  PLLM_LAUNCHED("penalize");
}
