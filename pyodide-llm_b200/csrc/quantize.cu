// quantize.cu: the activations as the products take them, and the float16 of the cache.
//   quantize_x   kernels/kernel/quantize.ts:124-151   a warp a group of 32
//   interleave   kernels/kernel/matmul.ts:129-146     a warp a block of 64, in place
//   int8_sums    kernels/kernel/matmul.ts:50-58       a thread a group
//   six_sums     kernels/kernel/matmul.ts:38-46
//   to_f16 / from_f16 / finite_f16   kernels/kernel/halves.ts:35-94
// All byte-exact with the reference: each is integer work or one IEEE float32 operation at a time.
#include "pllm_common.cuh"
#include "pllm_device.cuh"

namespace {

__global__ void quantize_x_kernel(uint8_t* __restrict__ xq, float* __restrict__ xs, const float* __restrict__ x,
                                  int n, int bias, long long token_stride) {
  const int lane = threadIdx.x & 31;
  const int g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const long long t = blockIdx.y;
  if (g * 32 >= n) return;
  const float v = x[t * token_stride + (long long)g * 32 + lane];
  float s;
  const int8_t q = quantize_group_warp(v, lane, bias, &s);
  xq[t * token_stride + (long long)g * 32 + lane] = (uint8_t)q;
  if (lane == 0) xs[t * (token_stride / 32) + g] = s;
}

__global__ void interleave_kernel(uint8_t* __restrict__ xq, float* __restrict__ xs, int n) {
  const int lane = threadIdx.x & 31;
  const int b = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 64;
  if (b >= n) return;
  const int8_t a0 = (int8_t)xq[b + lane], a1 = (int8_t)xq[b + 32 + lane];
  int s0 = a0, s1 = a1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s0 += __shfl_xor_sync(0xffffffffu, s0, o);
    s1 += __shfl_xor_sync(0xffffffffu, s1, o);
  }
  __syncwarp();
  // activation 4 c + p goes to byte 16 p + c of the block
  xq[b + 16 * (lane & 3) + (lane >> 2)] = (uint8_t)a0;
  xq[b + 16 * (lane & 3) + 8 + (lane >> 2)] = (uint8_t)a1;
  if (lane == 0) {
    int32_t* sums = reinterpret_cast<int32_t*>(xs + n / 32);
    sums[b / 32] = -s0;
    sums[b / 32 + 1] = -s1;
  }
}

__global__ void int8_sums_kernel(int32_t* __restrict__ out, const int8_t* __restrict__ w, int groups) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= groups) return;
  const int4* p = reinterpret_cast<const int4*>(w + (size_t)g * 32);
  int s = 0;
#pragma unroll
  for (int h = 0; h < 2; h++) {
    const int4 v = p[h];
    const int words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; k++) s = __dp4a(words[k], 0x01010101, s);
  }
  out[g] = -64 * s;
}

__global__ void six_sums_kernel(int32_t* __restrict__ out, const uint8_t* __restrict__ w, int groups) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= groups) return;
  uint32_t words[8];
  widen6_words(w + (size_t)g * 24, words);
  int s = 0;
#pragma unroll
  for (int k = 0; k < 8; k++) s = __dp4a((int)words[k], 0x01010101, s);
  out[g] = -64 * s;
}

__global__ void to_f16_kernel(uint16_t* __restrict__ out, const float* __restrict__ x, int n, int* __restrict__ bad) {
  int local = 0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = float_to_half_bits(x[i], &local);
  if (local) atomicAdd(bad, local);
}

__global__ void from_f16_kernel(float* __restrict__ out, const uint16_t* __restrict__ x, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    out[i] = half_bits_to_float(x[i]);
}

__global__ void finite_f16_kernel(const uint16_t* __restrict__ x, int n, int* __restrict__ found) {
  int any = 0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    any |= (x[i] & 0x7c00) == 0x7c00;
  if (any) atomicOr(found, 1);
}

// one int32 of device memory for the calls that return a count (to_f16, finite_f16), made once per device
int* status_word() {
  static int* words[64] = {nullptr};
  std::lock_guard<std::mutex> hold(pllm_lookup_lock());
  int dev = 0;
  cudaGetDevice(&dev);
  if (!words[dev & 63]) {
    if (cudaMalloc(&words[dev & 63], sizeof(int)) != cudaSuccess) {
      pllm_fail(PLLM_ENOMEM, "status word: cudaMalloc failed");
      return nullptr;
    }
  }
  return words[dev & 63];
}

int grid_for(int n, int threads) {
  const int want = (int)cdiv((unsigned)n, (unsigned)threads);
  const int most = pllm_num_sms() * 8;
  return want < 1 ? 1 : (want > most ? most : want);
}

}  // namespace

// ---- C-ABI (the reference's kernel names and argument order; addresses are device pointers)

// quantize.ts:124: bias 0, int8 in -127..127 (qmax 127); bias 64, 1..127 meaning q - 64 (qmax 63)
PLLM_API void quantize_x(uint64_t xq, uint64_t xs, uint64_t x, int32_t n, int32_t bias) {
  PLLM_REQUIRE(n >= 0 && n % 32 == 0, "quantize_x: n = %d is not whole groups of 32", n);
  PLLM_REQUIRE(bias == 0 || bias == 64, "quantize_x: bias %d is neither 0 nor 64", bias);
  if (n == 0) return;
  PLLM_REQUIRE(xq && xs && x, "quantize_x: null address");
  const int groups = n / 32;
  quantize_x_kernel<<<dim3(cdiv(groups, 8), 1), 256, 0, pllm_stream()>>>(dptr<uint8_t>(xq), dptr<float>(xs),
                                                                      dptr<const float>(x), n, bias, n);
  PLLM_LAUNCHED("quantize_x");
}

// count tokens a frame apart (floats for x, bytes for xq, frame / 32 floats for xs): a prompt's activations in one call
PLLM_API void pllm_quantize_tokens(uint64_t xq, uint64_t xs, uint64_t x, int32_t n, int32_t bias, int32_t count) {
  PLLM_REQUIRE(n > 0 && n % 32 == 0 && count > 0, "pllm_quantize_tokens: bad n %d or count %d", n, count);
  PLLM_REQUIRE(bias == 0 || bias == 64, "pllm_quantize_tokens: bias %d", bias);
  quantize_x_kernel<<<dim3(cdiv(n / 32, 8), count), 256, 0, pllm_stream()>>>(dptr<uint8_t>(xq), dptr<float>(xs),
                                                                           dptr<const float>(x), n, bias, n);
  PLLM_LAUNCHED("pllm_quantize_tokens");
}

PLLM_API void interleave(uint64_t xq, uint64_t xs, int32_t n) {
  PLLM_REQUIRE(n >= 0 && n % 64 == 0, "interleave: n = %d is not whole blocks of 64", n);
  if (n == 0) return;
  interleave_kernel<<<cdiv(n / 64, 8), 256, 0, pllm_stream()>>>(dptr<uint8_t>(xq), dptr<float>(xs), n);
  PLLM_LAUNCHED("interleave");
}

PLLM_API void int8_sums(uint64_t out, uint64_t w, int32_t groups) {
  PLLM_REQUIRE(groups >= 0, "int8_sums: groups %d", groups);
  if (!groups) return;
  int8_sums_kernel<<<cdiv(groups, 256), 256, 0, pllm_stream()>>>(dptr<int32_t>(out), dptr<const int8_t>(w), groups);
  PLLM_LAUNCHED("int8_sums");
}

PLLM_API void six_sums(uint64_t out, uint64_t w, int32_t groups) {
  PLLM_REQUIRE(groups >= 0, "six_sums: groups %d", groups);
  if (!groups) return;
  six_sums_kernel<<<cdiv(groups, 256), 256, 0, pllm_stream()>>>(dptr<int32_t>(out), dptr<const uint8_t>(w), groups);
  PLLM_LAUNCHED("six_sums");
}

// halves.ts:35: returns how many of the n were not finite (a synchronous call: it waits for the stream)
PLLM_API int32_t to_f16(uint64_t out, uint64_t x, int32_t n) {
  PLLM_REQUIRE_RET(n >= 0, -1, "to_f16: n %d", n);
  if (!n) return 0;
  std::lock_guard<std::mutex> hold(pllm_scratch_lock());  // one status word a device: one call at a time
  int* bad = status_word();
  if (!bad) return -1;
  cudaMemsetAsync(bad, 0, sizeof(int), pllm_stream());
  to_f16_kernel<<<grid_for(n, 256), 256, 0, pllm_stream()>>>(dptr<uint16_t>(out), dptr<const float>(x), n, bad);
  PLLM_LAUNCHED("to_f16");
  int host = 0;
  cudaMemcpyAsync(&host, bad, sizeof(int), cudaMemcpyDeviceToHost, pllm_stream());
  if (cudaStreamSynchronize(pllm_stream()) != cudaSuccess) {
    pllm_fail(PLLM_ECUDA, "to_f16: stream failed");
    return -1;
  }
  return host;
}

// the same without waiting: the count is added to the int32 at bad (device memory), which may be 0 (not counted)
PLLM_API void pllm_to_f16_async(uint64_t out, uint64_t x, int32_t n, uint64_t bad) {
  PLLM_REQUIRE(n >= 0, "pllm_to_f16_async: n %d", n);
  if (!n) return;
  int* counter = bad ? dptr<int>(bad) : status_word();
  to_f16_kernel<<<grid_for(n, 256), 256, 0, pllm_stream()>>>(dptr<uint16_t>(out), dptr<const float>(x), n, counter);
  PLLM_LAUNCHED("pllm_to_f16_async");
}

PLLM_API void from_f16(uint64_t out, uint64_t x, int32_t n) {
  PLLM_REQUIRE(n >= 0, "from_f16: n %d", n);
  if (!n) return;
  from_f16_kernel<<<grid_for(n, 256), 256, 0, pllm_stream()>>>(dptr<float>(out), dptr<const uint16_t>(x), n);
  PLLM_LAUNCHED("from_f16");
}

// halves.ts:82: 1 where all n halves are finite, else 0 (synchronous)
PLLM_API int32_t finite_f16(uint64_t x, int32_t n) {
  PLLM_REQUIRE_RET(n >= 0, -1, "finite_f16: n %d", n);
  if (!n) return 1;
  std::lock_guard<std::mutex> hold(pllm_scratch_lock());
  int* found = status_word();
  if (!found) return -1;
  cudaMemsetAsync(found, 0, sizeof(int), pllm_stream());
  finite_f16_kernel<<<grid_for(n, 256), 256, 0, pllm_stream()>>>(dptr<const uint16_t>(x), n, found);
  PLLM_LAUNCHED("finite_f16");
  int host = 0;
  cudaMemcpyAsync(&host, found, sizeof(int), cudaMemcpyDeviceToHost, pllm_stream());
  if (cudaStreamSynchronize(pllm_stream()) != cudaSuccess) {
    pllm_fail(PLLM_ECUDA, "finite_f16: stream failed");
    return -1;
  }
  return host ? 0 : 1;
}
