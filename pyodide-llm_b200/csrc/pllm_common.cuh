// pllm_common.cuh: what every translation unit of libpllm.so shares -- the sticky error word, the current stream,
// launch checks, and the device helpers whose arithmetic must match the reference's to the bit (float16 widening and
// narrowing, the int8 quantizer's rounding).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stdio.h>
#include <mutex>
#include "pllm.h"  // the declarations every definition must match

#define PLLM_API extern "C" __attribute__((visibility("default")))

// ---- the sticky error (pllm_last_error): the first failure since the last pllm_clear_error is kept
void pllm_fail(int code, const char* fmt, ...);
int pllm_failed();
cudaStream_t pllm_stream();  // the calling host thread's current stream (pllm_set_stream)
int pllm_num_sms();
// the library's host-side state is shared by every host thread: lookups that fill a per-device cache hold
// pllm_lookup_lock; the calls that wait for a result in the library's own device scratch (argmax, sample, to_f16,
// finite_f16) hold pllm_scratch_lock from their launch to their result
std::mutex& pllm_lookup_lock();
std::mutex& pllm_scratch_lock();

enum PllmError {
  PLLM_OK = 0,
  PLLM_EINVAL = 1,     // an argument the reference's kernel would not take (n % 32, r0 > r1, null address, ...)
  PLLM_ECUDA = 2,      // a CUDA call or launch failed
  PLLM_ETIMEOUT = 3,   // a bounded device-side wait gave up
  PLLM_ENOMEM = 4,
  PLLM_ERANGE = 5,     // a position read from device memory lay outside the cache (held at its edge)
};

// check the launch that was just enqueued
#define PLLM_LAUNCHED(name)                                                              \
  do {                                                                                   \
    cudaError_t e_ = cudaGetLastError();                                                 \
    if (e_ != cudaSuccess) pllm_fail(PLLM_ECUDA, "%s: launch failed: %s", name, cudaGetErrorString(e_)); \
  } while (0)

#define PLLM_REQUIRE(cond, ...)                 \
  do {                                          \
    if (!(cond)) {                              \
      pllm_fail(PLLM_EINVAL, __VA_ARGS__);      \
      return;                                   \
    }                                           \
  } while (0)

#define PLLM_REQUIRE_RET(cond, ret, ...)        \
  do {                                          \
    if (!(cond)) {                              \
      pllm_fail(PLLM_EINVAL, __VA_ARGS__);      \
      return ret;                               \
    }                                           \
  } while (0)

template <typename T>
static inline T* dptr(uint64_t a) { return reinterpret_cast<T*>(static_cast<uintptr_t>(a)); }

static inline unsigned cdiv(unsigned a, unsigned b) { return (a + b - 1) / b; }

// Programmatic dependent launch: a kernel launched with the attribute may begin before the one ahead of it in the
// stream has finished; it must wait (griddepcontrol.wait) before reading what that kernel wrote. Without the
// attribute both instructions are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---- float16 as the reference reads and writes it (kernels/kernel/halves.ts)
// halves.ts:12-23: the half's 16 bits sign-extended, shifted up by 13, the copies of the sign cleared, times 2^112.
// Exact for every finite half; an infinity reads as 65536 and a NaN is not kept.
__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
  const int s = (int)(int16_t)h;
  return __int_as_float((s << 13) & (int)0x8fffffff) * 5.192296858534828e33f;
}

// halves.ts:35-67: float32 to float16 bits, round to nearest even, too large to an infinity (a NaN too, counted as
// not finite by *bad)
__device__ __forceinline__ uint16_t float_to_half_bits(float x, int* bad) {
  const uint32_t bits = __float_as_uint(x);
  const uint32_t sign = (bits >> 16) & 0x8000u;
  const int exponent = (int)((bits >> 23) & 0xff) - 112;
  uint32_t mantissa = bits & 0x7fffffu, result;
  if (exponent >= 31) {
    result = sign | 0x7c00u;
    if (exponent == 143) ++*bad;
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
  return (uint16_t)result;
}

// WASM's f32 max: a NaN in either operand is NaN (CUDA's fmaxf drops a NaN)
__device__ __forceinline__ float wasm_max(float a, float b) {
  return (a != a || b != b) ? __int_as_float(0x7fc00000) : fmaxf(a, b);
}

// quantize.ts:141-149 for one value: round half to even, to int32 with saturation (a NaN is 0), the bias added in
// int32 (wrapping), narrowed to int8 with saturation. cvt.rni.s32.f32 is rint then the saturating conversion.
__device__ __forceinline__ int8_t quantize_one(float x, float inv, int bias) {
  const int q = __float2int_rn(__fmul_rn(x, inv));
  const int w = (int)((unsigned)q + (unsigned)bias);
  return (int8_t)(w < -128 ? -128 : (w > 127 ? 127 : w));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
