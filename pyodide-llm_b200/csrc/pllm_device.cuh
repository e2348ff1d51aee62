// pllm_device.cuh: device functions shared by the quantizer, the products and the debug sums. Every integer here is
// exact; the packings are the reference's (kernels/six.ts, kernels/ternary.ts, kernels/binary.ts,
// src/python/engine/packing.py).
#pragma once
#include "pllm_common.cuh"

// quantize.ts:8-19 + :124-151 for one group of 32 held one value a lane: the largest |x| of each of the four
// SIMD lanes (element j is in lane j % 4; a NaN there makes that lane NaN), the four compared in order, scale =
// amax / qmax, and the lane's int8. Returns the lane's byte; *scale gets the group's scale.
__device__ __forceinline__ int8_t quantize_group_warp(float v, int lane, int bias, float* scale) {
  float a = fabsf(v);
  a = wasm_max(a, __shfl_xor_sync(0xffffffffu, a, 4));
  a = wasm_max(a, __shfl_xor_sync(0xffffffffu, a, 8));
  a = wasm_max(a, __shfl_xor_sync(0xffffffffu, a, 16));
  const float m0 = __shfl_sync(0xffffffffu, a, 0), m1 = __shfl_sync(0xffffffffu, a, 1);
  const float m2 = __shfl_sync(0xffffffffu, a, 2), m3 = __shfl_sync(0xffffffffu, a, 3);
  float amax = m0;
  if (m1 > amax) amax = m1;
  if (m2 > amax) amax = m2;
  if (m3 > amax) amax = m3;
  const float s = __fdiv_rn(amax, bias == 0 ? 127.0f : 63.0f);
  *scale = s;
  const float inv = s > 0.0f ? __fdiv_rn(1.0f, s) : 0.0f;
  (void)lane;
  return quantize_one(v, inv, bias);
}

// six.ts:16-31 / packing.py:56-63: a group's 24 bytes (8-byte aligned) widened to its 32 int8 values (4 v), as eight
// little-endian words. Value v < 16: low nibble of byte v; v >= 16: high nibble of byte v - 16; its top two bits
// are bits 2 (v / 8) of byte 16 + v % 8.
__device__ __forceinline__ void widen6_regs(uint32_t l0, uint32_t l1, uint32_t l2, uint32_t l3, uint32_t t0,
                                            uint32_t t1, uint32_t w[8]) {
  const uint32_t N = 0x0F0F0F0Fu, T = 0x03030303u;
  w[0] = ((l0 & N) << 2) | ((t0 & T) << 6);
  w[1] = ((l1 & N) << 2) | ((t1 & T) << 6);
  w[2] = ((l2 & N) << 2) | (((t0 >> 2) & T) << 6);
  w[3] = ((l3 & N) << 2) | (((t1 >> 2) & T) << 6);
  w[4] = (((l0 >> 4) & N) << 2) | (((t0 >> 4) & T) << 6);
  w[5] = (((l1 >> 4) & N) << 2) | (((t1 >> 4) & T) << 6);
  w[6] = (((l2 >> 4) & N) << 2) | (((t0 >> 6) & T) << 6);
  w[7] = (((l3 >> 4) & N) << 2) | (((t1 >> 6) & T) << 6);
}
__device__ __forceinline__ void widen6_words(const uint8_t* p, uint32_t w[8]) {
  const uint2 a = *reinterpret_cast<const uint2*>(p), b = *reinterpret_cast<const uint2*>(p + 8),
              c = *reinterpret_cast<const uint2*>(p + 16);
  widen6_regs(a.x, a.y, b.x, b.y, c.x, c.y, w);
}

// the exact int32 of a group of 32: eight dp4a of the weights' words against the activations' (signed int8)
__device__ __forceinline__ int dot32_words(const uint32_t w[8], const int4 a0, const int4 a1) {
  int s = __dp4a((int)w[0], a0.x, 0);
  s = __dp4a((int)w[1], a0.y, s);
  s = __dp4a((int)w[2], a0.z, s);
  s = __dp4a((int)w[3], a0.w, s);
  s = __dp4a((int)w[4], a1.x, s);
  s = __dp4a((int)w[5], a1.y, s);
  s = __dp4a((int)w[6], a1.z, s);
  return __dp4a((int)w[7], a1.w, s);
}

// ternary.ts:25-27 and matmul.ts:106-128: a group of 128 ternary weights (eight words: byte c of the 16 bytes of
// block h holds the codes of weights 64 h + 4 c + p at bits 2 p) against the 128 interleaved activations of the group
// (32 words: byte 16 p + c of block h is activation 64 h + 4 c + p). acc[s] += the code-weighted sum of the s-th 32
// activations (the + 1 of the codes is taken out by the caller with the interleave's minus-sums).
__device__ __forceinline__ void ternary_group(const uint32_t w[8], const int4* act, int acc[4]) {
#pragma unroll
  for (int h = 0; h < 2; h++) {
#pragma unroll
    for (int p = 0; p < 4; p++) {
      const int4 a = act[4 * h + p];  // bytes 64 h + 16 p .. +16: plane p of block h
      const uint32_t sh = 2 * p;
      acc[2 * h] = __dp4a((int)((w[4 * h + 0] >> sh) & 0x03030303u), a.x, acc[2 * h]);
      acc[2 * h] = __dp4a((int)((w[4 * h + 1] >> sh) & 0x03030303u), a.y, acc[2 * h]);
      acc[2 * h + 1] = __dp4a((int)((w[4 * h + 2] >> sh) & 0x03030303u), a.z, acc[2 * h + 1]);
      acc[2 * h + 1] = __dp4a((int)((w[4 * h + 3] >> sh) & 0x03030303u), a.w, acc[2 * h + 1]);
    }
  }
}

// binary.ts:20-22: a group of 128 binary weights (four words: bit 4 h + p of byte c is weight 64 h + 4 c + p, set for
// +1, whose code is 2) against the interleaved activations, as ternary_group
__device__ __forceinline__ void binary_group(const uint32_t w[4], const int4* act, int acc[4]) {
#pragma unroll
  for (int h = 0; h < 2; h++) {
#pragma unroll
    for (int p = 0; p < 4; p++) {
      const int4 a = act[4 * h + p];
      const uint32_t sh = 4 * h + p;
      acc[2 * h] = __dp4a((int)(((w[0] >> sh) & 0x01010101u) << 1), a.x, acc[2 * h]);
      acc[2 * h] = __dp4a((int)(((w[1] >> sh) & 0x01010101u) << 1), a.y, acc[2 * h]);
      acc[2 * h + 1] = __dp4a((int)(((w[2] >> sh) & 0x01010101u) << 1), a.z, acc[2 * h + 1]);
      acc[2 * h + 1] = __dp4a((int)(((w[3] >> sh) & 0x01010101u) << 1), a.w, acc[2 * h + 1]);
    }
  }
}

// streaming loads of weights: read once, not kept in L1
__device__ __forceinline__ int4 ldg_stream(const void* p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// 32 bytes in one 256-bit load (sm_100): the address must be 32-byte aligned
__device__ __forceinline__ void ldg_stream32(const void* p, uint32_t w[8]) {
  asm volatile("ld.global.nc.L1::no_allocate.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]), "=r"(w[6]), "=r"(w[7])
               : "l"(p));
}
__device__ __forceinline__ uint2 ldg_stream8(const void* p) {
  uint2 v;
  asm volatile("ld.global.nc.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}
