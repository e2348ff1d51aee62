// blocks.cu: llama.cpp's blocks of 256 weights ("super-blocks", kernels/blocks/*.ts): the ten types the reference's
// block kernels multiply (Q2_K 10, Q4_K 12, IQ2_XXS 16, IQ2_XS 17, IQ3_XXS 18, IQ1_S 19, IQ3_S 21, IQ2_S 22,
// IQ4_XS 23, IQ1_M 29: the type's number in a GGUF), kept packed as the checkpoint holds them.
//
// The arithmetic is the reference's (kernels/blocks/types.ts:66-83): a weight is F S W - Fm M, F of its block, S an
// integer of its unit (16 or 32 weights), W a small integer, M (the K types) a minimum of its unit. For each block and
// each of its eight groups k of 32 activations (int8 and a float32 scale each, quantize_x(.., 0)):
//   G[k] = sum over the group of S W a          (an exact integer: int32 here, in any order)
//   M[k] = sum over the group's units of m (the sum of the unit's activations)
//   lane k & 3 += ((G[k] xs[k] + G[k + 4] xs[k + 4]) F) - ((M[k] xs[k] + M[k + 4] xs[k + 4]) Fm)
// and the row is the four lanes added in order. G and M are the reference's to the bit; the lanes here add the blocks
// in another order (a lane of a warp a block, the warp's sums at the end), so a row is within float32 rounding of it.
//
// A warp a row, a lane a block at a time. The tables (sb_tables: the checkpoint's codebooks as grids, the 7-bit signs'
// table, IQ4_XS's values) sit in shared memory, 34,992 bytes, with the token's activations and scales. A unit of 16
// weights is read as 16 signed bytes W (IQ1: 8 g + 1, or 8 g - 1 where its shift is down) and multiplied with dp4a.
#include "pllm_common.cuh"

namespace {

constexpr int T_IQ2XS = 2048, T_IQ2S = 6144, T_IQ3XXS = 14336, T_IQ3S = 15360, T_IQ1S = 17408;
constexpr int T_SIGNS = 33792, T_IQ4 = 34816, T_VECTORS = 34864, GRIDS = 33792, TABLES = 34992;
constexpr int SB_WARPS = 8;

__host__ __device__ constexpr int block_bytes(int type) {
  return type == 10 ? 84 : type == 12 ? 144 : type == 16 ? 66 : type == 17 ? 74 : type == 18 ? 98 : type == 19 ? 50 :
         type == 21 ? 110 : type == 22 ? 82 : type == 23 ? 136 : type == 29 ? 56 : 0;
}

__device__ __forceinline__ uint32_t u16at(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }
__device__ __forceinline__ uint32_t u32at(const uint8_t* p) { return u16at(p) | (u16at(p + 2) << 16); }
__device__ __forceinline__ float half_at(const uint8_t* p) { return half_bits_to_float((uint16_t)u16at(p)); }

// 8 magnitudes of a grid entry with the signs of a 7-bit index (the table's eighth sign keeps the minuses even), into
// W[o..o+8)
__device__ __forceinline__ void signed8(int* W, int o, const uint8_t* entry, const uint8_t* tab, uint32_t idx7) {
  const uint8_t* minus = tab + T_SIGNS + (idx7 & 127) * 8;
#pragma unroll
  for (int j = 0; j < 8; j++) W[o + j] = minus[j] ? -(int)entry[j] : (int)entry[j];
}

// unit u (16 weights) of the block at p (global memory), with the tables at tab (shared memory): W, S and m
template <int TYPE>
__device__ __forceinline__ void unit_of(const uint8_t* p, int u, const uint8_t* tab, int* W, int& S, int& m) {
  const int g = u >> 1;
  m = 0;
  if constexpr (TYPE == 10) {  // Q2_K: bits 2 s, 2 s + 1 of byte b of a half's 32 are weight 32 s + b of the half
    const uint8_t* q = p + 16 + 32 * (u >> 3) + 16 * (u & 1);
    const int sh = 2 * ((u & 7) >> 1);
#pragma unroll
    for (int j = 0; j < 16; j++) W[j] = (q[j] >> sh) & 3;
    S = p[u] & 15;
    m = p[u] >> 4;
  } else if constexpr (TYPE == 12) {  // Q4_K: of every 32 bytes the low halves are 32 weights, the high the next 32
    const uint8_t* q = p + 16 + 32 * (g >> 1) + 16 * (u & 1);
    const int sh = 4 * (g & 1);
#pragma unroll
    for (int j = 0; j < 16; j++) W[j] = (q[j] >> sh) & 15;
    const uint8_t* sc = p + 4;
    S = g < 4 ? sc[g] & 63 : (sc[g + 4] & 15) | ((sc[g - 4] >> 6) << 4);
    m = g < 4 ? sc[g + 4] & 63 : (sc[g + 4] >> 4) | ((sc[g] >> 6) << 4);
  } else if constexpr (TYPE == 23) {  // IQ4_XS: a group's 16 bytes, low halves its first 16 weights
    const uint8_t* q = p + 8 + 16 * g;
    const int sh = 4 * (u & 1);
#pragma unroll
    for (int j = 0; j < 16; j++) W[j] = (int)(int8_t)tab[T_IQ4 + ((q[j] >> sh) & 15)];
    S = (int)(((p[4 + (g >> 1)] >> (4 * (g & 1))) & 15) | (((u16at(p + 2) >> (2 * g)) & 3) << 4)) - 32;
  } else if constexpr (TYPE == 16) {  // IQ2_XXS
    const uint8_t* q = p + 2 + 8 * g;
    const uint32_t aux = u32at(q + 4), sh = 14 * (u & 1);
    signed8(W, 0, tab + q[2 * (u & 1)] * 8, tab, aux >> sh);
    signed8(W, 8, tab + q[2 * (u & 1) + 1] * 8, tab, aux >> (sh + 7));
    S = (int)(2 * (aux >> 28) + 1);
  } else if constexpr (TYPE == 17) {  // IQ2_XS: a word for 8 weights, 9 bits of index, 7 of signs
    const uint32_t q0 = u16at(p + 2 + 4 * u), q1 = u16at(p + 4 + 4 * u);
    signed8(W, 0, tab + T_IQ2XS + (q0 & 511) * 8, tab, q0 >> 9);
    signed8(W, 8, tab + T_IQ2XS + (q1 & 511) * 8, tab, q1 >> 9);
    S = (int)(2 * ((p[66 + g] >> (4 * (u & 1))) & 15) + 1);
  } else if constexpr (TYPE == 22) {  // IQ2_S: 10-bit indices, a byte of signs for each 8
    const uint32_t hi = p[66 + g] >> (4 * (u & 1)), signs = u16at(p + 34 + 2 * u);
    const uint8_t* e0 = tab + T_IQ2S + (p[2 + 2 * u] | ((hi & 3) << 8)) * 8;
    const uint8_t* e1 = tab + T_IQ2S + (p[3 + 2 * u] | ((hi & 12) << 6)) * 8;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      W[j] = ((signs >> j) & 1) ? -(int)e0[j] : (int)e0[j];
      W[8 + j] = ((signs >> (8 + j)) & 1) ? -(int)e1[j] : (int)e1[j];
    }
    S = (int)(2 * ((p[74 + g] >> (4 * (u & 1))) & 15) + 1);
  } else if constexpr (TYPE == 18) {  // IQ3_XXS: a byte an index of 4; a word a group, its signs and s
    const uint32_t aux = u32at(p + 66 + 4 * g), sh = 14 * (u & 1);
    const uint8_t* m0 = tab + T_SIGNS + ((aux >> sh) & 127) * 8;
    const uint8_t* m1 = tab + T_SIGNS + ((aux >> (sh + 7)) & 127) * 8;
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const uint8_t* e = tab + T_IQ3XXS + p[2 + 4 * u + i] * 4;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int w = 4 * i + j;
        const bool neg = (w < 8 ? m0[w] : m1[w - 8]) != 0;
        W[w] = neg ? -(int)e[j] : (int)e[j];
      }
    }
    S = (int)(2 * (aux >> 28) + 1);
  } else if constexpr (TYPE == 21) {  // IQ3_S: 9-bit indices, 16 bits of signs
    const uint32_t hi = p[66 + g] >> (4 * (u & 1)), signs = u16at(p + 74 + 2 * u);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const uint8_t* e = tab + T_IQ3S + (p[2 + 4 * u + i] | (((hi >> i) & 1) << 8)) * 4;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int w = 4 * i + j;
        W[w] = ((signs >> w) & 1) ? -(int)e[j] : (int)e[j];
      }
    }
    S = (int)(2 * ((p[106 + (u >> 2)] >> (4 * ((u >> 1) & 1))) & 15) + 1);
  } else if constexpr (TYPE == 19) {  // IQ1_S: 11-bit indices into codes 0, 1, 2; the group's word's top bit: down
    const uint32_t qh = u16at(p + 34 + 2 * g), hi = qh >> (6 * (u & 1));
    const int shift = (qh >> 15) ? -1 : 1;
    const uint8_t* e0 = tab + T_IQ1S + (p[2 + 2 * u] | ((hi & 7) << 8)) * 8;
    const uint8_t* e1 = tab + T_IQ1S + (p[3 + 2 * u] | ((hi & 56) << 5)) * 8;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      W[j] = 8 * ((int)e0[j] - 1) + shift;
      W[8 + j] = 8 * ((int)e1[j] - 1) + shift;
    }
    S = (int)(2 * ((qh >> 12) & 7) + 1);
  } else if constexpr (TYPE == 29) {  // IQ1_M: a byte of qh a unit, the shifts' signs at bits 3 and 7
    const uint32_t hq = p[32 + u];
    const uint8_t* e0 = tab + T_IQ1S + (p[2 * u] | ((hq & 7) << 8)) * 8;
    const uint8_t* e1 = tab + T_IQ1S + (p[2 * u + 1] | ((hq & 0x70) << 4)) * 8;
    const int s0 = ((hq >> 3) & 1) ? -1 : 1, s1 = (hq >> 7) ? -1 : 1;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      W[j] = 8 * ((int)e0[j] - 1) + s0;
      W[8 + j] = 8 * ((int)e1[j] - 1) + s1;
    }
    S = (int)(2 * ((u16at(p + 48 + 2 * (u >> 2)) >> (3 * (u & 3))) & 7) + 1);
  }
}

// IQ1_M's d: the top four bits of its four scale words (the first word's the lowest)
__device__ __forceinline__ float whole_d(const uint8_t* p) {
  const uint32_t w0 = u16at(p + 48), w1 = u16at(p + 50), w2 = u16at(p + 52), w3 = u16at(p + 54);
  return half_bits_to_float((uint16_t)((w0 >> 12) | ((w1 >> 8) & 0xf0) | ((w2 >> 4) & 0xf00) | (w3 & 0xf000)));
}
template <int TYPE>
__device__ __forceinline__ float block_F(const uint8_t* p) {
  if constexpr (TYPE == 16 || TYPE == 17 || TYPE == 22 || TYPE == 19) return half_at(p) * 0.125f;
  if constexpr (TYPE == 18) return half_at(p) * 0.25f;
  if constexpr (TYPE == 29) return whole_d(p) * 0.125f;
  if constexpr (TYPE == 10) return half_at(p + 80);
  return half_at(p);
}
template <int TYPE>
__device__ __forceinline__ float block_Fm(const uint8_t* p) {
  return TYPE == 10 ? half_at(p + 82) : half_at(p + 2);
}

__device__ __forceinline__ int pack4(const int* W) {
  return (int)((W[0] & 255) | ((W[1] & 255) << 8) | ((W[2] & 255) << 16) | ((unsigned)(W[3] & 255) << 24));
}

// The products: grid (row CTAs, tokens); a warp a row; the token's activations and the tables in shared memory
template <int TYPE>
__global__ void __launch_bounds__(SB_WARPS * 32) sb_kernel(float* out, const int8_t* xq, const float* xs,
                                                            const uint8_t* w, const uint8_t* tabg, int n, int r0, int r1,
                                                            long long os, long long frame) {
  extern __shared__ __align__(16) uint8_t sb_smem[];
  uint8_t* tab = sb_smem;                                           // TABLES bytes
  int8_t* sx = reinterpret_cast<int8_t*>(sb_smem + ((TABLES + 15) & ~15));  // n activations
  float* ss = reinterpret_cast<float*>(sx + n);                     // n / 32 scales
  const int t = blockIdx.y;
  const int8_t* xt = reinterpret_cast<const int8_t*>(reinterpret_cast<const uint8_t*>(xq) + t * frame);
  const float* st = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(xs) + t * frame);
  for (int i = threadIdx.x; i < TABLES; i += blockDim.x) tab[i] = tabg[i];
  for (int i = threadIdx.x; i < n / 4; i += blockDim.x) reinterpret_cast<int*>(sx)[i] = reinterpret_cast<const int*>(xt)[i];
  for (int i = threadIdx.x; i < n / 32; i += blockDim.x) ss[i] = st[i];
  __syncthreads();
  constexpr int SIZE = block_bytes(TYPE);
  constexpr bool KQ = TYPE == 10 || TYPE == 12;
  const int blocks = n / 256, lane = threadIdx.x & 31;
  float* o = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(out) + t * os);
  for (int row = r0 + blockIdx.x * SB_WARPS + (threadIdx.x >> 5); row < r1; row += gridDim.x * SB_WARPS) {
    const uint8_t* wr = w + (size_t)row * blocks * SIZE;
    float facc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int b = lane; b < blocks; b += 32) {
      const uint8_t* p = wr + (size_t)b * SIZE;
      const int8_t* x = sx + 256 * b;
      int G[8], M[8];
#pragma unroll
      for (int k = 0; k < 8; k++) G[k] = M[k] = 0;
#pragma unroll 1
      for (int u = 0; u < 16; u++) {
        int W[16], S, m;
        unit_of<TYPE>(p, u, tab, W, S, m);
        const int* xa = reinterpret_cast<const int*>(x + 16 * u);
        int d = 0, s16 = 0;
#pragma unroll
        for (int q = 0; q < 4; q++) {
          d = __dp4a(pack4(W + 4 * q), xa[q], d);
          if (KQ) s16 = __dp4a(0x01010101, xa[q], s16);
        }
        G[u >> 1] += S * d;
        if (KQ) M[u >> 1] += m * s16;
      }
      const float* s = ss + 8 * b;
      const float F = block_F<TYPE>(p);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        float part = __fmul_rn(__fadd_rn(__fmul_rn((float)G[j], s[j]), __fmul_rn((float)G[j + 4], s[j + 4])), F);
        if (KQ)
          part = __fsub_rn(part, __fmul_rn(__fadd_rn(__fmul_rn((float)M[j], s[j]), __fmul_rn((float)M[j + 4], s[j + 4])),
                                           block_Fm<TYPE>(p)));
        facc[j] = __fadd_rn(facc[j], part);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; j++) facc[j] = warp_sum(facc[j]);
    if (lane == 0) o[row] = ((facc[0] + facc[1]) + facc[2]) + facc[3];
  }
}

// sb_row: a row as float32, each weight as the reference's reader makes it (row.ts: the unit's float scale times W,
// IQ1 the grid's value +- 1/8, less Fm m for the K types); a thread a unit
template <int TYPE>
__global__ void sb_row_kernel(float* out, const uint8_t* w, const uint8_t* tabg, int n) {
  __shared__ uint8_t tab[TABLES];
  for (int i = threadIdx.x; i < TABLES; i += blockDim.x) tab[i] = tabg[i];
  __syncthreads();
  constexpr int SIZE = block_bytes(TYPE);
  const int units = n / 16;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < units; e += gridDim.x * blockDim.x) {
    const int b = e >> 4, u = e & 15;
    const uint8_t* p = w + (size_t)b * SIZE;
    int W[16], S, m;
    unit_of<TYPE>(p, u, tab, W, S, m);
    const float s = (float)(S >> 1);
    float scale;
    if constexpr (TYPE == 16 || TYPE == 17 || TYPE == 22) scale = __fmul_rn(__fmul_rn(half_at(p), 0.5f + s), 0.25f);
    else if constexpr (TYPE == 18) scale = __fmul_rn(__fmul_rn(half_at(p), 0.5f + s), 0.5f);
    else if constexpr (TYPE == 29) scale = __fmul_rn(whole_d(p), (float)S);
    else if constexpr (TYPE == 10) scale = __fmul_rn(half_at(p + 80), (float)S);
    else scale = __fmul_rn(half_at(p), (float)S);
#pragma unroll
    for (int j = 0; j < 16; j++) {
      float v;
      if constexpr (TYPE == 19 || TYPE == 29) {
        const int shift = ((W[j] & 7) == 1) ? 1 : -1;  // 8 g + 1 is 1 mod 8, 8 g - 1 is 7
        v = __fadd_rn((float)((W[j] - shift) / 8), shift < 0 ? -0.125f : 0.125f);
      } else {
        v = (float)W[j];
      }
      float o = __fmul_rn(scale, v);
      if constexpr (TYPE == 10 || TYPE == 12) o = __fsub_rn(o, __fmul_rn(block_Fm<TYPE>(p), (float)m));
      out[16 * e + j] = o;
    }
  }
}

__global__ void sb_tables_kernel(uint8_t* area, const uint8_t* books) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < GRIDS) area[i] = (uint8_t)(books[i] + (i >= T_IQ1S ? 1 : 0));
  if (i < 128) {
    const unsigned held = (unsigned)i | ((__popc(i) & 1u) << 7);
    for (int j = 0; j < 8; j++) area[T_SIGNS + i * 8 + j] = ((held >> j) & 1) ? 255 : 0;
  }
  if (i < 16) {
    const int8_t v = (int8_t)books[GRIDS + i];
    area[T_IQ4 + i] = (uint8_t)v;
    area[T_IQ4 + 16 + i] = (uint8_t)(v < 0 ? -v : v);
    area[T_IQ4 + 32 + i] = v < 0 ? 255 : 0;
    uint8_t* vec = area + T_VECTORS;
    vec[i] = (uint8_t)(1u << (i & 7));
    vec[16 + i] = (uint8_t)(i >> 3);
    vec[32 + i] = 3;
    vec[48 + i] = 15;
    vec[80 + i] = 7;
    vec[96 + i] = 1;
    if (i < 4) {
      const int p3 = 512 >> (i * 3), p4 = 4096 >> (i * 4);
      for (int k = 0; k < 4; k++) {
        vec[64 + 4 * i + k] = (uint8_t)(p3 >> (8 * k));
        vec[112 + 4 * i + k] = (uint8_t)(p4 >> (8 * k));
      }
    }
  }
}

__global__ void sums_x_kernel(float* xs, const int8_t* xq, int n) {
  int16_t* s16 = reinterpret_cast<int16_t*>(xs + n / 32);
  int16_t* s8 = s16 + n / 16;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n / 8; i += gridDim.x * blockDim.x) {
    const int2 v = reinterpret_cast<const int2*>(xq)[i];
    const int s = __dp4a(v.x, 0x01010101, 0) + __dp4a(v.y, 0x01010101, 0);
    s8[i] = (int16_t)s;
    if ((i & 1) == 0) {
      const int2 u = reinterpret_cast<const int2*>(xq)[i + 1];
      s16[i >> 1] = (int16_t)(s + __dp4a(u.x, 0x01010101, 0) + __dp4a(u.y, 0x01010101, 0));
    }
  }
}

// The same products with a row's blocks staged in shared memory: a warp takes two rows (half a warp a row, a lane
// its blocks hl, hl + 16, ...), copies both rows' bytes with 16-byte loads (4-byte where the rows are not 16-byte
// aligned) into its own buffer, then decodes from there; every block's integers and its float32 part as sb_kernel's,
// the lanes' parts added in another order (a lane 16 apart, a half-warp's reduction). (sb_kernel read each block's
// fields from global memory one at a time, 50 to 144 bytes from its neighbour lane's, with half the lanes idle at K
// 4096: 2 % of the copy rate.)
template <int TYPE>
__global__ void __launch_bounds__(SB_WARPS * 32) sb_staged_kernel(float* out, const int8_t* xq, const float* xs,
                                                                   const uint8_t* w, const uint8_t* tabg, int n, int r0,
                                                                   int r1, long long os, long long frame) {
  extern __shared__ __align__(16) uint8_t sb_smem[];
  constexpr int SIZE = block_bytes(TYPE);
  constexpr bool KQ = TYPE == 10 || TYPE == 12;
  const int blocks = n / 256, rowbytes = blocks * SIZE;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, half = lane >> 4, hl = lane & 15;
  uint8_t* tab = sb_smem;                                                   // TABLES bytes
  int8_t* sx = reinterpret_cast<int8_t*>(sb_smem + ((TABLES + 15) & ~15));  // n activations
  float* ss = reinterpret_cast<float*>(sx + n);                             // n / 32 scales
  uint8_t* wbuf = reinterpret_cast<uint8_t*>(ss + n / 32) + (size_t)warp * 2 * ((rowbytes + 15) & ~15);
  const int t = blockIdx.y;
  const int8_t* xt = reinterpret_cast<const int8_t*>(reinterpret_cast<const uint8_t*>(xq) + t * frame);
  const float* st = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(xs) + t * frame);
  for (int i = threadIdx.x; i < TABLES; i += blockDim.x) tab[i] = tabg[i];
  for (int i = threadIdx.x; i < n / 4; i += blockDim.x) reinterpret_cast<int*>(sx)[i] = reinterpret_cast<const int*>(xt)[i];
  for (int i = threadIdx.x; i < n / 32; i += blockDim.x) ss[i] = st[i];
  __syncthreads();
  const int rb16 = (rowbytes + 15) & ~15;
  const bool v16 = (rowbytes & 15) == 0 && (((uintptr_t)w) & 15) == 0;
  float* o = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(out) + t * os);
  for (int pr = r0 + 2 * (blockIdx.x * SB_WARPS + warp); pr < r1; pr += 2 * gridDim.x * SB_WARPS) {
    const int nr = pr + 1 < r1 ? 2 : 1;  // rows of this pair
    __syncwarp();  // the buffer's last pair is decoded
    for (int h = 0; h < nr; h++) {
      const uint8_t* src = w + (size_t)(pr + h) * rowbytes;
      uint8_t* dst = wbuf + h * rb16;
      if (v16) {
        for (int i = lane; i < rowbytes / 16; i += 32)
          reinterpret_cast<int4*>(dst)[i] = __ldg(reinterpret_cast<const int4*>(src) + i);
      } else if ((((uintptr_t)w) & 1) == 0) {  // rows a multiple of 2 bytes (every block's size is even)
        for (int i = lane; i < rowbytes / 2; i += 32)
          reinterpret_cast<uint16_t*>(dst)[i] = __ldg(reinterpret_cast<const unsigned short*>(src) + i);
      } else {
        for (int i = lane; i < rowbytes; i += 32) dst[i] = __ldg(src + i);
      }
    }
    __syncwarp();
    const int row = pr + half;
    float facc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (half < nr) {
      const uint8_t* wr = wbuf + half * rb16;
      for (int b = hl; b < blocks; b += 16) {
        const uint8_t* p = wr + (size_t)b * SIZE;
        const int8_t* x = sx + 256 * b;
        int G[8], M[8];
#pragma unroll
        for (int k = 0; k < 8; k++) G[k] = M[k] = 0;
#pragma unroll 1
        for (int u = 0; u < 16; u++) {
          int W[16], S, m;
          unit_of<TYPE>(p, u, tab, W, S, m);
          const int* xa = reinterpret_cast<const int*>(x + 16 * u);
          int d = 0, s16 = 0;
#pragma unroll
          for (int q = 0; q < 4; q++) {
            d = __dp4a(pack4(W + 4 * q), xa[q], d);
            if (KQ) s16 = __dp4a(0x01010101, xa[q], s16);
          }
          G[u >> 1] += S * d;
          if (KQ) M[u >> 1] += m * s16;
        }
        const float* s = ss + 8 * b;
        const float F = block_F<TYPE>(p);
#pragma unroll
        for (int j = 0; j < 4; j++) {
          float part = __fmul_rn(__fadd_rn(__fmul_rn((float)G[j], s[j]), __fmul_rn((float)G[j + 4], s[j + 4])), F);
          if (KQ)
            part = __fsub_rn(part, __fmul_rn(__fadd_rn(__fmul_rn((float)M[j], s[j]), __fmul_rn((float)M[j + 4], s[j + 4])),
                                             block_Fm<TYPE>(p)));
          facc[j] = __fadd_rn(facc[j], part);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) facc[j] += __shfl_xor_sync(0xffffffffu, facc[j], off);
    if (half < nr && hl == 0) o[row] = ((facc[0] + facc[1]) + facc[2]) + facc[3];
  }
}

bool known(int type) { return block_bytes(type) != 0; }

bool launch_products(float* out, const int8_t* xq, const float* xs, const uint8_t* w, const uint8_t* tab, int n, int r0,
                     int r1, int count, long long os, long long frame, int type) {
  const size_t smem = ((TABLES + 15) & ~15) + (size_t)n + (size_t)n / 8;
  const int rows = r1 - r0;
  // the staged form where every warp's two rows fit beside the tables and the activations
  const size_t rb16 = ((size_t)(n / 256) * block_bytes(type) + 15) & ~(size_t)15;
  const size_t staged = smem + (size_t)SB_WARPS * 2 * rb16;
  if (staged <= 200 * 1024) {
    int pairs = (rows + 2 * SB_WARPS - 1) / (2 * SB_WARPS);
    const int most_s = 4 * pllm_num_sms();
    pairs = pairs > most_s ? most_s : pairs;
    const dim3 grid_s(pairs < 1 ? 1 : pairs, count);
#define SB_STAGED(T)                                                                                            \
  case T: {                                                                                                     \
    if (cudaFuncSetAttribute(sb_staged_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)staged) != \
        cudaSuccess)                                                                                            \
      return false;                                                                                             \
    sb_staged_kernel<T><<<grid_s, SB_WARPS * 32, staged, pllm_stream()>>>(out, xq, xs, w, tab, n, r0, r1, os, frame); \
    return true;                                                                                                \
  }
    switch (type) {
      SB_STAGED(10) SB_STAGED(12) SB_STAGED(16) SB_STAGED(17) SB_STAGED(18) SB_STAGED(19) SB_STAGED(21) SB_STAGED(22)
      SB_STAGED(23) SB_STAGED(29)
    }
#undef SB_STAGED
    return false;
  }
  int ctas = (rows + SB_WARPS - 1) / SB_WARPS;
  const int most = 4 * pllm_num_sms();
  ctas = ctas > most ? most : ctas;
  const dim3 grid(ctas, count);
#define SB_CASE(T)                                                                                              \
  case T: {                                                                                                     \
    if (cudaFuncSetAttribute(sb_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) \
      return false;                                                                                             \
    sb_kernel<T><<<grid, SB_WARPS * 32, smem, pllm_stream()>>>(out, xq, xs, w, tab, n, r0, r1, os, frame);      \
    return true;                                                                                                \
  }
  switch (type) {
    SB_CASE(10) SB_CASE(12) SB_CASE(16) SB_CASE(17) SB_CASE(18) SB_CASE(19) SB_CASE(21) SB_CASE(22) SB_CASE(23)
    SB_CASE(29)
  }
#undef SB_CASE
  return false;
}

void products(const char* name, uint64_t xout, uint64_t xq, uint64_t xs, uint64_t w, uint64_t tab, int32_t n, int32_t r0,
              int32_t r1, int32_t count, int32_t os, int32_t frame, int32_t type) {
  PLLM_REQUIRE(known(type) && n > 0 && n % 256 == 0 && n <= 160 * 1024 && 0 <= r0 && r0 <= r1 && count >= 1 && xout &&
                   xq && xs && w && tab && !(xq & 3) && !(xs & 3) && !(frame & 3) && (count == 1 || frame > 0),
               "%s: type %d n %d rows %d..%d count %d", name, type, n, r0, r1, count);
  if (r0 == r1) return;
  if (!launch_products(dptr<float>(xout), dptr<const int8_t>(xq), dptr<const float>(xs), dptr<const uint8_t>(w),
                       dptr<const uint8_t>(tab), n, r0, r1, count, os, frame, type))
    pllm_fail(PLLM_ECUDA, "%s: launch", name);
  PLLM_LAUNCHED(name);
}

}  // namespace

// sb_tables (blocks/types.ts:294): the kernels' tables at area (34,992 bytes) from the checkpoint's codebooks row;
// returns the bytes written (enqueued, not waited for)
PLLM_API int32_t sb_tables(uint64_t area, uint64_t codebooks) {
  PLLM_REQUIRE_RET(area && codebooks, 0, "sb_tables: null address");
  sb_tables_kernel<<<(GRIDS + 255) / 256, 256, 0, pllm_stream()>>>(dptr<uint8_t>(area), dptr<const uint8_t>(codebooks));
  PLLM_LAUNCHED("sb_tables");
  return TABLES;
}

// sums_x (blocks/token.ts:160): after the n / 32 scales at xs, the int16 sums of each 16 activations, then of each 8
PLLM_API void sums_x(uint64_t xs, uint64_t xq, int32_t n) {
  PLLM_REQUIRE(xs && xq && n > 0 && n % 32 == 0 && !(xs & 3) && !(xq & 7), "sums_x: n %d", n);
  const int threads = 256, items = n / 8;
  sums_x_kernel<<<(items + threads - 1) / threads, threads, 0, pllm_stream()>>>(dptr<float>(xs), dptr<const int8_t>(xq),
                                                                                n);
  PLLM_LAUNCHED("sums_x");
}

// matmul_sb / matmul_sbr (blocks/token.ts:133-141): one token, rows r0..r1 of n weights in blocks of type
PLLM_API void matmul_sb(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t w, uint64_t tab, int32_t n, int32_t r0,
                        int32_t r1, int32_t type) {
  products("matmul_sb", xout, xq, xs, w, tab, n, r0, r1, 1, 0, 0, type);
}
PLLM_API void matmul_sbr(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t w, uint64_t tab, int32_t n, int32_t r0,
                         int32_t r1, int32_t type) {
  products("matmul_sbr", xout, xq, xs, w, tab, n, r0, r1, 1, 0, 0, type);
}
// matmul_sbr_tile (blocks/tile.ts:149): count tokens, each's activations and xs frame bytes apart, outputs os apart
PLLM_API void matmul_sbr_tile(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t w, uint64_t tab, int32_t n, int32_t r0,
                              int32_t r1, int32_t count, int32_t os, int32_t frame, int32_t type) {
  PLLM_REQUIRE(os > 0 && !(os & 3), "matmul_sbr_tile: os %d", os);
  products("matmul_sbr_tile", xout, xq, xs, w, tab, n, r0, r1, count, os, frame, type);
}
// matmul_sbw_tile (blocks/tile.ts): the same numbers; the caller's scratch (the reference's spread row) is not needed
PLLM_API void matmul_sbw_tile(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t w, uint64_t tab, int32_t n, int32_t r0,
                              int32_t r1, int32_t count, int32_t os, int32_t frame, int32_t type, uint64_t scratch) {
  (void)scratch;
  PLLM_REQUIRE(os > 0 && !(os & 3), "matmul_sbw_tile: os %d", os);
  products("matmul_sbw_tile", xout, xq, xs, w, tab, n, r0, r1, count, os, frame, type);
}

// signed_dots (blocks/tile.ts): out[l] = the sum of a[4 l + i] b[4 l + i] over i < 4, signed bytes by signed bytes
// (the device's dp4a multiplies every signed byte by every signed byte exactly, so matmul_sbw_tile may be chosen)
__global__ void signed_dots_kernel(int* out, const int* a, const int* b) {
  if (threadIdx.x < 4) out[threadIdx.x] = __dp4a(a[threadIdx.x], b[threadIdx.x], 0);
}
PLLM_API void signed_dots(uint64_t out, uint64_t a, uint64_t b) {
  PLLM_REQUIRE(out && a && b && !(out & 3) && !(a & 3) && !(b & 3), "signed_dots: null or misaligned address");
  signed_dots_kernel<<<1, 32, 0, pllm_stream()>>>(dptr<int>(out), dptr<const int>(a), dptr<const int>(b));
  PLLM_LAUNCHED("signed_dots");
}

// sb_row (blocks/row.ts:60): n weights of the row at w as float32
PLLM_API void sb_row(uint64_t out, uint64_t w, uint64_t tab, int32_t n, int32_t type) {
  PLLM_REQUIRE(known(type) && out && w && tab && n > 0 && n % 256 == 0, "sb_row: type %d n %d", type, n);
  const int units = n / 16, threads = 128, ctas = (units + threads - 1) / threads;
#define ROW_CASE(T) \
  case T: sb_row_kernel<T><<<ctas, threads, 0, pllm_stream()>>>(dptr<float>(out), dptr<const uint8_t>(w), dptr<const uint8_t>(tab), n); break;
  switch (type) {
    ROW_CASE(10) ROW_CASE(12) ROW_CASE(16) ROW_CASE(17) ROW_CASE(18) ROW_CASE(19) ROW_CASE(21) ROW_CASE(22) ROW_CASE(23)
    ROW_CASE(29)
  }
#undef ROW_CASE
  PLLM_LAUNCHED("sb_row");
}
