// synth.cu: seeded synthetic weights made on the device, for benchmarks and tests of model-sized shapes (no
// counterpart in the reference, whose tests build synthetic checkpoints in NumPy: tests/made_up.py:30). Values are
// N(mean, std) from a counter-based hash (splitmix64) through Box-Muller, so any element is a pure function of
// (seed, index); int8 matrices are then quantized group by group with quantize_x's arithmetic (the bytes
// engine/packing.py's quantize would write for the same float32 values).
#include "pllm_common.cuh"
#include "pllm_device.cuh"

namespace {

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// a standard normal of (seed, i)
__device__ __forceinline__ float normal_of(uint64_t seed, uint64_t i) {
  const uint64_t h = splitmix64(seed * 0x632be59bd9b4e019ull + i);
  const float u1 = ((float)(uint32_t)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);  // (0, 1)
  const float u2 = (float)(uint32_t)(h & 0xffffffu) * (1.0f / 16777216.0f);
  return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

__global__ void synth_f32_kernel(float* out, long long n, uint64_t seed, float mean, float std) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    out[i] = mean + std * normal_of(seed, (uint64_t)i);
}

// a warp a group of 32: N(0, std) values, quantized (bias 0: the converter's int8). The block's element (r, c) is
// element (row0 + r, col0 + c) of a matrix of full_cols columns, so a block is a slice of the whole matrix's bytes.
__global__ void synth_q8_kernel(int8_t* wq, float* ws, long long groups, int cols, long long row0, long long col0,
                                long long full_cols, uint64_t seed, float std) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const int per_row = cols / 32;
  for (long long g = blockIdx.x * (long long)(blockDim.x >> 5) + (threadIdx.x >> 5); g < groups; g += warps) {
    const long long r = g / per_row, c = (g % per_row) * 32 + lane;
    const float v = std * normal_of(seed, (uint64_t)((row0 + r) * full_cols + col0 + c));
    float s;
    const int8_t q = quantize_group_warp(v, lane, 0, &s);
    wq[g * 32 + lane] = q;
    if (lane == 0) ws[g] = s;
  }
}

// ternary rows: codes of weights uniform on {-1, 0, +1} (the code w + 1 at bits 2 (j & 3) of byte j / 4) and one
// float16 scale a row, N(mean, std) rounded to float16 and repeated for every group of 128 of the row
__global__ void synth_t2_kernel(uint8_t* wq, uint16_t* ws, long long rows, int cols, uint64_t seed, float mean,
                                float std) {
  const long long bytes = rows * (cols / 4);
  for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < bytes; b += (long long)gridDim.x * blockDim.x) {
    const uint64_t h = splitmix64(seed * 0x9e3779b97f4a7c15ull + (uint64_t)b);
    uint8_t v = 0;
    for (int k = 0; k < 4; k++) v |= (uint8_t)(((h >> (16 * k)) & 0xffff) % 3) << (2 * k);
    wq[b] = v;
  }
  const int groups = cols / 128;
  for (long long r = blockIdx.x * (long long)blockDim.x + threadIdx.x; r < rows; r += (long long)gridDim.x * blockDim.x) {
    int bad = 0;
    const uint16_t half = float_to_half_bits(mean + std * normal_of(seed ^ 0x5555, (uint64_t)r), &bad);
    for (int g = 0; g < groups; g++) ws[r * groups + g] = half;
  }
}

unsigned grid_n(long long n) {
  long long g = (n + 255) / 256;
  const long long most = (long long)pllm_num_sms() * 16;
  return (unsigned)(g < 1 ? 1 : (g > most ? most : g));
}

}  // namespace

PLLM_API void pllm_synth_f32(uint64_t out, int64_t n, uint64_t seed, float mean, float std) {
  PLLM_REQUIRE(n >= 0, "pllm_synth_f32: n %lld", (long long)n);
  if (!n) return;
  synth_f32_kernel<<<grid_n(n), 256, 0, pllm_stream()>>>(dptr<float>(out), n, seed, mean, std);
  PLLM_LAUNCHED("pllm_synth_f32");
}

PLLM_API void pllm_synth_q8_block(uint64_t wq, uint64_t ws, int64_t rows, int32_t cols, uint64_t seed, float std,
                                  int64_t row0, int64_t col0, int64_t full_cols) {
  PLLM_REQUIRE(rows >= 0 && cols > 0 && cols % 32 == 0 && row0 >= 0 && col0 >= 0 && col0 % 32 == 0 &&
                   full_cols % 32 == 0 && col0 + cols <= full_cols,
               "pllm_synth_q8_block: rows %lld cols %d at (%lld, %lld) of %lld", (long long)rows, cols, (long long)row0,
               (long long)col0, (long long)full_cols);
  const long long groups = rows * (cols / 32);
  if (!groups) return;
  synth_q8_kernel<<<grid_n(groups * 32), 256, 0, pllm_stream()>>>(dptr<int8_t>(wq), dptr<float>(ws), groups, cols,
                                                                   row0, col0, full_cols, seed, std);
  PLLM_LAUNCHED("pllm_synth_q8_block");
}

PLLM_API void pllm_synth_q8(uint64_t wq, uint64_t ws, int64_t rows, int32_t cols, uint64_t seed, float std) {
  PLLM_REQUIRE(rows >= 0 && cols > 0 && cols % 32 == 0, "pllm_synth_q8: rows %lld cols %d", (long long)rows, cols);
  pllm_synth_q8_block(wq, ws, rows, cols, seed, std, 0, 0, cols);
}

PLLM_API void pllm_synth_t2(uint64_t wq, uint64_t ws, int64_t rows, int32_t cols, uint64_t seed, float mean, float std) {
  PLLM_REQUIRE(rows >= 0 && cols > 0 && cols % 128 == 0, "pllm_synth_t2: rows %lld cols %d", (long long)rows, cols);
  if (!rows) return;
  synth_t2_kernel<<<grid_n(rows * (cols / 4)), 256, 0, pllm_stream()>>>(dptr<uint8_t>(wq), dptr<uint16_t>(ws), rows,
                                                                      cols, seed, mean, std);
  PLLM_LAUNCHED("pllm_synth_t2");
}
