// glue.cu: the vector work between the products and the stateful layers.
//   rmsnorm       kernels/kernel/activations.ts:8-20
//   swiglu        kernels/kernel/activations.ts:77-90
//   add_inplace   kernels/kernel/activations.ts:156-158
//   gate          kernels/kernel/stateful.ts:12-23
//   convolve      kernels/kernel/stateful.ts:49-63
//   short_conv    kernels/kernel/stateful.ts:70-86
//   delta_rule    kernels/kernel/stateful.ts:96-151 (the same float32 operations in the same order: to the bit)
//   pllm_embed_q8 the int8 embedding row as src/runtime/forward/tensors.ts:154-160 widens it (a device kernel where
//                 the reference's engine wrote the row from JavaScript)
#include "pllm_common.cuh"

namespace {

__global__ void rmsnorm_kernel(float* out, const float* x, const float* __restrict__ w, int n, float eps,
                               long long stride) {
  x += blockIdx.x * stride;
  out += blockIdx.x * stride;
  __shared__ float red[32];
  float s = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s = fmaf(x[i], x[i], s);
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  float tot = 0.0f;
  for (int i = 0; i < (int)(blockDim.x >> 5); i++) tot += red[i];
  const float r = 1.0f / sqrtf(tot / (float)n + eps);
  for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = w[i] * (r * x[i]);
}

__global__ void swiglu_kernel(float* out, const float* h1, const float* h3, int n) {
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) {
    const float v = h1[j];
    out[j] = (v / (1.0f + expf(-v))) * h3[j];
  }
}

__global__ void add_kernel(float* x, const float* y, int n) {
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x) x[j] = x[j] + y[j];
}

__global__ void gate_kernel(float* out, const float* x, const float* g, int n) {
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < n; j += gridDim.x * blockDim.x)
    out[j] = x[j] / (1.0f + expf(-g[j]));
}

__device__ __forceinline__ float taps_sum(const float* taps, const float* rows, int c, int n, int count) {
  float acc = __fmul_rn(taps[c], rows[c]);  // oldest first, as NumPy adds them
  for (int j = 1; j < count; j++) acc = __fadd_rn(acc, __fmul_rn(taps[(long long)j * n + c], rows[(long long)j * n + c]));
  return acc;
}

__global__ void convolve_kernel(float* out, const float* taps, const float* rows, int n, int count) {
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < n; c += gridDim.x * blockDim.x) {
    const float acc = taps_sum(taps, rows, c, n, count);
    out[c] = acc / (1.0f + expf(-acc));
  }
}

__global__ void short_conv_kernel(float* out, const float* taps, float* rows, const float* b, int n, int count) {
  float* newest = rows + (long long)(count - 1) * n;
  const float* gate = b + n;
  const float* z = b + 2 * (long long)n;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < n; c += gridDim.x * blockDim.x) {
    newest[c] = __fmul_rn(b[c], z[c]);
    out[c] = __fmul_rn(gate[c], taps_sum(taps, rows, c, n, count));
  }
}

// one block a value head; thread j a column of the state. Two passes over the rows i (ascending, as the reference),
// every operation rounded alone (no contraction), so the results are the reference's to the bit.
__global__ void delta_rule_kernel(float* out, const float* __restrict__ state, float* __restrict__ next,
                                  const float* __restrict__ c, float* work, int kh, int kd, int vd, int vh, int h0) {
  const int h = h0 + blockIdx.x;
  const int key = h / (vh / kh);
  const float* q = c + (long long)key * kd;
  const float* k = c + (long long)(kh + key) * kd;
  const float* v = c + (long long)(2 * kh) * kd + (long long)h * vd;
  const float beta = work[h], decay = work[vh + h];
  float* delta = work + 2 * (long long)vh + (long long)h * vd;
  const float* from = state + (long long)h * kd * vd;
  float* to = next + (long long)h * kd * vd;
  float* o = out + (long long)h * vd;
  for (int j = threadIdx.x; j < vd; j += blockDim.x) {
    float d = 0.0f;
    for (int i = 0; i < kd; i++) d = __fadd_rn(d, __fmul_rn(k[i], __fmul_rn(from[(long long)i * vd + j], decay)));
    d = __fmul_rn(__fsub_rn(v[j], d), beta);
    delta[j] = d;
    float acc = 0.0f;
    for (int i = 0; i < kd; i++) {
      const float s = __fadd_rn(__fmul_rn(from[(long long)i * vd + j], decay), __fmul_rn(k[i], d));
      to[(long long)i * vd + j] = s;
      acc = __fadd_rn(acc, __fmul_rn(q[i], s));
    }
    o[j] = acc;
  }
}

// The state once through shared memory: a CTA a (value head, DR_COLS columns); the columns of every row of the head's
// state staged by 16-byte asynchronous copies (read once), then thread j makes column j's chains in the reference's
// order (rows ascending, every operation rounded alone) for each of count tokens in turn, the state staying in shared
// memory between them; the last token's state written to next (written once). Token t's inputs at c + t c_stride,
// its gates and delta at work + t work_stride, its outputs at out + t out_stride (floats).
constexpr int DR_COLS = 16;
__device__ __forceinline__ void dr_cp16(void* smem, const void* gmem) {
  const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__global__ void __launch_bounds__(128) delta_rule_tile_kernel(float* out, long long out_stride,
                                                              const float* __restrict__ state, float* __restrict__ next,
                                                              const float* __restrict__ c, long long c_stride,
                                                              float* work, long long work_stride, int count, int kh,
                                                              int kd, int vd, int vh, int h0) {
  extern __shared__ __align__(16) float tile[];  // [kd][DR_COLS]
  const int h = h0 + blockIdx.x, j0 = blockIdx.y * DR_COLS, j = threadIdx.x;
  const int key = h / (vh / kh);
  const float* from = state + (long long)h * kd * vd + j0;
  float* to = next + (long long)h * kd * vd + j0;
  constexpr int P = DR_COLS / 4;  // 16-byte pieces a row of the tile
  for (int e = threadIdx.x; e < kd * P; e += blockDim.x) {
    const int i = e / P, p = e % P;
    dr_cp16(tile + i * DR_COLS + 4 * p, from + (long long)i * vd + 4 * p);
  }
  asm volatile("cp.async.commit_group;\ncp.async.wait_all;" ::: "memory");
  // each token's q and k rows (kd floats each) through shared memory, loaded by the whole CTA: the chains' operands
  // then come from shared memory (read from global memory inside the chains, a load a step held every step)
  float* sqk = tile + kd * DR_COLS;  // [2][kd]
  for (int t = 0; t < count; t++) {
    const float* ct = c + t * c_stride;
    __syncthreads();  // the tile is staged; the last token's q and k are read
    for (int e = threadIdx.x; e < kd; e += blockDim.x) {
      sqk[e] = ct[(long long)key * kd + e];
      sqk[kd + e] = ct[(long long)(kh + key) * kd + e];
    }
    __syncthreads();
    if (j < DR_COLS) {
      const float* q = sqk;
      const float* k = sqk + kd;
      const float* v = ct + (long long)(2 * kh) * kd + (long long)h * vd;
      float* wt = work + t * work_stride;
      const float beta = wt[h], decay = wt[vh + h];
      float d = 0.0f;
#pragma unroll 8
      for (int i = 0; i < kd; i++) d = __fadd_rn(d, __fmul_rn(k[i], __fmul_rn(tile[i * DR_COLS + j], decay)));
      d = __fmul_rn(__fsub_rn(v[j0 + j], d), beta);
      wt[2 * (long long)vh + (long long)h * vd + j0 + j] = d;
      float acc = 0.0f;
#pragma unroll 8
      for (int i = 0; i < kd; i++) {
        const float s = __fadd_rn(__fmul_rn(tile[i * DR_COLS + j], decay), __fmul_rn(k[i], d));
        tile[i * DR_COLS + j] = s;
        acc = __fadd_rn(acc, __fmul_rn(q[i], s));
      }
      out[t * out_stride + (long long)h * vd + j0 + j] = acc;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < kd * P; e += blockDim.x) {
    const int i = e / P, p = e % P;
    *reinterpret_cast<float4*>(to + (long long)i * vd + 4 * p) = *reinterpret_cast<const float4*>(tile + i * DR_COLS + 4 * p);
  }
}

__global__ void embed_q8_kernel(float* x, const int8_t* __restrict__ emb, const float* __restrict__ scales,
                                const int32_t* __restrict__ tokens, int token, int dim, long long stride) {
  const long long t = tokens ? tokens[blockIdx.y] : token;
  float* xo = x + blockIdx.y * stride;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < dim; i += gridDim.x * blockDim.x) {
    const long long at = t * dim + i;
    xo[i] = __fmul_rn((float)emb[at], scales[at / 32]);
  }
}

void launch_delta_tiles(uint64_t out, long long out_stride, uint64_t state, uint64_t next, uint64_t c,
                        long long c_stride, uint64_t work, long long work_stride, int count, int kh, int kd, int vd,
                        int vh, int h0, int h1) {
  const size_t smem = (size_t)kd * DR_COLS * 4 + 2 * (size_t)kd * 4;  // the tile, then a token's q and k
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(delta_rule_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) {
    pllm_fail(PLLM_ECUDA, "delta_rule: %zu bytes of shared memory", smem);
    return;
  }
  delta_rule_tile_kernel<<<dim3(h1 - h0, vd / DR_COLS), 128, smem, pllm_stream()>>>(
      dptr<float>(out), out_stride, dptr<const float>(state), dptr<float>(next), dptr<const float>(c), c_stride,
      dptr<float>(work), work_stride, count, kh, kd, vd, vh, h0);
  PLLM_LAUNCHED("delta_rule");
}

// The memory touches of the reference's engine between kernel calls, as device kernels (it read and wrote its WASM
// memory from JavaScript): each the same numbers as the JavaScript, whose arithmetic is in double precision and then
// stored as float32 (Math.exp, Math.log1p, Math.tanh are CUDA's double functions here).
// linear.ts:160-161 / convolution.ts:57: rows 1..count-1 of n floats move up one (copyWithin); the last is left
__global__ void shift_rows_kernel(float* rows, int n, int count) {
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < n; c += gridDim.x * blockDim.x) {
    float v = rows[(long long)(count - 1) * n + c];
    for (int j = count - 2; j >= 0; j--) {  // from the top: each value read before its row is written
      const float below = rows[(long long)j * n + c];
      rows[(long long)j * n + c] = v;
      v = below;
    }
  }
}
// linear.ts:151-158: per value head, beta = 1 / (1 + exp(-b)) and decay = exp(A softplus(g + dt_bias)), softplus(s) =
// s past 20, else log1p(exp(s)); b at work[h], g at work[vh + h] (each overwritten)
__global__ void delta_gates_kernel(float* work, const float* decays, const float* dt_bias, int vh) {
  const int h = blockIdx.x * blockDim.x + threadIdx.x;
  if (h >= vh) return;
  const double b = work[h], step = (double)work[vh + h] + (double)dt_bias[h];
  work[h] = (float)(1.0 / (1.0 + exp(-b)));
  work[vh + h] = (float)exp((double)decays[h] * (step > 20.0 ? step : log1p(exp(step))));
}
// engine.ts:452-455: count rows of n floats (stride apart) times a layer's scale (read from device memory)
__global__ void scale_rows_kernel(float* x, int n, int count, long long stride, const float* scale) {
  const float s = *scale;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < (long long)n * count;
       i += (long long)gridDim.x * blockDim.x) {
    const long long t = i / n, c = i % n;
    x[t * stride + c] = __fmul_rn(x[t * stride + c], s);
  }
}
// engine.ts:467-470: logits = cap tanh(logits / cap), the quotient, its tanh and the product each rounded to float32
__global__ void softcap_kernel(float* x, int n, float cap) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float q = (float)((double)x[i] / (double)cap);
    const float t = (float)tanh((double)q);
    x[i] = (float)((double)cap * (double)t);
  }
}

// An LFM2 convolution layer's step between its two products, for a batch of sequences (grid y): the rows move up one
// (convolution.ts:57's copyWithin; at position 0 the rows before are zero, as clear() leaves them), the newest row is
// B z, and out = C times the taps' sum over the rows, oldest first (stateful.ts:70-86's short_conv): the same float32
// operations in the same order, so the reference's numbers to the bit. mixed: [B | C | z] a sequence.
__global__ void conv_step_kernel(float* out, const float* __restrict__ taps, float* rows, const float* __restrict__ mixed,
                                 int n, int count, const int* pos_dev, long long rows_stride, long long mixed_stride,
                                 long long out_stride) {
  const int z = blockIdx.y;
  rows += z * rows_stride;
  mixed += z * mixed_stride;
  out += z * out_stride;
  const bool fresh = pos_dev && pos_dev[z] == 0;
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < n; c += gridDim.x * blockDim.x) {
    float r[8];
    for (int j = 0; j + 1 < count; j++) r[j] = fresh ? 0.0f : rows[(long long)(j + 1) * n + c];
    r[count - 1] = __fmul_rn(mixed[c], mixed[2 * (long long)n + c]);
    float acc = __fmul_rn(taps[c], r[0]);
    rows[c] = r[0];
    for (int j = 1; j < count; j++) {
      rows[(long long)j * n + c] = r[j];
      acc = __fadd_rn(acc, __fmul_rn(taps[(long long)j * n + c], r[j]));
    }
    out[c] = __fmul_rn(mixed[(long long)n + c], acc);
  }
}

unsigned grid_of(int n) {
  unsigned g = cdiv((unsigned)(n > 0 ? n : 1), 256u);
  const unsigned most = (unsigned)pllm_num_sms() * 4;
  return g > most ? most : g;
}

}  // namespace

PLLM_API void rmsnorm(uint64_t out, uint64_t x, uint64_t w, int32_t n, float eps) {
  PLLM_REQUIRE(n > 0, "rmsnorm: n %d", n);
  rmsnorm_kernel<<<1, 1024, 0, pllm_stream()>>>(dptr<float>(out), dptr<const float>(x), dptr<const float>(w), n, eps, 0);
  PLLM_LAUNCHED("rmsnorm");
}

// rmsnorm of rows rows of n, stride apart (floats), all with the same weight: the per-head norms of q and k
PLLM_API void pllm_rmsnorm_rows(uint64_t out, uint64_t x, uint64_t w, int32_t n, float eps, int32_t rows,
                                int64_t stride) {
  PLLM_REQUIRE(n > 0 && rows > 0, "pllm_rmsnorm_rows: n %d rows %d", n, rows);
  rmsnorm_kernel<<<rows, n >= 1024 ? 1024 : ((n + 31) / 32) * 32, 0, pllm_stream()>>>(
      dptr<float>(out), dptr<const float>(x), dptr<const float>(w), n, eps, stride);
  PLLM_LAUNCHED("pllm_rmsnorm_rows");
}

PLLM_API void swiglu(uint64_t out, uint64_t h1, uint64_t h3, int32_t n) {
  PLLM_REQUIRE(n >= 0, "swiglu: n %d", n);
  if (!n) return;
  swiglu_kernel<<<grid_of(n), 256, 0, pllm_stream()>>>(dptr<float>(out), dptr<const float>(h1), dptr<const float>(h3), n);
  PLLM_LAUNCHED("swiglu");
}

PLLM_API void add_inplace(uint64_t x, uint64_t y, int32_t n) {
  PLLM_REQUIRE(n >= 0, "add_inplace: n %d", n);
  if (!n) return;
  add_kernel<<<grid_of(n), 256, 0, pllm_stream()>>>(dptr<float>(x), dptr<const float>(y), n);
  PLLM_LAUNCHED("add_inplace");
}

PLLM_API void gate(uint64_t out, uint64_t x, uint64_t g, int32_t n) {
  PLLM_REQUIRE(n >= 0, "gate: n %d", n);
  if (!n) return;
  gate_kernel<<<grid_of(n), 256, 0, pllm_stream()>>>(dptr<float>(out), dptr<const float>(x), dptr<const float>(g), n);
  PLLM_LAUNCHED("gate");
}

PLLM_API void convolve(uint64_t out, uint64_t taps, uint64_t rows, int32_t n, int32_t count) {
  PLLM_REQUIRE(n >= 0 && count >= 1, "convolve: n %d count %d", n, count);
  if (!n) return;
  convolve_kernel<<<grid_of(n), 256, 0, pllm_stream()>>>(dptr<float>(out), dptr<const float>(taps),
                                                       dptr<const float>(rows), n, count);
  PLLM_LAUNCHED("convolve");
}

PLLM_API void short_conv(uint64_t out, uint64_t taps, uint64_t rows, uint64_t b, int32_t n, int32_t count) {
  PLLM_REQUIRE(n >= 0 && count >= 2, "short_conv: n %d count %d", n, count);
  if (!n) return;
  short_conv_kernel<<<grid_of(n), 256, 0, pllm_stream()>>>(dptr<float>(out), dptr<const float>(taps),
                                                         dptr<float>(rows), dptr<const float>(b), n, count);
  PLLM_LAUNCHED("short_conv");
}

PLLM_API void delta_rule(uint64_t out, uint64_t state, uint64_t next, uint64_t c, uint64_t work, int32_t kh,
                         int32_t kd, int32_t vd, int32_t vh, int32_t h0, int32_t h1) {
  PLLM_REQUIRE(kh > 0 && vh > 0 && vh % kh == 0 && kd > 0 && vd > 0, "delta_rule: kh %d vh %d kd %d vd %d", kh, vh,
               kd, vd);
  PLLM_REQUIRE(h0 >= 0 && h1 >= h0 && h1 <= vh, "delta_rule: heads %d..%d of %d", h0, h1, vh);
  PLLM_REQUIRE(state != next, "delta_rule: state and next must be apart (the reference writes next only)");
  if (h1 == h0) return;
  if (vd % DR_COLS == 0 && !(state & 15) && !(next & 15) && (size_t)kd * DR_COLS * 4 <= 200 * 1024) {
    launch_delta_tiles(out, 0, state, next, c, 0, work, 0, 1, kh, kd, vd, vh, h0, h1);
    return;
  }
  const int threads = vd >= 256 ? 256 : ((vd + 31) / 32) * 32;  // other widths: a block a head, the state read twice
  delta_rule_kernel<<<h1 - h0, threads, 0, pllm_stream()>>>(dptr<float>(out), dptr<const float>(state),
                                                           dptr<float>(next), dptr<const float>(c), dptr<float>(work),
                                                           kh, kd, vd, vh, h0);
  PLLM_LAUNCHED("delta_rule");
}

// count tokens of the recurrence in one launch (a prompt's block): token t's inputs at c + t c_stride floats, its
// gates, delta and outputs at work / out + t (work_stride, out_stride) floats; state is read once and the state after
// the last token written to next once (the states between stay on the chip). Every token's numbers are delta_rule's.
PLLM_API void pllm_delta_rule_block(uint64_t out, int64_t out_stride, uint64_t state, uint64_t next, uint64_t c,
                                    int64_t c_stride, uint64_t work, int64_t work_stride, int32_t count, int32_t kh,
                                    int32_t kd, int32_t vd, int32_t vh, int32_t h0, int32_t h1) {
  PLLM_REQUIRE(kh > 0 && vh > 0 && vh % kh == 0 && kd > 0 && vd > 0 && count >= 1 && vd % DR_COLS == 0 &&
                   !(state & 15) && !(next & 15) && state != next && (size_t)kd * DR_COLS * 4 <= 200 * 1024 &&
                   h0 >= 0 && h1 >= h0 && h1 <= vh,
               "pllm_delta_rule_block: kh %d vh %d kd %d vd %d count %d heads %d..%d", kh, vh, kd, vd, count, h0, h1);
  if (h1 == h0) return;
  launch_delta_tiles(out, out_stride, state, next, c, c_stride, work, work_stride, count, kh, kd, vd, vh, h0, h1);
}

PLLM_API void pllm_conv_step(uint64_t out, int64_t out_stride, uint64_t taps, uint64_t rows, int64_t rows_stride,
                              uint64_t mixed, int64_t mixed_stride, int32_t n, int32_t count, uint64_t pos_dev,
                              int32_t batch) {
  PLLM_REQUIRE(out && taps && rows && mixed && n > 0 && count >= 1 && count <= 8 && batch >= 1 && batch <= 65535,
               "pllm_conv_step: n %d count %d batch %d", n, count, batch);
  conv_step_kernel<<<dim3(cdiv(n, 256), batch), 256, 0, pllm_stream()>>>(
      dptr<float>(out), dptr<const float>(taps), dptr<float>(rows), dptr<const float>(mixed), n, count,
      dptr<const int>(pos_dev), rows_stride, mixed_stride, out_stride);
  PLLM_LAUNCHED("pllm_conv_step");
}

PLLM_API void pllm_shift_rows(uint64_t rows, int32_t n, int32_t count) {
  PLLM_REQUIRE(rows && n > 0 && count >= 1, "pllm_shift_rows: n %d count %d", n, count);
  if (count < 2) return;
  shift_rows_kernel<<<grid_of(n), 256, 0, pllm_stream()>>>(dptr<float>(rows), n, count);
  PLLM_LAUNCHED("pllm_shift_rows");
}
PLLM_API void pllm_delta_gates(uint64_t work, uint64_t decays, uint64_t dt_bias, int32_t vh) {
  PLLM_REQUIRE(work && decays && dt_bias && vh > 0, "pllm_delta_gates: vh %d", vh);
  delta_gates_kernel<<<cdiv(vh, 128), 128, 0, pllm_stream()>>>(dptr<float>(work), dptr<const float>(decays),
                                                               dptr<const float>(dt_bias), vh);
  PLLM_LAUNCHED("pllm_delta_gates");
}
PLLM_API void pllm_scale_rows(uint64_t x, int32_t n, int32_t count, int64_t stride, uint64_t scale) {
  PLLM_REQUIRE(x && scale && n > 0 && count > 0 && stride >= n, "pllm_scale_rows: n %d count %d", n, count);
  scale_rows_kernel<<<grid_of(n * count), 256, 0, pllm_stream()>>>(dptr<float>(x), n, count, stride,
                                                                    dptr<const float>(scale));
  PLLM_LAUNCHED("pllm_scale_rows");
}
PLLM_API void pllm_softcap(uint64_t x, int32_t n, float cap) {
  PLLM_REQUIRE(x && n > 0 && cap > 0.0f, "pllm_softcap: n %d cap %g", n, (double)cap);
  softcap_kernel<<<grid_of(n), 256, 0, pllm_stream()>>>(dptr<float>(x), n, cap);
  PLLM_LAUNCHED("pllm_softcap");
}

// count tokens' embedding rows (tokens: device int32[count], or 0 to take token) into x, stride floats apart
PLLM_API void pllm_embed_q8(uint64_t x, uint64_t emb, uint64_t scales, uint64_t tokens, int32_t token, int32_t dim,
                            int32_t count, int64_t stride) {
  PLLM_REQUIRE(dim > 0 && dim % 32 == 0 && count > 0, "pllm_embed_q8: dim %d count %d", dim, count);
  embed_q8_kernel<<<dim3(cdiv(dim, 256), count), 256, 0, pllm_stream()>>>(
      dptr<float>(x), dptr<const int8_t>(emb), dptr<const float>(scales), dptr<const int32_t>(tokens), token, dim,
      stride);
  PLLM_LAUNCHED("pllm_embed_q8");
}
