// gemm_q8.cu: the prefill product on the tensor cores: M tokens' int8 activations times int8 weights, each group of
// 32 scaled by its two quantize_x scales (the arithmetic of matmul.ts:77-104 / relaxed/int8.ts:17-166 over a tile of
// tokens, what the reference's q8rTile does four tokens at a time on the CPU: relaxed/int8.ts:89-166).
//
// out[m][n] = sum over groups g of  f32(G_g[m][n]) * (xs[m][g] * ws[n][g]),   G_g = sum_{k in g} xq[m][k] w[n][k]
//
// Every G_g is an exact int32, and the scales differ from group to group, so the groups cannot be summed in the
// integer accumulator: each group of 32 is one tcgen05.mma of kind::i8 (K = 32) into its own TMEM accumulator, read
// back by the epilogue warps, scaled and added in float32 registers. The MMA of a 128 x 128 tile and group takes ~64
// cycles of the tensor pipe; the epilogue's conversion, scale and add of its 16,384 values take ~3 float32 operations
// each, ~384 cycles of an SM's 128 float32 lanes: the kernel is bound by that epilogue, at roughly a sixth of the int8
// tensor peak (the price of the reference's per-group scales; a product that summed groups in the integer accumulator
// would not be the reference's numbers).
//
// A CTA: warp 0 issues the TMA copies (activations [128 tokens][128 bytes of K], weights [2 x 64 rows][128 bytes],
// their scales) into a ring of 4 stages; warp 1 allocates TMEM and one thread issues the MMAs (4 groups a stage) into
// 4 accumulator buffers of 128 columns; warps 2..17 take a buffer each group (warp w: TMEM lanes 32 (w % 4)..+31 =
// tokens, columns 32 h..+31 with h = (w - 2) / 4: four warps on each SM sub-partition, so that one's latency is
// another's issue), convert (exact: the int32 plus 2^23 + 2^22 read as a float32, minus that), scale and accumulate,
// then store the tile with the epilogue's operation (store, add into the residual, or the gated FFN's silu(w1 row) x
// (w3 row), the two halves of the weight tile being w1's and w3's rows).
// Every mbarrier wait is bounded: past the bound the kernel records PLLM_ETIMEOUT, stops issuing work, and still
// frees its TMEM before it returns.
#include <cuda.h>

#include "pllm_common.cuh"
#include "pllm_device.cuh"

namespace gemvk {
int* status_word();  // the device status word's address on the current device (gemv_tma.cu)
}

namespace {

constexpr int BM = 128, BN = 128, BKB = 128;  // a tile's tokens and weight rows; K bytes a stage
constexpr int GPS = BKB / 32;                 // groups a stage
constexpr int STAGES = 4, NBUF = 4;           // shared-memory stages; TMEM accumulator buffers of BN columns
constexpr int EPI_WARPS = 16;                 // four a TMEM lane quarter, 32 columns each
constexpr int GEMM_THREADS = (2 + EPI_WARPS) * 32;
constexpr int A_BYTES = BM * BKB, B_BYTES = BN * BKB;
constexpr int XS_BYTES = BM * GPS * 4, WS_BYTES = BN * GPS * 4;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES + XS_BYTES + WS_BYTES;  // 36,864 (a multiple of 1024)
constexpr int TMEM_COLS = NBUF * BN;                                   // 512: the whole TMEM of an SM
constexpr long long WAIT_BOUND = 1ll << 26;
constexpr uint32_t IDESC = (2u << 4)        // D: int32
                           | (1u << 7)      // A: signed 8-bit
                           | (1u << 10)     // B: signed 8-bit
                           | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);  // K-major A and B

enum { GE_STORE = 0, GE_ADD = 1, GE_SWIGLU = 2 };

struct GemmArgs {
  float* out;
  long long ldo;    // floats between tokens' rows of out
  int M, K;
  int N;            // output columns (GE_SWIGLU: hidden rows)
  long long pair;   // GE_SWIGLU: w3's first row in the weight tensor (w1's is 0)
  int* status;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, int* status) {
  const uint32_t addr = smem_u32(bar);
  for (long long i = 0; i < WAIT_BOUND; i++) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(addr), "r"(parity)
        : "memory");
    if (done) return true;
  }
  atomicExch(status, PLLM_ETIMEOUT);
  return false;
}
__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// K-major operand in 128-byte swizzled rows (8-row atoms of 1024 bytes): leading offset unused (1), stride 1024 bytes
__device__ __forceinline__ uint64_t smem_desc(const void* p) {
  return (uint64_t)((smem_u32(p) >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
__device__ __forceinline__ void mma_i8(uint32_t d, uint64_t a, uint64_t b) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(IDESC), "r"(0), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory"); }

template <int EPI>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_q8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmX,
                   const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmW, const GemmArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;
  uint64_t* acce = accf + NBUF;
  uint64_t* done = acce + NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BM;
  const int ngroups = a.K / 32, nkb = a.K / BKB;
  const int r0 = EPI == GE_SWIGLU ? blockIdx.y * (BN / 2) : blockIdx.y * BN;
  const int r1 = EPI == GE_SWIGLU ? (int)a.pair + r0 : r0 + BN / 2;
  auto stage = [&](int s) { return smem + (size_t)s * STAGE_BYTES; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + EPI_WARPS);  // the stage's last MMAs (a commit) and every epilogue warp's scales
    }
    for (int b = 0; b < NBUF; b++) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], EPI_WARPS);
    }
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0 && lane == 0) {  // ---- the copies
    int issued = 0;
    for (int kb = 0; kb < nkb; kb++, issued++) {
      const int s = kb % STAGES;
      if (!mbar_wait(&empty[s], ((kb / STAGES) & 1) ^ 1, a.status)) break;
      uint8_t* st = stage(s);
      mbar_expect_tx(&full[s], STAGE_BYTES);
      tma_2d(st, &tmA, kb * BKB, m0, &full[s]);
      tma_2d(st + A_BYTES, &tmB, kb * BKB, r0, &full[s]);
      tma_2d(st + A_BYTES + B_BYTES / 2, &tmB, kb * BKB, r1, &full[s]);
      tma_2d(st + A_BYTES + B_BYTES, &tmX, kb * GPS, m0, &full[s]);
      tma_2d(st + A_BYTES + B_BYTES + XS_BYTES, &tmW, r0, kb * GPS, &full[s]);
      tma_2d(st + A_BYTES + B_BYTES + XS_BYTES + WS_BYTES / 2, &tmW, r1, kb * GPS, &full[s]);
    }
    // the copies still in flight land before the CTA leaves (bounded: each stage's latest copy)
    for (int kb = issued - STAGES < 0 ? 0 : issued - STAGES; kb < issued; kb++)
      mbar_wait(&full[kb % STAGES], (kb / STAGES) & 1, a.status);
  } else if (warp == 1 && lane == 0) {  // ---- the MMAs
    int g = 0;
    bool ok = true;
    for (int kb = 0; kb < nkb && ok; kb++) {
      const int s = kb % STAGES;
      ok = mbar_wait(&full[s], (kb / STAGES) & 1, a.status);
      if (!ok) break;
      fence_after();
      const uint8_t* st = stage(s);
      for (int j = 0; j < GPS && ok; j++, g++) {
        const int b = g % NBUF;
        ok = mbar_wait(&acce[b], ((g / NBUF) & 1) ^ 1, a.status);
        if (!ok) break;
        fence_after();
        mma_i8(tmem + (uint32_t)(b * BN), smem_desc(st + 32 * j), smem_desc(st + A_BYTES + 32 * j));
        mma_commit(&accf[b]);
      }
      mma_commit(&empty[s]);
    }
    mma_commit(done);  // every MMA issued has completed once this arrives
    mbar_wait(done, 0, a.status);
  } else if (warp >= 2) {  // ---- the epilogue
    // warp w: TMEM lanes 32 (w % 4).. (tokens) and columns 32 h..+31 with h = (w - 2) / 4 (h 0, 1: the weight tile's
    // first half, w1's rows for the gated FFN; 2, 3: its second half, w3's)
    const int q = warp & 3, h = (warp - 2) >> 2;
    const int m = 32 * q + lane;
    float2 acc2[16];  // column pairs (2 c, 2 c + 1): the packed float32 operations take two columns an instruction
#pragma unroll
    for (int c = 0; c < 16; c++) acc2[c] = make_float2(0.0f, 0.0f);
    bool ok = true;
    for (int g = 0; g < ngroups; g++) {
      const int b = g % NBUF, kb = g / GPS, j = g % GPS, s = kb % STAGES;
      if (ok) ok = mbar_wait(&accf[b], (g / NBUF) & 1, a.status);
      fence_after();
      uint32_t r[32];
      const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(b * BN + 32 * h);
      tmem_ld32(taddr, r);
      tmem_wait_ld();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[b]);
      if (ok) {
        const uint8_t* st = stage(s);
        const float xsv = reinterpret_cast<const float*>(st + A_BYTES + B_BYTES)[m * GPS + j];
        const float2 xs2 = make_float2(xsv, xsv), off2 = make_float2(-12582912.0f, -12582912.0f);
        const float4* wsv = reinterpret_cast<const float4*>(st + A_BYTES + B_BYTES + XS_BYTES +
                                                            (h >> 1) * (WS_BYTES / 2)) + j * 16 + (h & 1) * 8;
#pragma unroll
        for (int c4 = 0; c4 < 8; c4++) {
          const float4 w = wsv[c4];
#pragma unroll
          for (int u = 0; u < 2; u++) {
            const int c = 4 * c4 + 2 * u;
            // exact: |G| < 2^22, its bits added to those of 1.5 x 2^23 and that taken off (two columns at once)
            const float2 G = __fadd2_rn(make_float2(__int_as_float((int)r[c] + 0x4B400000),
                                                    __int_as_float((int)r[c + 1] + 0x4B400000)), off2);
            const float2 s = __fmul2_rn(u ? make_float2(w.z, w.w) : make_float2(w.x, w.y), xs2);
            acc2[c / 2] = __ffma2_rn(G, s, acc2[c / 2]);
          }
        }
      }
      if (j == GPS - 1) {  // this stage's scales are read: the copies may refill it
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
    }
    // the tile out
    float acc[32];
#pragma unroll
    for (int c = 0; c < 16; c++) {
      acc[2 * c] = acc2[c].x;
      acc[2 * c + 1] = acc2[c].y;
    }
    const int row = m0 + m;
    if (EPI == GE_SWIGLU) {
      float* sw = reinterpret_cast<float*>(smem);  // [BM][65]: the w3 rows' results (the stages are done)
      if (h >= 2)
#pragma unroll
        for (int c = 0; c < 32; c++) sw[m * 65 + 32 * (h - 2) + c] = acc[c];
      epi_sync();
      if (h < 2 && row < a.M) {
        float* o = a.out + (long long)row * a.ldo + blockIdx.y * (BN / 2) + 32 * h;
#pragma unroll
        for (int c = 0; c < 32; c += 4) {
          float4 v;
          const float h1[4] = {acc[c], acc[c + 1], acc[c + 2], acc[c + 3]};
          float res[4];
#pragma unroll
          for (int u = 0; u < 4; u++) res[u] = (h1[u] / (1.0f + expf(-h1[u]))) * sw[m * 65 + 32 * h + c + u];
          v = make_float4(res[0], res[1], res[2], res[3]);
          *reinterpret_cast<float4*>(o + c) = v;
        }
      }
    } else if (row < a.M) {
      const int n0 = blockIdx.y * BN + 32 * h;
      float* o = a.out + (long long)row * a.ldo + n0;
#pragma unroll
      for (int c = 0; c < 32; c += 4) {
        if (n0 + c >= a.N) break;
        float4 v = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);
        if (EPI == GE_ADD) {
          const float4 old = *reinterpret_cast<const float4*>(o + c);
          v.x += old.x;
          v.y += old.y;
          v.z += old.z;
          v.w += old.w;
        }
        *reinterpret_cast<float4*>(o + c) = v;
      }
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
}

// ---- tensor maps (the driver's encoder, looked up through the runtime: no link to libcuda)

typedef CUresult (*EncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  std::lock_guard<std::mutex> hold(pllm_lookup_lock());
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  }
  return fn;
}

// a 2-D map of rows x cols elements (row stride cols), copied box_rows x box_cols at a time
bool make_map(CUtensorMap* map, const void* base, CUtensorMapDataType type, int elem, long long rows, long long cols,
              int box_cols, int box_rows, bool swizzle) {
  EncodeTiled enc = encoder();
  if (!enc) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(cols * elem)};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---- the prefill's activations: RMSNorm (optional) then quantize_x, a row a CTA, signed int8 out

__global__ void norm_quantize_kernel(int8_t* xq, float* xs, const float* x, long long x_stride, const float* norm,
                                     float eps, int n, int bias) {
  const long long row = blockIdx.x;
  const float* xr = x + row * x_stride;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, warps = blockDim.x >> 5;
  __shared__ float red[32];
  float rs = 1.0f;
  if (norm) {  // activations.ts:8-20: the sum of squares, then w * (rs * x)
    float s = 0.0f;
    for (int i = tid; i < n; i += blockDim.x) s = fmaf(xr[i], xr[i], s);
    s = warp_sum(s);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < warps; i++) tot += red[i];
    rs = 1.0f / sqrtf(tot / (float)n + eps);
  }
  for (int g = warp; g < n / 32; g += warps) {  // a warp a group (quantize.ts:124-151, value j in lane j)
    float v = xr[32 * g + lane];
    if (norm) v = norm[32 * g + lane] * (rs * v);
    float s;
    const int8_t q = quantize_group_warp(v, lane, bias, &s);
    xq[row * n + 32 * g + lane] = (int8_t)(q - bias);
    if (lane == 0) xs[row * (n / 32) + g] = s;
  }
}

__global__ void transpose_scales_kernel(float* dst, const float* src, long long rows, int groups) {
  const long long total = rows * groups;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const long long g = i / rows, r = i % rows;
    dst[i] = src[r * groups + g];
  }
}

}  // namespace

// The prefill product: out (M x N floats, ldo floats a row) from xq (M x K signed int8, pllm_norm_quantize_rows),
// xs (M x K/32 floats), wq (w_rows x K int8) and ws_t (its scales transposed: K/32 x w_rows floats,
// pllm_transpose_scales). epi 0 store, 1 add into out, 2 the gated FFN: N = hidden, w1's rows 0..N and w3's at
// pair.. (silu(w1 row) x w3 row). K a multiple of 128, N a multiple of 128 (64 for epi 2).
PLLM_API void pllm_gemm_q8(uint64_t out, int64_t ldo, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws_t, int32_t M,
                           int32_t N, int32_t K, int64_t w_rows, int32_t epi, int64_t pair) {
  PLLM_REQUIRE(M > 0 && K > 0 && K % 128 == 0 && epi >= GE_STORE && epi <= GE_SWIGLU && ldo >= N && ldo % 4 == 0 &&
                   (epi == GE_SWIGLU ? N % 64 == 0 && pair >= N && pair + N <= w_rows : N % 128 == 0 && N <= w_rows),
               "pllm_gemm_q8: M %d N %d K %d rows %lld epi %d pair %lld ldo %lld", M, N, K, (long long)w_rows, epi,
               (long long)pair, (long long)ldo);
  PLLM_REQUIRE(!(xq & 15) && !(xs & 15) && !(wq & 15) && !(ws_t & 15) && !(out & 15) && w_rows % 4 == 0,
               "pllm_gemm_q8: addresses must be 16-byte aligned and w_rows a multiple of 4");
  CUtensorMap mA, mX, mB, mW;
  const int tiles_n = epi == GE_SWIGLU ? N / 64 : N / 128;
  if (!make_map(&mA, dptr<void>(xq), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, K, BKB, BM, true) ||
      !make_map(&mX, dptr<void>(xs), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, M, K / 32, GPS, BM, false) ||
      !make_map(&mB, dptr<void>(wq), CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, w_rows, K, BKB, BN / 2, true) ||
      !make_map(&mW, dptr<void>(ws_t), CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, K / 32, w_rows, BN / 2, GPS, false)) {
    pllm_fail(PLLM_ECUDA, "pllm_gemm_q8: tensor map encoding failed");
    return;
  }
  GemmArgs a = {};
  a.out = dptr<float>(out);
  a.ldo = ldo;
  a.M = M;
  a.N = N;
  a.K = K;
  a.pair = pair;
  a.status = gemvk::status_word();
  if (!a.status) {
    pllm_fail(PLLM_ECUDA, "pllm_gemm_q8: no status word");
    return;
  }
  const size_t smem = (size_t)STAGES * STAGE_BYTES + 1024 + 256;
  const dim3 grid((M + BM - 1) / BM, tiles_n);
  cudaError_t e;
  auto run = [&](auto kernel) {
    cudaError_t r = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (r != cudaSuccess) return r;
    kernel<<<grid, GEMM_THREADS, smem, pllm_stream()>>>(mA, mX, mB, mW, a);
    return cudaGetLastError();
  };
  if (epi == GE_STORE) e = run(gemm_q8_kernel<GE_STORE>);
  else if (epi == GE_ADD) e = run(gemm_q8_kernel<GE_ADD>);
  else e = run(gemm_q8_kernel<GE_SWIGLU>);
  if (e != cudaSuccess) pllm_fail(PLLM_ECUDA, "pllm_gemm_q8: launch failed: %s", cudaGetErrorString(e));
}

// rows rows of n floats (x_stride floats apart): RMSNorm with norm (or none: 0), then quantize_x with bias, written as
// signed int8 (the bias taken off: the tensor-core product's operand) and n / 32 scales a row
PLLM_API void pllm_norm_quantize_rows(uint64_t xq, uint64_t xs, uint64_t x, int64_t x_stride, uint64_t norm, float eps,
                                      int32_t n, int32_t rows, int32_t bias) {
  PLLM_REQUIRE(n > 0 && n % 32 == 0 && rows >= 0 && (bias == 0 || bias == 64), "pllm_norm_quantize_rows: n %d rows %d",
               n, rows);
  if (!rows) return;
  norm_quantize_kernel<<<rows, 256, 0, pllm_stream()>>>(dptr<int8_t>(xq), dptr<float>(xs), dptr<const float>(x),
                                                       x_stride, dptr<const float>(norm), eps, n, bias);
  PLLM_LAUNCHED("pllm_norm_quantize_rows");
}

// dst[g][r] = src[r][g]: a matrix's scales (rows x groups) in the layout the tensor-core product reads
PLLM_API void pllm_transpose_scales(uint64_t dst, uint64_t src, int64_t rows, int32_t groups) {
  PLLM_REQUIRE(rows >= 0 && groups > 0, "pllm_transpose_scales: rows %lld groups %d", (long long)rows, groups);
  if (!rows) return;
  const long long total = rows * groups;
  long long blocks = (total + 255) / 256;
  if (blocks > 4096) blocks = 4096;
  transpose_scales_kernel<<<(unsigned)blocks, 256, 0, pllm_stream()>>>(dptr<float>(dst), dptr<const float>(src), rows,
                                                                      groups);
  PLLM_LAUNCHED("pllm_transpose_scales");
}
