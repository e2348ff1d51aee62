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
#include <cfloat>

#include "pllm_common.cuh"

namespace {

constexpr int AM_THREADS = 256;

// a float's bits made to order as unsigned: larger value, larger key (-inf lowest of the non-NaN)
__device__ __forceinline__ unsigned ordered(float v) {
  const unsigned b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// key_out (the tensor-parallel form): instead of the index, the slice's key with its global index (offset + i), for the
// ranks' largest key to be taken by a max across the ranks; the slice that starts the vocabulary (offset 0) with a NaN
// first gives the largest key of all, which names index 0 (the reference's walk: nothing is greater than a NaN start)
__global__ void argmax_kernel(const float* __restrict__ x, int n, unsigned long long* key, unsigned* count, int* out,
                              unsigned long long* key_out = nullptr, long long offset = 0) {
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
  if (key_out) {
    unsigned long long g = k ? (k & 0xFFFFFFFF00000000ull) | (0xFFFFFFFFu - (unsigned)(offset + idx)) : 0ull;
    if (offset == 0 && x0 != x0) g = ~0ull;
    *key_out = g;
    *count = 0;
    return;
  }
  if (x0 != x0) idx = 0;  // the walk starts from a NaN: nothing is greater
  *out = idx;
  *count = 0;
}

// the token of the ranks' largest key (after a max across the ranks): its global index, 0 where no rank had a
// number (every logit a NaN)
__global__ void key_token_kernel(int* out, const unsigned long long* key) {
  const unsigned long long k = *key;
  *out = k ? (int)(0xFFFFFFFFu - (unsigned)(k & 0xFFFFFFFFu)) : 0;
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
// zero between calls. The call holds the library's scratch lock from its launch until it has the index, so host
// threads that call it at once take turns.
static __device__ unsigned long long g_argmax_key = 0;
static __device__ unsigned g_argmax_count = 0;
static __device__ int g_argmax_out = 0;

// argmax (sample.ts:6): the first index of the largest of n floats at x
PLLM_API int32_t argmax(uint64_t x, int32_t n) {
  PLLM_REQUIRE_RET(x && n > 0, 0, "argmax: n %d", n);
  std::lock_guard<std::mutex> hold(pllm_scratch_lock());  // the scratch is the library's: one call at a time
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

// The tensor-parallel greedy step (no counterpart in the reference, which holds the whole vocabulary in one memory):
// rank r's slice of n logits at x starts at token offset; key (8 bytes of device memory) gets the slice's largest
// as (ordered float bits, complement of the global token), so that the largest key across the ranks (an integer max,
// e.g. an all-reduce) names the reference argmax's token (sample.ts:6: the first index of the largest, a NaN skipped,
// index 0 where the walk starts from a NaN); scratch as pllm_argmax_dev's
PLLM_API void pllm_argmax_key_dev(uint64_t key, uint64_t x, int32_t n, int64_t offset, uint64_t scratch) {
  PLLM_REQUIRE(key && !(key & 7) && x && n > 0 && offset >= 0 && offset + n <= 0x7FFFFFFFll && scratch && !(scratch & 7),
               "pllm_argmax_key_dev: n %d offset %lld", n, (long long)offset);
  argmax_kernel<<<grid_for(n), AM_THREADS, 0, pllm_stream()>>>(
      dptr<const float>(x), n, dptr<unsigned long long>(scratch), dptr<unsigned>(scratch + 8), nullptr,
      dptr<unsigned long long>(key), offset);
  PLLM_LAUNCHED("pllm_argmax_key_dev");
}
// the token (one int32 at out) that the largest of the ranks' keys names
PLLM_API void pllm_key_token_dev(uint64_t out, uint64_t key) {
  PLLM_REQUIRE(out && key && !(key & 7), "pllm_key_token_dev: addresses");
  key_token_kernel<<<1, 1, 0, pllm_stream()>>>(dptr<int>(out), dptr<const unsigned long long>(key));
  PLLM_LAUNCHED("pllm_key_token_dev");
}

// penalize (sample.ts:16): the logits of the distinct tokens of tokens[0..count)
PLLM_API void penalize(uint64_t logits, uint64_t tokens, int32_t count, float penalty, float presence) {
  PLLM_REQUIRE(count >= 0 && (count == 0 || (logits && tokens)), "penalize: count %d", count);
  if (!count) return;
  penalize_kernel<<<(count + 255) / 256, 256, 0, pllm_stream()>>>(dptr<float>(logits), dptr<const int>(tokens), count,
                                                                 penalty, presence);
  PLLM_LAUNCHED("penalize");
}

// ---- sample (sample.ts:248-337): a token drawn from softmax(logits / temperature) by one random number, with the
// reference's top-k, nucleus (top-p) and min-p, in the reference's order of the walk:
//   1. the largest logit (a NaN anywhere or an infinity: -1), a grid of CTAs;
//   2. the candidates (with a nucleus, those within 16.118095 temperature of it; else all), kept in token order:
//      each CTA counts its share, then writes its candidates behind the counts of the CTAs before it;
//   3. one CTA of 1024 threads does the rest: the probabilities (the first 4 (count / 4) as the reference's four-lane
//      exp of x (1 / temperature) clamped to [-87, 88], the rest as its scalar one of x / temperature, 0 below -87:
//      CUDA's expf inside the clamps, where the reference has its own table-free exp: probabilities within an ulp or
//      two of its), their double sum and maximum; top-k by a radix select on (probability bits, complement of the
//      token), 8 bits a pass; with a nucleus or a top-k, the survivors of the cutoff and min-p walked from the most
//      probable (chunks of at most 1024 selected the same way and sorted by a bitonic sort in shared memory); else
//      walked in token order (each thread a contiguous part, the parts' double sums scanned).
// Double sums in another association than the reference's one-by-one walk may differ in their last bits: a draw
// differs only where the random number falls within about 1e-15 of a boundary.
namespace {

// SP_CHUNK: the keys the final kernel sorts at once, in its dynamic shared memory (128 KB)
constexpr int SP_THREADS = 256, SP_FINAL = 1024, SP_MAX_CTAS = 1024, SP_CHUNK = 16384;

struct SampleScratch {
  float part_max[SP_MAX_CTAS];
  int counts[SP_MAX_CTAS];
};
__device__ SampleScratch g_sample;
__device__ int g_sample_out;

__device__ __forceinline__ unsigned long long sp_key(float p, int token) {
  return ((unsigned long long)__float_as_uint(p) << 32) | (0xFFFFFFFFu - (unsigned)token);
}
__device__ __forceinline__ int sp_share(int n, int ctas, int c, int* hi) {
  const int per = (n + ctas - 1) / ctas;
  const int lo = min(n, c * per);
  *hi = min(n, lo + per);
  return lo;
}

__global__ void sample_max_kernel(const float* __restrict__ x, int n) {
  int hi;
  const int lo = sp_share(n, gridDim.x, blockIdx.x, &hi);
  float best = -INFINITY;
  bool nan = false;
  for (int i = lo + threadIdx.x; i < hi; i += SP_THREADS) {
    const float v = x[i];
    nan |= v != v;
    best = fmaxf(best, v);
  }
  best = warp_max(best);
  nan = __any_sync(0xffffffffu, nan);
  __shared__ float wm[SP_THREADS / 32];
  __shared__ int wn[SP_THREADS / 32];
  if ((threadIdx.x & 31) == 0) {
    wm[threadIdx.x >> 5] = best;
    wn[threadIdx.x >> 5] = nan;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < SP_THREADS / 32; w++) {
      best = fmaxf(best, wm[w]);
      nan |= wn[w] != 0;
    }
    g_sample.part_max[blockIdx.x] = nan ? __int_as_float(0x7fc00000) : best;
  }
}

// the largest logit from the CTAs' maxima (NaN if any was)
__device__ float sp_best(int ctas) {
  __shared__ float b;
  if (threadIdx.x == 0) {
    float best = -INFINITY;
    bool nan = false;
    for (int c = 0; c < ctas; c++) {
      const float v = g_sample.part_max[c];
      nan |= v != v;
      best = fmaxf(best, v);
    }
    b = nan ? __int_as_float(0x7fc00000) : best;
  }
  __syncthreads();
  return b;
}

__device__ __forceinline__ float sp_floor(float best, float temperature, float topp) {
  return (topp > 0.0f && topp < 1.0f) ? best - temperature * 16.118095f : -FLT_MAX;
}

__global__ void sample_count_kernel(const float* __restrict__ x, int n, float temperature, float topp) {
  const float best = sp_best(gridDim.x);
  if (!isfinite(best)) return;
  const float fl = sp_floor(best, temperature, topp);
  int hi;
  const int lo = sp_share(n, gridDim.x, blockIdx.x, &hi);
  int c = 0;
  for (int i = lo + threadIdx.x; i < hi; i += SP_THREADS) c += x[i] >= fl;
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  __shared__ int wc[SP_THREADS / 32];
  if ((threadIdx.x & 31) == 0) wc[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < SP_THREADS / 32; w++) c += wc[w];
    g_sample.counts[blockIdx.x] = c;
  }
}

// this CTA's candidates in token order behind the earlier CTAs' counts: probs = x - best, index = the token
__global__ void sample_scatter_kernel(const float* __restrict__ x, int n, float temperature, float topp, float* probs,
                                      int* index) {
  const float best = sp_best(gridDim.x);
  if (!isfinite(best)) return;
  const float fl = sp_floor(best, temperature, topp);
  __shared__ int base, wc[SP_THREADS / 32];
  if (threadIdx.x == 0) {
    int s = 0;
    for (int c = 0; c < (int)blockIdx.x; c++) s += g_sample.counts[c];
    base = s;
  }
  __syncthreads();
  int hi;
  const int lo = sp_share(n, gridDim.x, blockIdx.x, &hi);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int t0 = lo; t0 < hi; t0 += SP_THREADS) {
    const int i = t0 + threadIdx.x;
    const float v = i < hi ? x[i] : 0.0f;
    const bool keep = i < hi && v >= fl;
    const unsigned m = __ballot_sync(0xffffffffu, keep);
    if (lane == 0) wc[warp] = __popc(m);
    __syncthreads();
    int before = 0, all = 0;
    for (int w = 0; w < SP_THREADS / 32; w++) {
      before += w < warp ? wc[w] : 0;
      all += wc[w];
    }
    if (keep) {
      const int at = base + before + __popc(m & ((1u << lane) - 1));
      probs[at] = v - best;
      index[at] = i;
    }
    __syncthreads();
    if (threadIdx.x == 0) base += all;
    __syncthreads();
  }
}

__device__ double sp_sum(double v, double* red) {  // a block's sum (every thread gets it)
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    double s = threadIdx.x < SP_FINAL / 32 ? red[threadIdx.x] : 0.0;
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) red[32] = s;
  }
  __syncthreads();
  return red[32];
}
__device__ float sp_fmax(float v, float* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float s = threadIdx.x < SP_FINAL / 32 ? red[threadIdx.x] : -INFINITY;
    s = warp_max(s);
    if (threadIdx.x == 0) red[32] = s;
  }
  __syncthreads();
  return red[32];
}

// the rank-th largest (rank from 1) key among the elements where in(i) holds and key < upper: a radix select, 8 bits a
// pass from the top (every thread returns it); none: 0
template <typename In>
__device__ unsigned long long sp_select(const float* probs, const int* index, int count, In in, unsigned long long upper,
                                        int rank, unsigned* hist) {
  unsigned long long prefix = 0, mask = 0;
  for (int shift = 56; shift >= 0; shift -= 8) {
    for (int b = threadIdx.x; b < 256; b += SP_FINAL) hist[b] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < count; i += SP_FINAL) {
      if (!in(i)) continue;
      const unsigned long long k = sp_key(probs[i], index[i]);
      if (k >= upper || (k & mask) != prefix) continue;
      atomicAdd(&hist[(k >> shift) & 255], 1u);
    }
    __syncthreads();
    __shared__ int pick, left;
    if (threadIdx.x == 0) {
      int r = rank, b = 255;
      for (; b >= 0; b--) {
        if ((int)hist[b] >= r) break;
        r -= hist[b];
      }
      pick = b;
      left = r;
    }
    __syncthreads();
    if (pick < 0) return 0;
    prefix |= (unsigned long long)pick << shift;
    mask |= 255ull << shift;
    rank = left;
    __syncthreads();
  }
  return prefix;
}

// the elements of the set with lo <= key < upper (at most SP_CHUNK of them) into shared memory, sorted descending
// (a bitonic sort of the next power of two of them); returns how many
template <typename In>
__device__ int sp_chunk(const float* probs, const int* index, int count, In in, unsigned long long lo,
                        unsigned long long upper, unsigned long long* keys, int* fill) {
  if (threadIdx.x == 0) *fill = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < count; i += SP_FINAL) {
    if (!in(i)) continue;
    const unsigned long long k = sp_key(probs[i], index[i]);
    if (k >= lo && k < upper) {
      const int at = atomicAdd(fill, 1);
      if (at < SP_CHUNK) keys[at] = k;
    }
  }
  __syncthreads();
  const int m = min(*fill, SP_CHUNK);
  int width = 32;
  while (width < m) width <<= 1;
  for (int i = m + threadIdx.x; i < width; i += SP_FINAL) keys[i] = 0;  // padding sorts last
  __syncthreads();
  for (int size = 2; size <= width; size <<= 1)  // bitonic sort, descending
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = threadIdx.x; i < width; i += SP_FINAL) {
        const int j = i ^ stride;
        if (j > i) {
          const bool down = (i & size) == 0;
          const unsigned long long a = keys[i], b = keys[j];
          if (down ? a < b : a > b) {
            keys[i] = b;
            keys[j] = a;
          }
        }
      }
      __syncthreads();
    }
  return m;
}

__device__ __forceinline__ float sp_prob(unsigned long long k) { return __uint_as_float((unsigned)(k >> 32)); }
__device__ __forceinline__ int sp_token(unsigned long long k) { return (int)(0xFFFFFFFFu - (unsigned)k); }

__global__ void __launch_bounds__(SP_FINAL) sample_final_kernel(int ctas, float temperature, float topp,
                                                                 const double* random_dev, double random_val, int topk,
                                                                 float minp, float* probs, const int* index, int* out) {
  __shared__ double red[33];
  __shared__ float redf[33];
  __shared__ unsigned hist[256];
  extern __shared__ unsigned long long keys[];  // [SP_CHUNK]
  __shared__ int fill, result;
  const float best = sp_best(ctas);
  if (!isfinite(best)) {
    if (threadIdx.x == 0) *out = -1;
    return;
  }
  const double random = random_dev ? *random_dev : random_val;
  int count = 0;
  for (int c = 0; c < ctas; c++) count += g_sample.counts[c];
  const bool nucleus = topp > 0.0f && topp < 1.0f;
  const int fours = count / 4 * 4;
  const float inverse = 1.0f / temperature;
  double s = 0.0;
  float top = 0.0f;
  for (int i = threadIdx.x; i < count; i += SP_FINAL) {
    const float x = probs[i];
    float p;
    if (i < fours) {
      p = expf(fminf(fmaxf(x * inverse, -87.0f), 88.0f));
    } else {
      const float y = x / temperature;
      p = y < -87.0f ? 0.0f : expf(fminf(y, 88.0f));
    }
    probs[i] = p;
    s += p;
    top = fmaxf(top, p);
  }
  double total = sp_sum(s, red);
  top = sp_fmax(top, redf);
  const bool narrowed = topk > 0 && topk < count;
  unsigned long long kth = 0;  // narrowed: the top-k's smallest key
  if (narrowed) {
    kth = sp_select(probs, index, count, [](int) { return true; }, ~0ull, topk, hist);
    s = 0.0;
    for (int i = threadIdx.x; i < count; i += SP_FINAL)
      if (sp_key(probs[i], index[i]) >= kth) s += probs[i];
    total = sp_sum(s, red);
  }
  const int live = narrowed ? topk : count;
  const float least = minp > 0.0f ? fminf(minp, 1.0f) * top : 0.0f;
  if (nucleus || narrowed) {
    const double c0 = (1.0 - (double)topp) / (double)(live > 1 ? live - 1 : 1) * total;
    const double cutoff = nucleus ? fmin(c0, (double)top) : 0.0;
    auto in = [&](int i) {
      const float p = probs[i];
      return (!narrowed || sp_key(p, index[i]) >= kth) && (double)p >= cutoff && p >= least;
    };
    const double limit = nucleus ? (double)topp * total : INFINITY;
    __shared__ double mass;
    __shared__ unsigned long long last_key;
    __shared__ bool done;
    // The walk's keys at once where they fit in one chunk: a histogram of the set's mass by probability (the float's
    // top 11 bits), summed from the most probable bin down to the first bin where the mass passes the limit (by a
    // relative 1e-9 more than the walk's own sums could differ by), names a floor that holds every key the walk can
    // reach; the keys at or above it, sorted once, are walked for both passes in the same descending order as the
    // chunk-by-chunk walk below, so the same sums, the same token (each of those chunks is a full scan of the
    // candidates: a draw with a wide nucleus took ~100 scans).
    {
      __shared__ double hmass[1024];
      __shared__ unsigned hcount[1024];
      __shared__ int lo_bin, fits;
      for (int b = threadIdx.x; b < 1024; b += SP_FINAL) {
        hmass[b] = 0.0;
        hcount[b] = 0;
      }
      __syncthreads();
      for (int i = threadIdx.x; i < count; i += SP_FINAL) {
        if (!in(i)) continue;
        const float p = probs[i];
        const int b = (int)(__float_as_uint(p) >> 21) & 1023;  // p >= 0: its bits' order is its order
        atomicAdd(&hmass[b], (double)p);
        atomicAdd(&hcount[b], 1u);
      }
      __syncthreads();
      if (threadIdx.x == 0) {
        double cum = 0.0;
        unsigned n = 0;
        int lo = 0;
        for (int b = 1023; b >= 0; b--) {
          cum += hmass[b];
          n += hcount[b];
          if (cum >= limit * (1.0 + 1e-9)) {
            lo = b;
            break;
          }
        }
        lo_bin = lo;
        fits = n <= (unsigned)SP_CHUNK;
      }
      __syncthreads();
      if (fits) {
        const unsigned long long lo_key = (unsigned long long)((unsigned)lo_bin << 21) << 32;
        const int m = sp_chunk(probs, index, count, in, lo_key, ~0ull, keys, &fill);
        if (threadIdx.x == 0) {
          double walked = 0.0;
          unsigned long long last = 0;
          for (int k = 0; k < m; k++) {  // pass 1: the nucleus's mass and its last key
            walked += sp_prob(keys[k]);
            last = keys[k];
            if (walked >= limit) break;
          }
          const double target = random * walked;  // pass 2: the first whose cumulative sum passes random x mass
          int pick = sp_token(last);
          double cumulative = 0.0;
          for (int k = 0; k < m; k++) {
            cumulative += sp_prob(keys[k]);
            if (cumulative > target) {
              pick = sp_token(keys[k]);
              break;
            }
            if (keys[k] == last) break;
          }
          *out = pick;
        }
        return;
      }
    }
    // pass 1: the nucleus's mass and its last key, chunk by chunk from the most probable
    if (threadIdx.x == 0) {
      mass = 0.0;
      last_key = 0;
      done = false;
    }
    __syncthreads();
    unsigned long long upper = ~0ull;
    while (!done) {
      const unsigned long long lo = sp_select(probs, index, count, in, upper, SP_CHUNK, hist);
      const int m = sp_chunk(probs, index, count, in, lo, upper, keys, &fill);
      if (threadIdx.x == 0) {
        for (int k = 0; k < m; k++) {
          mass += sp_prob(keys[k]);
          last_key = keys[k];
          if (mass >= limit) {
            done = true;
            break;
          }
        }
        if (lo == 0 || m == 0) done = true;  // the set is walked whole
      }
      __syncthreads();
      upper = lo;
    }
    // pass 2: the first whose cumulative sum passes random x mass, from the most probable (else the last)
    const double target = random * mass;
    if (threadIdx.x == 0) {
      result = sp_token(last_key);
      done = false;
    }
    __syncthreads();
    double cumulative = 0.0;
    upper = ~0ull;
    while (!done) {
      const unsigned long long lo = sp_select(probs, index, count, in, upper, SP_CHUNK, hist);
      const int m = sp_chunk(probs, index, count, in, lo, upper, keys, &fill);
      if (threadIdx.x == 0) {
        for (int k = 0; k < m && !done; k++) {
          cumulative += sp_prob(keys[k]);
          if (cumulative > target) {
            result = sp_token(keys[k]);
            done = true;
          }
          if (keys[k] == last_key) done = true;
        }
        if (lo == 0 || m == 0) done = true;
      }
      __syncthreads();
      upper = lo;
    }
    if (threadIdx.x == 0) *out = result;
    return;
  }
  // token order: every candidate, or those at or above least; a thread a contiguous part
  const int per = (count + SP_FINAL - 1) / SP_FINAL;
  const int a = min(count, (int)threadIdx.x * per), b = min(count, a + per);
  double part = 0.0;
  int mine_last = -1;
  for (int i = a; i < b; i++)
    if (probs[i] >= least) {
      part += probs[i];
      mine_last = i;
    }
  // the parts' exclusive scan (in thread order) and their total
  __shared__ double scan[SP_FINAL];
  __shared__ int lastv[SP_FINAL];
  scan[threadIdx.x] = part;
  lastv[threadIdx.x] = mine_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    double run = 0.0;
    int lastc = -1;
    for (int t = 0; t < SP_FINAL; t++) {
      const double v = scan[t];
      scan[t] = run;
      run += v;
      lastc = lastv[t] >= 0 ? lastv[t] : lastc;
    }
    red[32] = run;
    result = lastc >= 0 ? index[lastc] : -1;
    fill = 0;
  }
  __syncthreads();
  const double target = random * red[32];
  double cumulative = scan[threadIdx.x];
  if (cumulative <= target && cumulative + part > target) {
    for (int i = a; i < b; i++) {
      if (probs[i] < least) continue;
      cumulative += probs[i];
      if (cumulative > target) {
        if (atomicAdd(&fill, 1) == 0) result = index[i];
        break;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *out = result;
}

int sample_ctas(int n) {
  int c = (n + 4095) / 4096;
  return c < 1 ? 1 : (c > SP_MAX_CTAS ? SP_MAX_CTAS : c);
}

bool sample_enqueue(const float* x, int n, float temperature, float topp, const double* random_dev, double random,
                    int topk, float minp, float* probs, int* index, int* out) {
  const int ctas = sample_ctas(n);
  cudaStream_t s = pllm_stream();
  sample_max_kernel<<<ctas, SP_THREADS, 0, s>>>(x, n);
  sample_count_kernel<<<ctas, SP_THREADS, 0, s>>>(x, n, temperature, topp);
  sample_scatter_kernel<<<ctas, SP_THREADS, 0, s>>>(x, n, temperature, topp, probs, index);
  static bool sized[64] = {false};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  if (!sized[dev]) {  // the key buffer's dynamic shared memory, set once a device (outside any stream capture)
    if (cudaFuncSetAttribute(sample_final_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             SP_CHUNK * (int)sizeof(unsigned long long)) != cudaSuccess)
      return false;
    sized[dev] = true;
  }
  sample_final_kernel<<<1, SP_FINAL, SP_CHUNK * sizeof(unsigned long long), s>>>(ctas, temperature, topp, random_dev,
                                                                               random, topk, minp, probs, index, out);
  return cudaGetLastError() == cudaSuccess;
}

}  // namespace

// sample (sample.ts:248): the token drawn by random in [0, 1) (-1: the largest logit is not a finite number); probs and
// index: device scratch of n floats and n int32
PLLM_API int32_t sample(uint64_t logits, int32_t n, float temperature, float topp, double random, uint64_t probs,
                        uint64_t index, int32_t topk, float minp) {
  PLLM_REQUIRE_RET(logits && probs && index && n > 0 && temperature > 0.0f, -1, "sample: n %d temperature %g", n,
                   (double)temperature);
  std::lock_guard<std::mutex> hold(pllm_scratch_lock());
  void* out = nullptr;
  if (cudaGetSymbolAddress(&out, g_sample_out) != cudaSuccess ||
      !sample_enqueue(dptr<const float>(logits), n, temperature, topp, nullptr, random, topk, minp, dptr<float>(probs),
                      dptr<int>(index), (int*)out)) {
    pllm_fail(PLLM_ECUDA, "sample: launch");
    return -1;
  }
  int token = -1;
  const cudaError_t e = cudaMemcpyAsync(&token, out, sizeof token, cudaMemcpyDeviceToHost, pllm_stream());
  if (e != cudaSuccess || cudaStreamSynchronize(pllm_stream()) != cudaSuccess) {
    pllm_fail(PLLM_ECUDA, "sample: %s", cudaGetErrorString(e));
    return -1;
  }
  return token;
}

// the same into device memory without waiting (a recorded step): out one int32, the random number a double in device
// memory (written before the step runs)
PLLM_API void pllm_sample_dev(uint64_t out, uint64_t logits, int32_t n, float temperature, float topp,
                              uint64_t random_dev, uint64_t probs, uint64_t index, int32_t topk, float minp) {
  PLLM_REQUIRE(out && logits && probs && index && random_dev && n > 0 && temperature > 0.0f,
               "pllm_sample_dev: n %d temperature %g", n, (double)temperature);
  if (!sample_enqueue(dptr<const float>(logits), n, temperature, topp, dptr<const double>(random_dev), 0.0, topk, minp,
                      dptr<float>(probs), dptr<int>(index), dptr<int>(out)))
    pllm_fail(PLLM_ECUDA, "pllm_sample_dev: launch");
}
