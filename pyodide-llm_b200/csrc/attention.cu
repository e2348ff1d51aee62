// attention.cu: RoPE, the cache write, and one token's attention over the cache (kernels/kernel/attention.ts).
//   rope                       attention.ts:7-20
//   attention, attention_f16   attention.ts:28-36 (attentionOf :87-211)
//   attention_capped, attention_f16_capped   attention.ts:40-45
// The cache is the reference's layout: a layer's keys (and values) [position][kv heads * head size], float32 or the
// float16 bits halves.ts writes. Grouped-query: q head h reads kv head h / (nh / nkv).
//
// B200 form: split-KV ("flash decoding"). A CTA takes one kv head and a slice of the positions for all of that head's
// query heads (the keys and values of the slice are read once for kvMul heads) and makes the slice's partial result
// (max, sum, weighted values a head): float16 caches on the tensor cores, a warp per 16-position chunk with its own
// online softmax; float32 caches by scalar float32 products over 64-position tiles. The last CTA of a kv head to
// finish combines the slices (the forward driver's calls), or a second small kernel does (the registry's calls).
// With one slice the first kernel writes the output itself.
// The numbers differ from the reference's in the order of the float32 sums and in exp (CUDA's expf in place of the
// reference's table-free one): the outputs agree within float32 rounding (the tests hold them to 1e-5 relative).
//
// The forward driver's calls read the position from device memory (pos_dev), so that one CUDA graph serves every
// position; their grid covers the cache's capacity and the slices past the position return at once.
#include <cooperative_groups.h>

#include "pllm_common.cuh"

namespace gemvk {
int* status_word();  // the device status word's address on the current device (gemv_tma.cu)
}

namespace {

constexpr int ATT_THREADS = 128, ATT_WARPS = ATT_THREADS / 32;

struct AttArgs {
  float* out;
  const float* q;
  const void* kc;
  const void* vc;
  float* part;          // slices' partials: [nh][nsplit][hs + 4] (weighted values, max, sum, 2 floats of pad)
  const int* pos_dev;   // device position (or null: pos)
  int pos, nh, nkv, hs, h0, h1;
  int split_len;        // positions a slice
  int nsplit;           // slices (the grid's y); with pos_dev, those past the position return
  float cap;
  int* counters;        // [nkv] slices done, zero between calls; null: a second kernel combines the slices
  int cs;               // the chunk kernel's cluster size (its CL form), 2..CS_MAX
  // a batch of sequences (grid z; 1 for one): sequence z's out, q (and the Fuse's k, v), cache, partials and counts
  // are these strides after sequence 0's (floats; the cache in bytes; the counts with the partials, in 4-byte
  // words), and its position is pos_dev[z]
  int batch;
  long long z_out, z_q, z_kv, z_part;
  int capacity;         // the cache's positions (a device position past them is held at the last: see position())
  int* status;          // the device status word (PLLM_ERANGE: a device position out of the cache)
};

// the call's position: the host's, or the one in device memory held inside the cache (a position below 0 or past the
// cache's capacity is taken as the first or last row and reported in the status word as PLLM_ERANGE, so that no
// read or write leaves the cache or the rope tables)
__device__ __forceinline__ int position(const AttArgs& a) {
  if (!a.pos_dev) return a.pos;
  const int pos = *a.pos_dev;
  if (pos >= 0 && pos < a.capacity) return pos;
  if (a.status && threadIdx.x == 0) atomicExch(a.status, PLLM_ERANGE);
  return pos < 0 ? 0 : a.capacity - 1;
}

// sequence z's arguments (grid z) from sequence 0's, each array assigned from the launch's own argument
__device__ __forceinline__ AttArgs sequence_of(const AttArgs& a0, int z) {
  AttArgs a = a0;
  const long long zz = z;
  a.out = a0.out + zz * a0.z_out;
  a.q = a0.q + zz * a0.z_q;
  a.kc = reinterpret_cast<const uint8_t*>(a0.kc) + zz * a0.z_kv;
  a.vc = reinterpret_cast<const uint8_t*>(a0.vc) + zz * a0.z_kv;
  a.pos_dev = a0.pos_dev ? a0.pos_dev + zz : nullptr;
  a.part = a0.part ? a0.part + zz * a0.z_part : nullptr;
  a.counters = a0.counters ? a0.counters + zz * a0.z_part : nullptr;
  return a;
}


// What the forward driver's attention does before it reads the cache (FUSE): the per-head RMSNorm of q and k
// (Qwen3's q_norm / k_norm, forward/attention.ts:140-143), RoPE at the position (kernels/kernel/attention.ts:7-20
// with the tables' row of pos), and this position's key and value into the cache (halves.ts:35-67's rounding for a
// float16 cache). Every CTA makes its own query heads; the CTA whose slice holds the position also makes the key and
// value of its kv head, writes them to the cache and into its shared tile.
struct Fuse {
  const float* k;       // this token's keys (nkv heads) and values, as the q/k/v product wrote them
  const float* v;
  const float* qn;      // q_norm / k_norm (null: none)
  const float* kn;
  const float* cos_t;   // [capacity][hs / 2]
  const float* sin_t;
  float eps;
  int rot;
  int* bad;             // non-finite keys or values written to a float16 cache are counted here (may be null)
};

__device__ __forceinline__ Fuse sequence_of(const Fuse& f0, const AttArgs& a0, int z) {
  Fuse f = f0;
  f.k = f0.k ? f0.k + (long long)z * a0.z_q : nullptr;
  f.v = f0.v ? f0.v + (long long)z * a0.z_q : nullptr;
  return f;
}

// tensor-core helpers (float16 caches): ldmatrix fragments and the m16n8k16 product with float32 accumulation
__device__ __forceinline__ void ldsm_x4(uint32_t r[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t r[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void mma16816(float c[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// x as the sum of two float16: hi = rn(x), lo = rn(x - hi) (the products of a float16 key or value with both are
// exact in the float32 accumulation, so the sum keeps x to about 2^-22 of itself)
__device__ __forceinline__ uint32_t pack_halves(__half lo16, __half hi16) {
  return (uint32_t)__half_as_ushort(lo16) | ((uint32_t)__half_as_ushort(hi16) << 16);
}
__device__ __forceinline__ void split_half(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn(x - __half2float(hi));
}

__device__ __forceinline__ uint32_t lds32(const __half* p) { return *reinterpret_cast<const uint32_t*>(p); }

// The last slice of a kv head to finish combines every slice's partials (no CTA waits for another: the others are
// done when the count reaches nsplit) and sets the count back to zero for the next call. The partials of the kv
// head's query heads are contiguous: copied into shared memory (stage, stage_bytes) by asynchronous 16-byte copies,
// as many slices at once as it holds (every copy of a chunk in flight together). sw: KVM x nsplit floats for the
// slices' weights exp(m_s - M); sL: KVM floats.
template <int KVM, int THREADS>
__device__ __forceinline__ void combine_slices(const AttArgs& a, int kvh, int nsplit, uint8_t* stage_mem,
                                               size_t stage_bytes, float* sw, float* sL) {
  __shared__ int last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  __syncthreads();  // every partial of this CTA is written; one fence orders them before the count (cumulativity)
  if (tid == 0) {
    __threadfence();
    last = atomicAdd(&a.counters[kvh], 1) == nsplit - 1;
    __threadfence();
  }
  __syncthreads();
  if (!last) return;
  const int hs = a.hs, hbase = kvh * KVM;
  const int row = hs + 4;  // floats a slice's partial (16-byte rows)
  const int room = (int)(stage_bytes / ((size_t)KVM * row * 4));
  float* stage = reinterpret_cast<float*>(stage_mem);
  constexpr int PMAX = (KVM * 256 + THREADS - 1) / THREADS;  // (head, dimension) pairs a thread (hs <= 256)
  float o[PMAX];
#pragma unroll
  for (int k = 0; k < PMAX; k++) o[k] = 0.0f;
  for (int c0 = 0; c0 < nsplit; c0 += room) {
    const int cn = min(room, nsplit - c0);
    const int per4 = cn * row / 4;  // 16-byte pieces a head's chunk
    __syncthreads();                // the previous chunk is read
    for (int e = tid; e < KVM * per4; e += THREADS) {
      const int j = e / per4, f4 = e % per4;
      cp_async16(stage + 4 * e, a.part + ((long long)(hbase + j) * a.nsplit + c0) * row + 4 * f4);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    cp_async_wait_all();
    __syncthreads();
    if (c0 == 0) {  // the maxima and sums of every slice (the first chunk holds them when room >= nsplit; else L2)
      for (int j = warp; j < KVM; j += THREADS / 32) {
        float M = -INFINITY;
        for (int s2 = lane; s2 < nsplit; s2 += 32) {
          const float m = s2 < cn ? stage[(j * cn + s2) * row + hs]
                                  : __ldcg(a.part + ((long long)(hbase + j) * a.nsplit + s2) * row + hs);
          sw[j * nsplit + s2] = m;
          M = fmaxf(M, m);
        }
        M = warp_max(M);
        float Ls = 0.0f;
        for (int s2 = lane; s2 < nsplit; s2 += 32) {
          const float w = expf(sw[j * nsplit + s2] - M);
          sw[j * nsplit + s2] = w;
          const float l = s2 < cn ? stage[(j * cn + s2) * row + hs + 1]
                                  : __ldcg(a.part + ((long long)(hbase + j) * a.nsplit + s2) * row + hs + 1);
          Ls = fmaf(l, w, Ls);
        }
        Ls = warp_sum(Ls);
        if (lane == 0) sL[j] = Ls;
      }
      __syncthreads();
    }
#pragma unroll
    for (int k = 0; k < PMAX; k++) {
      const int e = tid + THREADS * k;
      if (e >= KVM * hs) break;
      const int j = e / hs, d = e % hs;
      float acc = o[k];
      for (int s2 = 0; s2 < cn; s2++) acc = fmaf(stage[(j * cn + s2) * row + d], sw[j * nsplit + c0 + s2], acc);
      o[k] = acc;
    }
  }
#pragma unroll
  for (int k = 0; k < PMAX; k++) {
    const int e = tid + THREADS * k;
    if (e >= KVM * hs) break;
    const int j = e / hs, d = e % hs, h = hbase + j;
    if (h >= a.h0 && h < a.h1) a.out[(long long)h * hs + d] = o[k] / sL[j];
  }
  if (tid == 0) a.counters[kvh] = 0;
}

// ---- float32 caches
// grid (nkv, nsplit): one kv head's slice of positions for its KVM query heads, taken TILE positions at a time: every
// thread first issues its 16-byte copies of the tile's keys and values (all of them in flight at once) into shared
// memory (rows padded by 16 bytes: conflict-free 16-byte reads of a row by consecutive threads), then the scores (a
// thread a position and head pair), an online softmax of the slice (running max and sum, the partial output
// rescaled), and the weighted values (a thread a head dimension).
constexpr int TILE = 64;

// a head of hs floats in shared memory normalized (w: null for none) and turned at pos by one warp
__device__ __forceinline__ void norm_rope_warp(float* x, const float* w, const Fuse& f, int hs, int pos) {
  const int lane = threadIdx.x & 31;
  if (w) {
    float s = 0.0f;
    for (int d = lane; d < hs; d += 32) s = fmaf(x[d], x[d], s);
    s = warp_sum(s);
    const float r = 1.0f / sqrtf(s / (float)hs + f.eps);
    for (int d = lane; d < hs; d += 32) x[d] = w[d] * (r * x[d]);
    __syncwarp();
  }
  const int turned = f.rot > 0 && f.rot < hs ? f.rot : hs;
  const float* c = f.cos_t + (long long)pos * (hs / 2);
  const float* sn = f.sin_t + (long long)pos * (hs / 2);
  for (int i = lane; i < turned / 2; i += 32) {
    const float v0 = x[2 * i], v1 = x[2 * i + 1];
    x[2 * i] = v0 * c[i] - v1 * sn[i];
    x[2 * i + 1] = v0 * sn[i] + v1 * c[i];
  }
  __syncwarp();
}

template <int KVM, bool FUSE>
__global__ void __launch_bounds__(ATT_THREADS) attention_f32_kernel(const AttArgs a, const Fuse f) {
  extern __shared__ __align__(16) uint8_t att_smem[];
  const int hs = a.hs;
  const int rowb = hs * 4 + 16;                      // a padded row of the tile, bytes
  const int tileb = TILE * rowb;
  uint8_t* ring = att_smem;                          // [2 buffers][K tile, V tile]: 4 x tileb bytes
  float* sq = reinterpret_cast<float*>(ring + 4 * tileb);  // [KVM][hs]
  float* sx = sq + KVM * hs;                         // [2][hs] (FUSE) this position's key and value
  float* sp = sx + 2 * hs;                           // [KVM][TILE] scores, then probabilities; the combine's weights
  __shared__ float sM[KVM], sL[KVM], sScale[KVM];
  pdl_launch_dependents();  // the next kernel waits for this one's completion; its CTAs may take the SMs this one leaves
  // the position: written by the host before the step's first kernel, so readable before the dependency wait
  const int pos = position(a);
  const int count = pos + 1;
  const int kvh = blockIdx.x, split = blockIdx.y;
  const int nsplit = a.pos_dev ? (count + a.split_len - 1) / a.split_len : a.nsplit;
  if (split >= nsplit) return;
  const int p0 = split * a.split_len;
  const int p1 = min(count, p0 + a.split_len);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kvdim = a.nkv * hs, hbase = kvh * KVM;
  const float isq = 1.0f / sqrtf((float)hs);
  const int chunks = hs / 4;                         // 16-byte pieces a row
  const uint8_t* kbase = reinterpret_cast<const uint8_t*>(a.kc) + (long long)kvh * hs * 4;
  const uint8_t* vbase = reinterpret_cast<const uint8_t*>(a.vc) + (long long)kvh * hs * 4;
  // a tile's keys and values by asynchronous 16-byte copies, all in flight at once (positions before this token's:
  // not the previous kernel's output); rows past the tile's length zeroed (a probability of 0 must meet a 0)
  auto load_tile = [&](int t0, int buf) {
    uint8_t* sK = ring + (size_t)(2 * buf) * tileb;
    uint8_t* sV = sK + tileb;
    const int len = min(TILE, p1 - t0);
    for (int e = tid; e < TILE * chunks; e += ATT_THREADS) {
      const int t = e / chunks, c = e % chunks;
      if (t < len) {
        const long long off = (long long)(t0 + t) * kvdim * 4 + c * 16;
        cp_async16(sK + t * rowb + c * 16, kbase + off);
        cp_async16(sV + t * rowb + c * 16, vbase + off);
      } else {
        *reinterpret_cast<int4*>(sK + t * rowb + c * 16) = make_int4(0, 0, 0, 0);
        *reinterpret_cast<int4*>(sV + t * rowb + c * 16) = make_int4(0, 0, 0, 0);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  load_tile(p0, 0);  // before the wait: it overlaps the kernel ahead's tail
  if (p0 + TILE < p1) load_tile(p0 + TILE, 1);
  pdl_wait();
  for (int e = tid; e < KVM * hs; e += ATT_THREADS) sq[e] = a.q[(long long)hbase * hs + e];
  if (tid < KVM) {
    sM[tid] = -INFINITY;
    sL[tid] = 0.0f;
  }
  const bool holds_pos = FUSE && p1 == count;
  if (FUSE && holds_pos)
    for (int d = tid; d < hs; d += ATT_THREADS) {
      sx[d] = f.k[(long long)kvh * hs + d];
      sx[hs + d] = f.v[(long long)kvh * hs + d];
    }
  __syncthreads();
  if (FUSE) {  // the heads' norms and RoPE, a warp a head; the key's too where this slice holds the position
    for (int j = warp; j < KVM + (holds_pos ? 1 : 0); j += ATT_WARPS) {
      if (j < KVM) norm_rope_warp(sq + j * hs, f.qn, f, hs, pos);
      else norm_rope_warp(sx, f.kn, f, hs, pos);
    }
    __syncthreads();
    if (holds_pos)  // this position's key and value into the cache
      for (int e = tid; e < 2 * hs; e += ATT_THREADS) {
        float* cache = reinterpret_cast<float*>(const_cast<void*>(e < hs ? a.kc : a.vc));
        cache[(long long)pos * kvdim + (long long)kvh * hs + e % hs] = sx[e];
      }
  }
  float acc[KVM][2];  // a thread a dimension d = tid + ATT_THREADS i of every head (hs <= 256)
#pragma unroll
  for (int j = 0; j < KVM; j++) acc[j][0] = acc[j][1] = 0.0f;
  int buf = 0;
  for (int t0 = p0; t0 < p1; t0 += TILE, buf ^= 1) {
    const int len = min(TILE, p1 - t0);
    uint8_t* sK = ring + (size_t)(2 * buf) * tileb;
    uint8_t* sV = sK + tileb;
    // this tile's copies are done when at most the next tile's group is still in flight
    if (t0 + TILE < p1) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else cp_async_wait_all();
    __syncthreads();
    if (holds_pos && pos >= t0 && pos < t0 + len) {  // this position's row: the fresh key and value
      for (int e = tid; e < 2 * hs; e += ATT_THREADS)
        reinterpret_cast<float*>((e < hs ? sK : sV) + (size_t)(pos - t0) * rowb)[e % hs] = sx[e];
      __syncthreads();
    }
    // scores: a thread a (position, head) pair
    for (int e = tid; e < KVM * TILE; e += ATT_THREADS) {
      const int t = e % TILE, j = e / TILE;
      float sc = -INFINITY;
      if (t < len) {
        const uint8_t* row = sK + t * rowb;
        const float* qj = sq + j * hs;
        sc = 0.0f;
        for (int c = 0; c < chunks; c++) {
          const float4 w = *reinterpret_cast<const float4*>(row + c * 16);
          sc = fmaf(qj[c * 4], w.x, sc);
          sc = fmaf(qj[c * 4 + 1], w.y, sc);
          sc = fmaf(qj[c * 4 + 2], w.z, sc);
          sc = fmaf(qj[c * 4 + 3], w.w, sc);
        }
        sc *= isq;
        if (a.cap > 0.0f) sc = a.cap * tanhf(sc / a.cap);
      }
      sp[j * TILE + t] = sc;
    }
    __syncthreads();
    // the online softmax: a warp a head
    for (int j = warp; j < KVM; j += ATT_WARPS) {
      float m = -INFINITY;
      for (int t = lane; t < len; t += 32) m = fmaxf(m, sp[j * TILE + t]);
      m = warp_max(m);
      const float mnew = fmaxf(sM[j], m);
      float l = 0.0f;
      for (int t = lane; t < TILE; t += 32) {
        const float p = t < len ? expf(sp[j * TILE + t] - mnew) : 0.0f;
        sp[j * TILE + t] = p;
        l += p;
      }
      l = warp_sum(l);
      if (lane == 0) {
        const float scale = expf(sM[j] - mnew);  // 0 at the first tile (exp(-inf))
        sScale[j] = scale;
        sL[j] = sL[j] * scale + l;
        sM[j] = mnew;
      }
    }
    __syncthreads();
    // the weighted values: a thread a dimension
#pragma unroll
    for (int i = 0; i < 2; i++) {
      const int d = tid + ATT_THREADS * i;
      if (d >= hs) continue;
#pragma unroll
      for (int j = 0; j < KVM; j++) acc[j][i] *= sScale[j];
      for (int t = 0; t < len; t++) {
        const float v = reinterpret_cast<const float*>(sV + t * rowb)[d];
#pragma unroll
        for (int j = 0; j < KVM; j++) acc[j][i] = fmaf(sp[j * TILE + t], v, acc[j][i]);
      }
    }
    // the tile after next into this buffer, once every warp is done with it
    if (t0 + 2 * TILE < p1) {
      __syncthreads();
      load_tile(t0 + 2 * TILE, buf);
    }
  }
  // the slice's output (one slice: the head's output itself)
#pragma unroll
  for (int i = 0; i < 2; i++) {
    const int d = tid + ATT_THREADS * i;
    if (d >= hs) continue;
#pragma unroll
    for (int j = 0; j < KVM; j++) {
      const int h = hbase + j;
      if (h < a.h0 || h >= a.h1) continue;
      if (nsplit == 1) {
        a.out[(long long)h * hs + d] = acc[j][i] / sL[j];
      } else {
        float* part = a.part + ((long long)h * a.nsplit + split) * (hs + 4);
        part[d] = acc[j][i];
        if (d == 0) {
          part[hs] = sM[j];
          part[hs + 1] = sL[j];
        }
      }
    }
  }
  if (nsplit == 1 || !a.counters) return;
  combine_slices<KVM, ATT_THREADS>(a, kvh, nsplit, ring, 4 * (size_t)tileb, sp, sL);
}

// ---- float16 caches
// grid (nkv, nsplit), W warps (CH_WARPS; the clusters' form CL_WARPS where hs <= 128). A CTA takes one kv head's slice
// of positions for its KVM query heads; the slice is cut into chunks of 16 positions dealt to the warps in turn (warp
// w: chunks w, w + W, ...). Each warp copies
// its chunks' keys and values into its own ring in shared memory (asynchronous 16-byte copies, the first ones issued
// before the dependency wait: the cache rows before this token's are not the previous kernel's output) and keeps its
// own online softmax (a running max and sum a head) and output over them, with no barrier shared with other warps:
//   scores S (16 positions x 8 heads) = K . q^T,   output O^T (dims x heads) += V^T . P^T
// on the tensor cores (mma m16n8k16, float32 accumulation), q and the probabilities each split into two float16
// halves (hi + lo: their products with a float16 key or value are exact in the accumulation, so the sum keeps them to
// about 2^-22 of themselves). The score fragment's columns (heads 2 t4, 2 t4 + 1) are the output fragment's columns,
// so a thread rescales its own output with its own running maxima. The warps' parts are merged at the slice's end.
// CL (the forward driver's calls): a thread-block cluster of cs CTAs a kv head takes all of its positions, the
// chunks dealt to the cluster's cs x W warps in turn (grid (cs, nkv), cluster (cs, 1, 1)); each CTA merges its
// warps, and the CTAs' parts are combined through distributed shared memory, each CTA making 1/cs of the output (the
// cluster's CTAs run together, so they can wait for one another; no partials leave the SMs).
constexpr int CH_WARPS = 8, CH_THREADS = 32 * CH_WARPS, CHUNK = 16;
constexpr int CL_WARPS = 16;  // the clusters' warps a CTA (hs <= 128)
constexpr int HP = 8;    // heads padded to the products' n = 8
constexpr int PST = 24;  // halves a head's row of a warp's probabilities (conflict-free fragment reads)

constexpr int CS_MAX = 16;  // the largest cluster (a non-portable size)

template <int KVM, bool FUSE, int MBM, bool CL, int W>
__global__ void __launch_bounds__(32 * W, 1) attention_chunk_kernel(const AttArgs a0, const Fuse f0, const int ring) {
  extern __shared__ __align__(16) uint8_t att_smem[];
  const AttArgs a = sequence_of(a0, blockIdx.z);
  const Fuse f = sequence_of(f0, a0, blockIdx.z);
  constexpr int DL = MBM / 2;                          // a lane's values of a head: d = lane + 32 i (hs <= 32 DL)
  const int hs = a.hs, nmb = hs / 16;
  const int rowb = hs * 2 + 16;                        // a padded row of a chunk, bytes (conflict-free ldmatrix)
  const int chunkb = 2 * CHUNK * rowb;                 // a chunk's keys, then its values
  const int qst = hs + 8;                              // halves a row of q's halves (conflict-free fragment reads)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;              // an mma fragment's row group and column pair
  const int j0 = 2 * t4, j1 = 2 * t4 + 1;              // this thread's two head columns
  uint8_t* myring = att_smem + (size_t)warp * ring * chunkb;
  __half* sqh = reinterpret_cast<__half*>(att_smem + (size_t)W * ring * chunkb);  // [HP][qst] high halves
  __half* sql = sqh + HP * qst;                                                          // and low halves
  __half* sph = sql + HP * qst + warp * 2 * HP * PST;  // this warp's probabilities [HP][PST]: high, then low halves
  __half* spl = sph + HP * PST;
  uint16_t* sx = reinterpret_cast<uint16_t*>(sql + HP * qst + W * 2 * HP * PST);  // [2][hs] new key, value
  float* sml = reinterpret_cast<float*>(sx + 2 * hs);  // [W][KVM][2] the warps' maxima and sums
  float* sw = sml + W * KVM * 2;                // [KVM][nsplit] the combine's weights
  // CL: [ncta][per + 2 KVM] the cluster's parts of the (head, dimension) pairs this CTA makes (outputs, then maxima
  // and sums), stored by the other CTAs
  float* rcv = sw;
  __shared__ float sL[KVM];
  // CL: this CTA has started (other CTAs store into its shared memory only once every CTA of the cluster has)
  if constexpr (CL) asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  pdl_launch_dependents();  // the next kernel waits for this one's completion; its CTAs may take the SMs this one leaves
  // the position: written by the host before the step's first kernel, so readable before the dependency wait
  const int pos = position(a);
  const int count = pos + 1;
  const int kvh = CL ? blockIdx.y : blockIdx.x, split = CL ? 0 : blockIdx.y;
  const int rank = CL ? blockIdx.x : 0;  // the CTA's rank in its cluster
  const int ncta = CL ? a.cs : 1;  // the cluster's CTAs
  const int nsplit = CL ? 1 : a.pos_dev ? (count + a.split_len - 1) / a.split_len : a.nsplit;
  if (split >= nsplit) return;
  const int p0 = CL ? 0 : split * a.split_len, p1 = CL ? count : min(count, p0 + a.split_len);
  const int TW = ncta * W;  // the warps the chunks are dealt to
  const int gw = rank * W + warp;       // this warp's turn
  const int nchunk = (p1 - p0 + CHUNK - 1) / CHUNK;
  const int mine = gw < nchunk ? (nchunk - 1 - gw) / TW + 1 : 0;  // chunks of this warp
  const int kvdim = a.nkv * hs, hbase = kvh * KVM, pieces = hs / 8;       // 16-byte pieces a row
  const uint8_t* kbase = reinterpret_cast<const uint8_t*>(a.kc) + (long long)kvh * hs * 2;
  const uint8_t* vbase = reinterpret_cast<const uint8_t*>(a.vc) + (long long)kvh * hs * 2;
  // this warp's i-th chunk into its ring slot i % ring; value rows past the chunk's length zeroed (a probability of
  // 0 must meet a 0; key rows past it only make scores that are replaced by -inf)
  auto load_chunk = [&](int i) {
    uint8_t* sK = myring + (size_t)(i % ring) * chunkb;
    uint8_t* sV = sK + CHUNK * rowb;
    const int t0 = p0 + CHUNK * (gw + TW * i);
    const int len = min(CHUNK, p1 - t0);
    for (int e = lane; e < CHUNK * pieces; e += 32) {
      const int t = e / pieces, c = e % pieces;
      if (t < len) {
        const long long off = (long long)(t0 + t) * kvdim * 2 + c * 16;
        cp_async16(sK + t * rowb + c * 16, kbase + off);
        cp_async16(sV + t * rowb + c * 16, vbase + off);
      } else {
        *reinterpret_cast<int4*>(sV + t * rowb + c * 16) = make_int4(0, 0, 0, 0);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  const bool holds_pos = FUSE && (CL ? (pos / CHUNK) % TW / W == rank : p1 == count);
  // CL: the warps of the q / k / v prologue issue their chunks' copies after it, the others at once (a CTA's copies
  // take microseconds to issue, the memory being busy with them: the prologue need not wait behind them)
  const bool late = CL && warp < KVM + (holds_pos ? 2 : 0);
  if (!late)
    for (int i = 0; i < ring && i < mine; i++) load_chunk(i);
  for (int e = tid; e < (HP - KVM) * qst; e += (32 * W)) {  // the padded heads' q: zero
    sqh[KVM * qst + e] = __float2half_rn(0.0f);
    sql[KVM * qst + e] = __float2half_rn(0.0f);
  }
  // the head norms' weights and the RoPE tables' row of pos (not the previous kernel's output): read before the wait
  const int turned = f.rot > 0 && f.rot < hs ? f.rot : hs;
  float wq[DL], wk[DL], cs[DL], sn[DL];
  if (FUSE) {
    const float* crow = f.cos_t + (long long)pos * (hs / 2);
    const float* srow = f.sin_t + (long long)pos * (hs / 2);
#pragma unroll
    for (int i = 0; i < DL; i++) {
      const int d = lane + 32 * i;
      wq[i] = d < hs && f.qn ? f.qn[d] : 1.0f;
      wk[i] = d < hs && f.kn ? f.kn[d] : 1.0f;
      cs[i] = d < turned ? crow[d >> 1] : 1.0f;
      sn[i] = d < turned ? srow[d >> 1] : 0.0f;
    }
  }
  pdl_wait();
  // the query heads a warp each; where this slice holds the position, its key and value too (FUSE: the heads' RMSNorm
  // over the lanes' strided sums, then RoPE on lane pairs)
  for (int j = warp; j < KVM + (holds_pos ? 2 : 0); j += W) {
    const float* src = j < KVM ? a.q + (long long)(hbase + j) * hs : (j == KVM ? f.k : f.v) + (long long)kvh * hs;
    float x[DL];
#pragma unroll
    for (int i = 0; i < DL; i++) {
      const int d = lane + 32 * i;
      x[i] = d < hs ? src[d] : 0.0f;
    }
    if (FUSE && j <= KVM) {
      if (j < KVM ? f.qn : f.kn) {
        float s = 0.0f;
#pragma unroll
        for (int i = 0; i < DL; i++) s = fmaf(x[i], x[i], s);
        s = warp_sum(s);
        const float r = 1.0f / sqrtf(s / (float)hs + f.eps);
#pragma unroll
        for (int i = 0; i < DL; i++) x[i] = (j < KVM ? wq[i] : wk[i]) * (r * x[i]);
      }
#pragma unroll
      for (int i = 0; i < DL; i++) {
        const float o = __shfl_xor_sync(0xffffffffu, x[i], 1);  // the pair's other value
        const int d = lane + 32 * i;
        if (d < turned) x[i] = (d & 1) ? o * sn[i] + x[i] * cs[i] : x[i] * cs[i] - o * sn[i];
      }
    }
    if (j < KVM) {  // q as two float16 halves
#pragma unroll
      for (int i = 0; i < DL; i++) {
        const int d = lane + 32 * i;
        if (d >= hs) continue;
        __half hi, lo;
        split_half(x[i], hi, lo);
        sqh[j * qst + d] = hi;
        sql[j * qst + d] = lo;
      }
    } else {  // this position's key (j == KVM) or value into the cache, and into the chunk that holds it
      uint16_t* cache = reinterpret_cast<uint16_t*>(const_cast<void*>(j == KVM ? a.kc : a.vc)) +
                        (long long)pos * kvdim + (long long)kvh * hs;
      int local = 0;
#pragma unroll
      for (int i = 0; i < DL; i++) {
        const int d = lane + 32 * i;
        if (d >= hs) continue;
        const uint16_t b = float_to_half_bits(x[i], &local);
        cache[d] = b;
        sx[(j - KVM) * hs + d] = b;
      }
      if (local && f.bad) atomicAdd(f.bad, local);
    }
  }
  if (late)
    for (int i = 0; i < ring && i < mine; i++) load_chunk(i);
  __syncthreads();
  float M0 = -INFINITY, M1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;  // heads j0, j1: running max and (lane-partial) sum
  float oc[MBM][4];
#pragma unroll
  for (int mb = 0; mb < MBM; mb++)
#pragma unroll
    for (int c = 0; c < 4; c++) oc[mb][c] = 0.0f;
  const float isq = 1.0f / sqrtf((float)hs);
  for (int i = 0; i < mine; i++) {
    // this chunk's copies are done when at most the next chunk's group is still in flight
    if (ring > 1 && i + 1 < mine) asm volatile("cp.async.wait_group 1;" ::: "memory");
    else cp_async_wait_all();
    __syncwarp();
    uint8_t* sK = myring + (size_t)(i % ring) * chunkb;
    uint8_t* sV = sK + CHUNK * rowb;
    const int t0 = p0 + CHUNK * (gw + TW * i);
    const int len = min(CHUNK, p1 - t0);
    if (holds_pos && pos >= t0 && pos < t0 + len) {  // this position's row: the fresh key and value
      for (int e = lane; e < 2 * hs; e += 32)
        reinterpret_cast<uint16_t*>((e < hs ? sK : sV) + (size_t)(pos - t0) * rowb)[e % hs] = sx[e];
      __syncwarp();
    }
    // scores, the high and low halves' products in two accumulators
    float ch[4] = {0.0f, 0.0f, 0.0f, 0.0f}, cl[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const uint8_t* arow = sK + ((lane & 7) + ((lane >> 3) & 1) * 8) * rowb + (lane >> 4) * 16;
#pragma unroll
    for (int kk = 0; kk < MBM; kk++) {
      if (kk >= nmb) break;
      uint32_t af[4];
      ldsm_x4(af, arow + kk * 32);
      const int qo = g * qst + 16 * kk + 2 * t4;
      mma16816(ch, af, lds32(sqh + qo), lds32(sqh + qo + 8));
      mma16816(cl, af, lds32(sql + qo), lds32(sql + qo + 8));
    }
    float sc[4];
#pragma unroll
    for (int r = 0; r < 4; r++) {  // rows g, g, g + 8, g + 8; columns j0, j1, j0, j1
      float v = (ch[r] + cl[r]) * isq;
      if (a.cap > 0.0f) v = a.cap * tanhf(v / a.cap);
      sc[r] = g + (r >> 1) * 8 < len ? v : -INFINITY;
    }
    // the chunk's maxima over its 16 positions (the lanes of a column pair differ in g)
    float m0 = fmaxf(sc[0], sc[2]), m1 = fmaxf(sc[1], sc[3]);
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, o));
      m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, o));
    }
    const float n0 = fmaxf(M0, m0), n1 = fmaxf(M1, m1);
    const float b0 = n0 == -INFINITY ? 0.0f : n0, b1 = n1 == -INFINITY ? 0.0f : n1;
    const float r0 = expf(M0 - b0), r1 = expf(M1 - b1);  // 0 at the first chunk (exp(-inf))
    M0 = n0;
    M1 = n1;
    const float q0 = expf(sc[0] - b0), q1 = expf(sc[1] - b1), q2 = expf(sc[2] - b0), q3 = expf(sc[3] - b1);
    l0 = fmaf(l0, r0, q0 + q2);
    l1 = fmaf(l1, r1, q1 + q3);
    __half hi, lo;  // P as [head][position] halves, read back as the weighted values' B fragments
    split_half(q0, hi, lo);
    sph[j0 * PST + g] = hi;
    spl[j0 * PST + g] = lo;
    split_half(q1, hi, lo);
    sph[j1 * PST + g] = hi;
    spl[j1 * PST + g] = lo;
    split_half(q2, hi, lo);
    sph[j0 * PST + g + 8] = hi;
    spl[j0 * PST + g + 8] = lo;
    split_half(q3, hi, lo);
    sph[j1 * PST + g + 8] = hi;
    spl[j1 * PST + g + 8] = lo;
    __syncwarp();
    const uint32_t ph0 = lds32(sph + g * PST + 2 * t4), ph1 = lds32(sph + g * PST + 2 * t4 + 8);
    const uint32_t pl0 = lds32(spl + g * PST + 2 * t4), pl1 = lds32(spl + g * PST + 2 * t4 + 8);
    // the weighted values, 16 dimensions an m-block
    const uint8_t* vrow = sV + ((lane & 7) + ((lane >> 4) & 1) * 8) * rowb + ((lane >> 3) & 1) * 16;
#pragma unroll
    for (int mb = 0; mb < MBM; mb++) {
      if (mb >= nmb) break;
      oc[mb][0] *= r0;
      oc[mb][1] *= r1;
      oc[mb][2] *= r0;
      oc[mb][3] *= r1;
      uint32_t af[4];
      ldsm_x4_trans(af, vrow + mb * 32);
      mma16816(oc[mb], af, ph0, ph1);
      mma16816(oc[mb], af, pl0, pl1);
    }
    __syncwarp();  // the chunk's slot and the probabilities are read: both may be rewritten
    if (i + ring < mine) load_chunk(i + ring);
  }
  // this warp's part: the sums over its row groups; output, maxima and sums to shared memory (its ring is free)
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, o);
    l1 += __shfl_xor_sync(0xffffffffu, l1, o);
  }
  float* so = reinterpret_cast<float*>(myring);  // [KVM][hs + 4]
#pragma unroll
  for (int mb = 0; mb < MBM; mb++) {
    if (mb >= nmb) break;
    const int d = 16 * mb + g;
    if (j0 < KVM) {
      so[j0 * (hs + 4) + d] = oc[mb][0];
      so[j0 * (hs + 4) + d + 8] = oc[mb][2];
    }
    if (j1 < KVM) {
      so[j1 * (hs + 4) + d] = oc[mb][1];
      so[j1 * (hs + 4) + d + 8] = oc[mb][3];
    }
  }
  if (g == 0) {
    if (j0 < KVM) {
      sml[(warp * KVM + j0) * 2] = M0;
      sml[(warp * KVM + j0) * 2 + 1] = l0;
    }
    if (j1 < KVM) {
      sml[(warp * KVM + j1) * 2] = M1;
      sml[(warp * KVM + j1) * 2 + 1] = l1;
    }
  }
  __syncthreads();
  // the warps' parts merged, a thread a (head, dimension) pair: the slice's output (one slice: the head's output);
  // CL: the CTA's part of pair e stored into the receive buffer of the CTA that makes e (slot: this CTA's rank), the
  // part's maxima and sums into every CTA's
  namespace cg = cooperative_groups;
  const int per = CL ? (KVM * hs + ncta - 1) / ncta : 1, RS = per + 2 * KVM;  // CL: the pairs a CTA makes; a slot
  // each head's largest warp maximum, then each (warp, head)'s weight, once (a head's pairs share them)
  __shared__ float s_mx[KVM], s_wt[W * KVM];
  if (tid < KVM) {
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < W; w++) mx = fmaxf(mx, sml[(w * KVM + tid) * 2]);
    s_mx[tid] = mx;
  }
  __syncthreads();
  if (tid < W * KVM) {
    const int w = tid / KVM, j = tid % KVM;
    const float base = s_mx[j] == -INFINITY ? 0.0f : s_mx[j];
    s_wt[tid] = expf(sml[(w * KVM + j) * 2] - base);  // 0 for a warp without chunks
  }
  __syncthreads();
  if constexpr (CL) asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every CTA has started
  for (int e = tid; e < KVM * hs; e += (32 * W)) {
    const int j = e / hs, d = e % hs, h = hbase + j;
    const float mx = s_mx[j];
    float o = 0.0f, l = 0.0f;
#pragma unroll
    for (int w = 0; w < W; w++) {
      const float wt = s_wt[w * KVM + j];
      o = fmaf(reinterpret_cast<const float*>(att_smem + (size_t)w * ring * chunkb)[j * (hs + 4) + d], wt, o);
      l = fmaf(sml[(w * KVM + j) * 2 + 1], wt, l);
    }
    if (CL) {
      cg::cluster_group cluster = cg::this_cluster();
      const int c = e / per;
      cluster.map_shared_rank(rcv, c)[rank * RS + e - c * per] = o;
      if (d == 0)
        for (int c2 = 0; c2 < ncta; c2++) {
          float* dst = cluster.map_shared_rank(rcv, c2) + rank * RS + per;
          dst[j] = mx;
          dst[KVM + j] = l;
        }
      continue;
    }
    if (h < a.h0 || h >= a.h1) continue;
    if (nsplit == 1) {
      a.out[(long long)h * hs + d] = o / l;
    } else {
      float* part = a.part + ((long long)h * a.nsplit + split) * (hs + 4);
      part[d] = o;
      if (d == 0) {
        part[hs] = mx;
        part[hs + 1] = l;
      }
    }
  }
  if constexpr (CL) {  // the cluster's parts combined: this CTA makes pairs [rank per, (rank + 1) per), each CTA's part
    // in its receive buffer (no CTA reads another's shared memory after the barrier, so none waits to leave)
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();  // every part stored (release / acquire)
    // each head's largest CTA maximum, then each (CTA, head)'s weight, once
    __shared__ float c_mx[KVM], c_wt[CS_MAX * KVM];
    if (tid < KVM) {
      float mx = -INFINITY;
      for (int c = 0; c < ncta; c++) mx = fmaxf(mx, rcv[c * RS + per + tid]);
      c_mx[tid] = mx;
    }
    __syncthreads();
    if (tid < ncta * KVM) {
      const int c = tid / KVM, j = tid % KVM;
      const float base = c_mx[j] == -INFINITY ? 0.0f : c_mx[j];
      c_wt[tid] = expf(rcv[c * RS + per + j] - base);  // 0 for a CTA without chunks
    }
    __syncthreads();
    const int e = rank * per + tid;
    if (tid < per && e < KVM * hs) {
      const int j = e / hs, d = e % hs;
      float os = 0.0f, ls = 0.0f;
#pragma unroll
      for (int c = 0; c < CS_MAX; c++) {
        if (c >= ncta) break;
        const float* src = rcv + c * RS;
        const float wt = c_wt[c * KVM + j];
        os = fmaf(src[tid], wt, os);
        ls = fmaf(src[per + KVM + j], wt, ls);
      }
      a.out[(long long)(hbase + j) * hs + d] = os / ls;
    }
    return;
  }
  if (nsplit == 1 || !a.counters) return;
  combine_slices<KVM, (32 * W)>(a, kvh, nsplit, att_smem, (size_t)W * ring * chunkb, sw, sL);
}

// a block a head: the slices' partials combined
__global__ void attention_combine_kernel(const AttArgs a0) {
  const AttArgs a = sequence_of(a0, blockIdx.z);
  pdl_wait();
  const int pos = position(a);
  const int count = pos + 1;
  const int nsplit = a.pos_dev ? (count + a.split_len - 1) / a.split_len : a.nsplit;
  const int h = a.h0 + blockIdx.x;
  if (nsplit == 1 || h >= a.h1) return;
  const int hs = a.hs;
  const float* part = a.part + (long long)h * a.nsplit * (hs + 4);
  float M = -INFINITY;
  for (int s = 0; s < nsplit; s++) M = fmaxf(M, part[s * (hs + 4) + hs]);
  float L = 0.0f;
  for (int s = 0; s < nsplit; s++) L += part[s * (hs + 4) + hs + 1] * expf(part[s * (hs + 4) + hs] - M);
  const float inv = 1.0f / L;
  for (int d = threadIdx.x; d < hs; d += blockDim.x) {
    float o = 0.0f;
    for (int s = 0; s < nsplit; s++) o += part[s * (hs + 4) + d] * expf(part[s * (hs + 4) + hs] - M);
    a.out[(long long)h * hs + d] = o * inv;
  }
}

cudaLaunchConfig_t launch_config(dim3 grid, int threads, size_t smem, bool pdl, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = pllm_stream();
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cfg;
}

template <typename K, typename... Args>
cudaError_t launch_with(K kernel, const cudaLaunchConfig_t& cfg, Args... args) {
  if (cfg.dynamicSmemBytes > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cfg.dynamicSmemBytes);
    if (e != cudaSuccess) return e;
  }
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <int KVM>
cudaError_t launch_f32(const AttArgs& a, const Fuse* f, const cudaLaunchConfig_t& cfg) {
  if (f) return launch_with(attention_f32_kernel<KVM, true>, cfg, a, *f);
  return launch_with(attention_f32_kernel<KVM, false>, cfg, a, Fuse{});
}

template <int KVM>
cudaError_t launch_chunks(const AttArgs& a, const Fuse* f, const cudaLaunchConfig_t& cfg, int ring) {
  const Fuse none = {};
  if (a.hs <= 128) {
    if (f) return launch_with(attention_chunk_kernel<KVM, true, 8, false, CH_WARPS>, cfg, a, *f, ring);
    return launch_with(attention_chunk_kernel<KVM, false, 8, false, CH_WARPS>, cfg, a, none, ring);
  }
  if (f) return launch_with(attention_chunk_kernel<KVM, true, 16, false, CH_WARPS>, cfg, a, *f, ring);
  return launch_with(attention_chunk_kernel<KVM, false, 16, false, CH_WARPS>, cfg, a, none, ring);
}

// One cluster size's launch (grid (cs, nkv), cluster (cs, 1, 1)), or (fits non-null) the number of such clusters
// the device can hold at once.
template <int KVM, bool FUSE, int MBM, int W>
cudaError_t launch_cluster_cs(AttArgs a, const Fuse& f, const cudaLaunchConfig_t& base, int ring, int cs, int* fits) {
  auto k = attention_chunk_kernel<KVM, FUSE, MBM, true, W>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)base.dynamicSmemBytes);
  if (e == cudaSuccess && cs > 8) e = cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = base;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1] = base.numAttrs ? base.attrs[0] : attr[0];  // the dependent-launch attribute, where asked for
  cfg.gridDim = dim3((unsigned)cs, a.nkv, a.batch > 1 ? a.batch : 1);
  cfg.attrs = attr;
  cfg.numAttrs = 1 + (base.numAttrs ? 1 : 0);
  if (fits) {
    cfg.numAttrs = 1;
    return cudaOccupancyMaxActiveClusters(fits, k, &cfg);
  }
  a.cs = cs;
  return cudaLaunchKernelEx(&cfg, k, a, f, ring);
}

// The cluster size for a configuration: the largest of 16 (a non-portable size) down to 8 CTAs of which the device
// holds all nkv clusters at once (the most warps to deal the chunks to, with no cluster waiting for another's SMs:
// on the B200s measured 10, where 16 and 12 held only 7 clusters), else 8 where it holds one, else 0 (the slices'
// kernel). Found once a configuration (kernel, shared memory, nkv) and device, before its first launch.
template <int KVM, bool FUSE, int MBM, int W>
cudaError_t launch_cluster(const AttArgs& a, const Fuse& f, const cudaLaunchConfig_t& cfg, int ring, bool* launched) {
  struct Choice {
    int dev, nkv, hs;
    size_t smem;
    int cs;
  };
  static Choice cache[64];
  static int used = 0;
  std::lock_guard<std::mutex> hold(pllm_lookup_lock());
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  int cs = -1;
  for (int i = 0; i < used; i++)
    if (cache[i].dev == dev && cache[i].nkv == a.nkv && cache[i].hs == a.hs && cache[i].smem == cfg.dynamicSmemBytes)
      cs = cache[i].cs;
  if (cs < 0) {
    cs = 0;
    for (int c = CS_MAX; c >= 8 && !cs; c--) {
      int n = 0;
      if (launch_cluster_cs<KVM, FUSE, MBM, W>(a, f, cfg, ring, c, &n) != cudaSuccess) n = 0;
      if (n >= a.nkv || (c == 8 && n >= 1)) cs = c;
    }
    cudaGetLastError();  // a refused query leaves no error behind: the choice falls back
    if (used < 64) cache[used++] = Choice{dev, a.nkv, a.hs, cfg.dynamicSmemBytes, cs};
  }
  *launched = cs != 0;
  if (cs) return launch_cluster_cs<KVM, FUSE, MBM, W>(a, f, cfg, ring, cs, nullptr);
  return cudaSuccess;
}

template <int KVM>
cudaError_t launch_clusters(const AttArgs& a, const Fuse* f, const cudaLaunchConfig_t& cfg, int ring, bool* launched) {
  const Fuse none = {};
  if (a.hs <= 128) {  // CL_WARPS warps, a ring slot each
    if (f) return launch_cluster<KVM, true, 8, CL_WARPS>(a, *f, cfg, ring, launched);
    return launch_cluster<KVM, false, 8, CL_WARPS>(a, none, cfg, ring, launched);
  }
  if (f) return launch_cluster<KVM, true, 16, CH_WARPS>(a, *f, cfg, ring, launched);
  return launch_cluster<KVM, false, 16, CH_WARPS>(a, none, cfg, ring, launched);
}

// the forward driver's float16 attention by clusters (1) or by slices and a combine (0); pllm_set_attention_mode
int g_cluster_attention = 1;

void run_attention(const char* name, AttArgs a, bool half, bool pdl, const Fuse* f = nullptr) {
  const int kvm = a.nh / a.nkv;
  const dim3 grid(a.nkv, a.nsplit, a.batch > 1 ? a.batch : 1);
  const size_t comb = a.counters ? (size_t)a.nsplit : 0;  // the combine's weights: kvm x nsplit floats
  cudaLaunchAttribute attr[1];
  cudaError_t e;
  if (half) {
    const size_t rowb = (size_t)a.hs * 2 + 16;
    auto smem_of = [&](int ring, size_t comb_floats, int warps = CH_WARPS) {
      return (size_t)warps * ring * 2 * CHUNK * rowb + 2 * (size_t)HP * (a.hs + 8) * 2 +
             (size_t)warps * 2 * HP * PST * 2 + 2 * (size_t)a.hs * 2 + (size_t)warps * kvm * 2 * 4 +
             (size_t)kvm * comb_floats * 4;
    };
    if (a.pos_dev && a.h0 == 0 && a.h1 == a.nh && g_cluster_attention) {
      // the whole cache a cluster: one ring slot a warp (hs <= 128: CL_WARPS warps, so that a cluster of 10 holds a
      // chunk a warp up to 2,560 positions), no partials
      const int ring = 1, warps = a.hs <= 128 ? CL_WARPS : CH_WARPS;
      // the receive buffer: at most kvm hs outputs + CS_MAX x (1 + 2 kvm) floats over the cluster's slots
      const size_t rcv = ((size_t)kvm * a.hs + (size_t)CS_MAX * (1 + 2 * kvm)) * 4;
      const cudaLaunchConfig_t cfg = launch_config(grid, 32 * warps, smem_of(ring, 0, warps) + rcv, pdl, attr);
      bool launched = false;
      switch (kvm) {
        case 1: e = launch_clusters<1>(a, f, cfg, ring, &launched); break;
        case 2: e = launch_clusters<2>(a, f, cfg, ring, &launched); break;
        case 4: e = launch_clusters<4>(a, f, cfg, ring, &launched); break;
        case 8: e = launch_clusters<8>(a, f, cfg, ring, &launched); break;
        default: e = cudaErrorInvalidValue;
      }
      if (e != cudaSuccess) {
        pllm_fail(PLLM_ECUDA, "%s: cluster launch failed: %s", name, cudaGetErrorString(e));
        return;
      }
      if (launched) return;
    }
    // two ring slots a warp where a warp has two chunks or more (hs <= 128: the slots fit beside each other)
    const int per_warp = ((a.split_len + CHUNK - 1) / CHUNK + CH_WARPS - 1) / CH_WARPS;
    const int ring = per_warp >= 2 && a.hs <= 128 ? 2 : 1;
    const cudaLaunchConfig_t cfg = launch_config(grid, CH_THREADS, smem_of(ring, comb), pdl, attr);
    switch (kvm) {
      case 1: e = launch_chunks<1>(a, f, cfg, ring); break;
      case 2: e = launch_chunks<2>(a, f, cfg, ring); break;
      case 4: e = launch_chunks<4>(a, f, cfg, ring); break;
      case 8: e = launch_chunks<8>(a, f, cfg, ring); break;
      default: e = cudaErrorInvalidValue;
    }
  } else {
    const size_t rowb = (size_t)a.hs * 4 + 16;
    const size_t scores = (size_t)kvm * ((size_t)TILE > comb ? (size_t)TILE : comb) * 4;
    const size_t smem = 4 * TILE * rowb + (size_t)kvm * a.hs * 4 + 2 * (size_t)a.hs * 4 + scores;
    const cudaLaunchConfig_t cfg = launch_config(grid, ATT_THREADS, smem, pdl, attr);
    switch (kvm) {
      case 1: e = launch_f32<1>(a, f, cfg); break;
      case 2: e = launch_f32<2>(a, f, cfg); break;
      case 4: e = launch_f32<4>(a, f, cfg); break;
      case 8: e = launch_f32<8>(a, f, cfg); break;
      default: e = cudaErrorInvalidValue;
    }
  }
  if (e != cudaSuccess) {
    pllm_fail(PLLM_ECUDA, "%s: launch failed: %s", name, cudaGetErrorString(e));
    return;
  }
  if ((a.nsplit > 1 || a.pos_dev) && !a.counters) {
    const cudaLaunchConfig_t cfg =
        launch_config(dim3(a.h1 - a.h0, 1, a.batch > 1 ? a.batch : 1), a.hs >= 128 ? 128 : 64, 0, pdl, attr);
    e = cudaLaunchKernelEx(&cfg, attention_combine_kernel, a);
    if (e != cudaSuccess) pllm_fail(PLLM_ECUDA, "%s: combine launch failed: %s", name, cudaGetErrorString(e));
  }
}

bool check_heads(const char* name, int nh, int nkv, int hs, int h0, int h1) {
  if (nh <= 0 || nkv <= 0 || nh % nkv || hs <= 0 || hs > 256 || hs % 16 || h0 < 0 || h1 < h0 || h1 > nh) {
    pllm_fail(PLLM_EINVAL, "%s: nh %d nkv %d hs %d heads %d..%d", name, nh, nkv, hs, h0, h1);
    return false;
  }
  const int kvm = nh / nkv;
  if (kvm != 1 && kvm != 2 && kvm != 4 && kvm != 8) {
    pllm_fail(PLLM_EINVAL, "%s: %d query heads a kv head (1, 2, 4 or 8 are built)", name, kvm);
    return false;
  }
  return true;
}

// the registry's call: the slices' partials go to the reference's scratch att (nh (pos + 1) floats), so a slice
// count is chosen whose partials fit in it (and att must be 16-byte aligned)
void registry_attention(const char* name, uint64_t out, uint64_t q, uint64_t kc, uint64_t vc, uint64_t att, int pos,
                        int nh, int nkv, int hs, int h0, int h1, float cap, bool half) {
  if (!check_heads(name, nh, nkv, hs, h0, h1)) return;
  PLLM_REQUIRE(pos >= 0, "%s: pos %d", name, pos);
  PLLM_REQUIRE(!(kc & 15) && !(vc & 15) && !(att & 15), "%s: the cache and att must be 16-byte aligned", name);
  if (h1 == h0) return;
  const int count = pos + 1;
  int nsplit = (count + 127) / 128;
  const int fit = count / (hs + 4);
  if (nsplit > fit) nsplit = fit;
  if (nsplit < 1) nsplit = 1;
  AttArgs a = {};
  a.out = dptr<float>(out);
  a.q = dptr<const float>(q);
  a.kc = dptr<const void>(kc);
  a.vc = dptr<const void>(vc);
  a.part = dptr<float>(att);
  a.pos = pos;
  a.nh = nh;
  a.nkv = nkv;
  a.hs = hs;
  a.h0 = h0;
  a.h1 = h1;
  a.nsplit = nsplit;
  a.split_len = (count + nsplit - 1) / nsplit;
  a.cap = cap;
  run_attention(name, a, half, false);
}

__global__ void rope_kernel(float* v, const float* fcr, const float* fci, int nh, int hs, int turned) {
  const int pairs = turned / 2;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < nh * pairs; e += gridDim.x * blockDim.x) {
    const int h = e / pairs, i = e % pairs;
    float* p = v + (long long)h * hs + 2 * i;
    const float c = fcr[i], s = fci[i];
    const float v0 = p[0], v1 = p[1];
    p[0] = v0 * c - v1 * s;
    p[1] = v0 * s + v1 * c;
  }
}

// ---- prefill: count tokens at positions p0.. attend causally over the float16 cache (attention.ts:87-211 for each
// token, all of a prompt at once). grid (nkv, tiles): a CTA takes PF_ROWS query rows = PF_ROWS / KVM tokens x the KVM
// query heads of kv head kvh (row r: token r / KVM, head r % KVM), a warp 16 rows; the keys of positions 0 .. the
// CTA's last token come in chunks of PF_KEYS by cp.async (double-buffered). On the tensor cores (mma m16n8k16, float32
// accumulation): S = Q K^T with q split into float16 hi + lo (exact products with the float16 keys), an online softmax
// a row (keys past the row's own position are -inf), O += P V with P split the same way. The f16 cache rows are the
// ones the decode step reads, so the prefill's numbers differ from token-by-token decoding only in summation order.
constexpr int PF_ROWS = 64, PF_KEYS = 64, PF_THREADS = 128;

template <int KVM>
__global__ void __launch_bounds__(PF_THREADS) attention_prefill_kernel(float* out, long long ostride, const float* qkv,
                                                                      long long qstride, const uint16_t* kc,
                                                                      const uint16_t* vc, int p0, int count, int nkv,
                                                                      int hs) {
  constexpr int QT = PF_ROWS / KVM;  // tokens a CTA
  extern __shared__ __align__(16) uint8_t pf_smem[];
  const int rowb = hs * 2 + 16;      // a padded float16 row (conflict-free ldmatrix)
  uint8_t* sQh = pf_smem;
  uint8_t* sQl = sQh + PF_ROWS * rowb;
  uint8_t* ring = sQl + PF_ROWS * rowb;  // [2 buffers][keys, values][PF_KEYS][rowb]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t4 = lane & 3;
  const int kvh = blockIdx.x, t0 = blockIdx.y * QT;
  const int ntok = min(QT, count - t0);
  const int kvdim = nkv * hs, nmb = hs / 16, ndb = hs / 8;
  const int nkeys = p0 + t0 + ntok;  // positions 0 .. the CTA's last token
  const int nchunk = (nkeys + PF_KEYS - 1) / PF_KEYS;
  const int pieces = hs / 8;         // 16-byte pieces a row
  const float isq = 1.0f / sqrtf((float)hs);
  auto load_chunk = [&](int c, int buf) {
    uint8_t* sK = ring + (size_t)(2 * buf) * PF_KEYS * rowb;
    uint8_t* sV = sK + PF_KEYS * rowb;
    const int k0 = c * PF_KEYS;
    for (int e = tid; e < PF_KEYS * pieces; e += PF_THREADS) {
      const int t = e / pieces, pc = e % pieces;
      if (k0 + t < nkeys) {
        const long long off = ((long long)(k0 + t) * kvdim + (long long)kvh * hs) * 2 + pc * 16;
        cp_async16(sK + t * rowb + pc * 16, reinterpret_cast<const uint8_t*>(kc) + off);
        cp_async16(sV + t * rowb + pc * 16, reinterpret_cast<const uint8_t*>(vc) + off);
      } else {  // a probability of 0 must meet a 0 (and no key past the cache is read)
        *reinterpret_cast<int4*>(sK + t * rowb + pc * 16) = make_int4(0, 0, 0, 0);
        *reinterpret_cast<int4*>(sV + t * rowb + pc * 16) = make_int4(0, 0, 0, 0);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  load_chunk(0, 0);
  for (int e = tid; e < PF_ROWS * hs; e += PF_THREADS) {  // the query rows as float16 hi + lo (rows past ntok: 0)
    const int r = e / hs, d = e % hs, t = r / KVM, j = r % KVM;
    const float x = t < ntok ? qkv[(long long)(t0 + t) * qstride + (long long)(kvh * KVM + j) * hs + d] : 0.0f;
    __half hi, lo;
    split_half(x, hi, lo);
    reinterpret_cast<__half*>(sQh + r * rowb)[d] = hi;
    reinterpret_cast<__half*>(sQl + r * rowb)[d] = lo;
  }
  // this thread's rows (g and g + 8 of the warp's 16) and their positions
  const int rA = 16 * warp + g, rB = rA + 8;
  const int qpA = p0 + t0 + rA / KVM, qpB = p0 + t0 + rB / KVM;
  float o[16][4];  // O rows g, g + 8 x dims (8 nd + 2 t4, +1), hs <= 128
#pragma unroll
  for (int nd = 0; nd < 16; nd++) o[nd][0] = o[nd][1] = o[nd][2] = o[nd][3] = 0.0f;
  float mA = -INFINITY, mB = -INFINITY, lA = 0.0f, lB = 0.0f;
  const uint8_t* qa_h = sQh + (16 * warp + (lane & 7) + ((lane >> 3) & 1) * 8) * rowb + (lane >> 4) * 16;
  const uint8_t* qa_l = qa_h - sQh + sQl;
  for (int c = 0; c < nchunk; c++) {
    const int buf = c & 1;
    if (c + 1 < nchunk) {
      load_chunk(c + 1, buf ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      cp_async_wait_all();
    }
    __syncthreads();
    const uint8_t* sK = ring + (size_t)(2 * buf) * PF_KEYS * rowb;
    const uint8_t* sV = sK + PF_KEYS * rowb;
    const int k0 = c * PF_KEYS;
    // S (16 rows x 64 keys): 8 key blocks of 8; keys as B (col-major k = dims x n = keys: the key rows as stored)
    float sc[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; nb++) sc[nb][0] = sc[nb][1] = sc[nb][2] = sc[nb][3] = 0.0f;
    for (int kk = 0; kk < nmb; kk++) {
      uint32_t ah[4], al[4];
      ldsm_x4(ah, qa_h + kk * 32);
      ldsm_x4(al, qa_l + kk * 32);
#pragma unroll
      for (int nb = 0; nb < 8; nb += 2) {  // two key blocks a load: matrices (keys 8 nb.., dims +0 / +8), (8 nb + 8..)
        uint32_t b[4];
        ldsm_x4(b, sK + (8 * nb + (lane & 7) + ((lane >> 4) & 1) * 8) * rowb + kk * 32 + ((lane >> 3) & 1) * 16);
        mma16816(sc[nb], ah, b[0], b[1]);
        mma16816(sc[nb], al, b[0], b[1]);
        mma16816(sc[nb + 1], ah, b[2], b[3]);
        mma16816(sc[nb + 1], al, b[2], b[3]);
      }
    }
    // scale, causal mask, the chunk's row maxima (a row's 64 keys are over the 4 threads of its quad)
    float xA = -INFINITY, xB = -INFINITY;
#pragma unroll
    for (int nb = 0; nb < 8; nb++)
#pragma unroll
      for (int u = 0; u < 2; u++) {
        const int kp = k0 + 8 * nb + 2 * t4 + u;
        sc[nb][u] = kp <= qpA ? sc[nb][u] * isq : -INFINITY;
        sc[nb][2 + u] = kp <= qpB ? sc[nb][2 + u] * isq : -INFINITY;
        xA = fmaxf(xA, sc[nb][u]);
        xB = fmaxf(xB, sc[nb][2 + u]);
      }
    xA = fmaxf(xA, __shfl_xor_sync(0xffffffffu, xA, 1));
    xA = fmaxf(xA, __shfl_xor_sync(0xffffffffu, xA, 2));
    xB = fmaxf(xB, __shfl_xor_sync(0xffffffffu, xB, 1));
    xB = fmaxf(xB, __shfl_xor_sync(0xffffffffu, xB, 2));
    const float nA = fmaxf(mA, xA), nB = fmaxf(mB, xB);
    const float bA = nA == -INFINITY ? 0.0f : nA, bB = nB == -INFINITY ? 0.0f : nB;
    const float aA = expf(mA - bA), aB = expf(mB - bB);  // 0 at the first chunk
    mA = nA;
    mB = nB;
    lA *= aA;
    lB *= aB;
#pragma unroll
    for (int nd = 0; nd < 16; nd++) {
      o[nd][0] *= aA;
      o[nd][1] *= aA;
      o[nd][2] *= aB;
      o[nd][3] *= aB;
    }
    // P = exp(S - m) as float16 hi + lo A fragments, O += P V (V as B: ldmatrix.trans of the value rows)
#pragma unroll
    for (int k2 = 0; k2 < 4; k2++) {
      float p[8];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        p[u] = expf(sc[2 * k2][u] - (u < 2 ? bA : bB));
        p[4 + u] = expf(sc[2 * k2 + 1][u] - (u < 2 ? bA : bB));
      }
      lA += p[0] + p[1] + p[4] + p[5];
      lB += p[2] + p[3] + p[6] + p[7];
      __half h[8], l[8];
#pragma unroll
      for (int u = 0; u < 8; u++) split_half(p[u], h[u], l[u]);
      uint32_t ph[4], pl[4];
      // a0: row g keys 2 t4.. (block 2 k2: p0 p1), a1: row g + 8 (p2 p3), a2: row g keys +8 (block 2 k2 + 1: p4 p5),
      // a3: row g + 8 keys +8 (p6 p7)
      ph[0] = pack_halves(h[0], h[1]);
      ph[1] = pack_halves(h[2], h[3]);
      ph[2] = pack_halves(h[4], h[5]);
      ph[3] = pack_halves(h[6], h[7]);
      pl[0] = pack_halves(l[0], l[1]);
      pl[1] = pack_halves(l[2], l[3]);
      pl[2] = pack_halves(l[4], l[5]);
      pl[3] = pack_halves(l[6], l[7]);
#pragma unroll
      for (int nd = 0; nd < 16; nd += 2) {
        if (nd >= ndb) break;
        uint32_t b[4];  // matrices: keys 16 k2 + 0..7 / 8..15 of dims 8 nd.., then of dims 8 nd + 8..
        ldsm_x4_trans(b, sV + (16 * k2 + (lane & 7) + ((lane >> 3) & 1) * 8) * rowb + (8 * nd + (lane >> 4) * 8) * 2);
        mma16816(o[nd], ph, b[0], b[1]);
        mma16816(o[nd], pl, b[0], b[1]);
        mma16816(o[nd + 1], ph, b[2], b[3]);
        mma16816(o[nd + 1], pl, b[2], b[3]);
      }
    }
    __syncthreads();  // the chunk's buffer is read: the next load may take it
  }
  lA += __shfl_xor_sync(0xffffffffu, lA, 1);
  lA += __shfl_xor_sync(0xffffffffu, lA, 2);
  lB += __shfl_xor_sync(0xffffffffu, lB, 1);
  lB += __shfl_xor_sync(0xffffffffu, lB, 2);
  const int tA = rA / KVM, tB = rB / KVM;
  float* outA = out + (long long)(t0 + tA) * ostride + (long long)(kvh * KVM + rA % KVM) * hs;
  float* outB = out + (long long)(t0 + tB) * ostride + (long long)(kvh * KVM + rB % KVM) * hs;
#pragma unroll
  for (int nd = 0; nd < 16; nd++) {
    if (nd >= ndb) break;
    const int d = 8 * nd + 2 * t4;
    if (tA < ntok) {
      outA[d] = o[nd][0] / lA;
      outA[d + 1] = o[nd][1] / lA;
    }
    if (tB < ntok) {
      outB[d] = o[nd][2] / lB;
      outB[d + 1] = o[nd][3] / lB;
    }
  }
}

// The forward driver's step between the q/k/v product and the attention: per head the RMSNorm of q and k (Qwen3's
// q_norm / k_norm, forward/attention.ts:140-143; skipped where the weight is null), RoPE at the position
// (attention.ts:7-20 with the tables' row of pos), and the key and value into the cache at pos (float16 by
// halves.ts's rounding, or float32). Blocks: nh query heads, then nkv key heads, then nkv value heads; blockIdx.y: a
// token of a prefill (its q / k / v stride floats after the previous token's, its position pos + y).
template <bool HALF>
__global__ void qk_rope_cache_kernel(float* q, const float* k, const float* v, const float* qn, const float* kn,
                                     const float* cos_t, const float* sin_t, const int* pos_dev, int pos, void* kc,
                                     void* vc, int nh, int nkv, int hs, int rot, float eps, int* bad,
                                     long long stride) {
  pdl_wait();
  if (pos_dev) pos = *pos_dev;
  pos += blockIdx.y;
  q += blockIdx.y * stride;
  k += blockIdx.y * stride;
  v += blockIdx.y * stride;
  __shared__ float buf[512];
  __shared__ float red[8];
  const int b = blockIdx.x;
  const int kind = b < nh ? 0 : (b < nh + nkv ? 1 : 2);
  const int head = kind == 0 ? b : (kind == 1 ? b - nh : b - nh - nkv);
  const float* src = kind == 0 ? q + (long long)head * hs : (kind == 1 ? k : v) + (long long)head * hs;
  const float* w = kind == 0 ? qn : (kind == 1 ? kn : nullptr);
  for (int d = threadIdx.x; d < hs; d += blockDim.x) buf[d] = src[d];
  __syncthreads();
  if (w) {
    float s = 0.0f;
    for (int d = threadIdx.x; d < hs; d += blockDim.x) s = fmaf(buf[d], buf[d], s);
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    float tot = 0.0f;
    for (int i = 0; i < (int)(blockDim.x >> 5); i++) tot += red[i];
    const float r = 1.0f / sqrtf(tot / (float)hs + eps);
    __syncthreads();
    for (int d = threadIdx.x; d < hs; d += blockDim.x) buf[d] = w[d] * (r * buf[d]);
    __syncthreads();
  }
  if (kind < 2) {
    const int turned = rot > 0 && rot < hs ? rot : hs;
    const float* c = cos_t + (long long)pos * (hs / 2);
    const float* s = sin_t + (long long)pos * (hs / 2);
    for (int i = threadIdx.x; i < turned / 2; i += blockDim.x) {
      const float v0 = buf[2 * i], v1 = buf[2 * i + 1];
      buf[2 * i] = v0 * c[i] - v1 * s[i];
      buf[2 * i + 1] = v0 * s[i] + v1 * c[i];
    }
    __syncthreads();
  }
  if (kind == 0) {
    for (int d = threadIdx.x; d < hs; d += blockDim.x) q[(long long)head * hs + d] = buf[d];
    return;
  }
  void* cache = kind == 1 ? kc : vc;
  const long long at = (long long)pos * nkv * hs + (long long)head * hs;
  int local = 0;
  for (int d = threadIdx.x; d < hs; d += blockDim.x) {
    if (HALF) reinterpret_cast<uint16_t*>(cache)[at + d] = float_to_half_bits(buf[d], &local);
    else reinterpret_cast<float*>(cache)[at + d] = buf[d];
  }
  if (local && bad) atomicAdd(bad, local);
}

}  // namespace

// ---- the registry

PLLM_API void rope(uint64_t v, uint64_t fcr, uint64_t fci, int32_t nh, int32_t hs, int32_t rot) {
  PLLM_REQUIRE(nh >= 0 && hs > 0 && hs % 2 == 0, "rope: nh %d hs %d", nh, hs);
  if (!nh) return;
  const int turned = rot > 0 && rot < hs ? rot : hs;
  const int total = nh * (turned / 2);
  rope_kernel<<<cdiv(total, 256), 256, 0, pllm_stream()>>>(dptr<float>(v), dptr<const float>(fcr),
                                                          dptr<const float>(fci), nh, hs, turned);
  PLLM_LAUNCHED("rope");
}

// att: the reference's scratch of nh (pos + 1) floats; here it holds the slices' partials, and what it holds after
// the call is not the scores (the reference leaves the probabilities there; nothing of its engine reads them)
PLLM_API void attention(uint64_t out, uint64_t q, uint64_t kc, uint64_t vc, uint64_t att, int32_t pos, int32_t nh,
                        int32_t nkv, int32_t hs, int32_t h0, int32_t h1) {
  registry_attention("attention", out, q, kc, vc, att, pos, nh, nkv, hs, h0, h1, 0.0f, false);
}
PLLM_API void attention_f16(uint64_t out, uint64_t q, uint64_t kc, uint64_t vc, uint64_t att, int32_t pos,
                            int32_t nh, int32_t nkv, int32_t hs, int32_t h0, int32_t h1) {
  registry_attention("attention_f16", out, q, kc, vc, att, pos, nh, nkv, hs, h0, h1, 0.0f, true);
}
PLLM_API void attention_capped(uint64_t out, uint64_t q, uint64_t kc, uint64_t vc, uint64_t att, int32_t pos,
                               int32_t nh, int32_t nkv, int32_t hs, int32_t h0, int32_t h1, float cap) {
  PLLM_REQUIRE(cap > 0, "attention_capped: cap %g", cap);
  registry_attention("attention_capped", out, q, kc, vc, att, pos, nh, nkv, hs, h0, h1, cap, false);
}
PLLM_API void attention_f16_capped(uint64_t out, uint64_t q, uint64_t kc, uint64_t vc, uint64_t att, int32_t pos,
                                   int32_t nh, int32_t nkv, int32_t hs, int32_t h0, int32_t h1, float cap) {
  PLLM_REQUIRE(cap > 0, "attention_f16_capped: cap %g", cap);
  registry_attention("attention_f16_capped", out, q, kc, vc, att, pos, nh, nkv, hs, h0, h1, cap, true);
}

// ---- the same attention for callers that cannot allocate device memory
// Some callers cannot hand the attention a scratch buffer: they own a fixed device arena and may not allocate beside
// it (as the reference's engine owns one linear memory and never allocates outside it), or they run where an
// allocation is not allowed or would stall the device (a real-time decode loop, a plugin without access to the
// process's allocator). This variant keeps the slices' partials in a file-scope device array instead: 4 MiB
// (NOALLOC_FLOATS floats), held by every GPU that loads the library until the process exits. A call whose partials
// (nh x slices x (hs + 4) floats, one slice per 128 positions) do not fit is refused with an error.
// The array is shared by every call and keeps the last call's partials; nothing in it has to start at zero (each
// call writes every partial it reads). Calls that overlap on the GPU (two streams, or two threads' streams) race on it.
// The first call on a device looks up the array's device address (cudaGetSymbolAddress, with that device current);
// make that first call before any stream capture.
constexpr long long NOALLOC_FLOATS = 1ll << 20;
static __device__ __align__(256) float g_noalloc_partials[NOALLOC_FLOATS];

namespace {
float* noalloc_partials() {
  static float* ptrs[64] = {nullptr};
  std::lock_guard<std::mutex> hold(pllm_lookup_lock());
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    pllm_fail(PLLM_ECUDA, "pllm_attention_f16_noalloc: no current device");
    return nullptr;
  }
  if (!ptrs[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_partials);
    if (e != cudaSuccess || !p) {
      pllm_fail(PLLM_ECUDA, "pllm_attention_f16_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      return nullptr;
    }
    ptrs[dev] = static_cast<float*>(p);
  }
  return ptrs[dev];
}
}  // namespace

PLLM_API void pllm_attention_f16_noalloc(uint64_t out, uint64_t q, uint64_t kc, uint64_t vc, int32_t pos, int32_t nh,
                                         int32_t nkv, int32_t hs, int32_t h0, int32_t h1) {
  const char* name = "pllm_attention_f16_noalloc";
  if (!check_heads(name, nh, nkv, hs, h0, h1)) return;
  PLLM_REQUIRE(pos >= 0, "%s: pos %d", name, pos);
  PLLM_REQUIRE(!(kc & 15) && !(vc & 15), "%s: the cache must be 16-byte aligned", name);
  const long long nsplit = ((long long)pos + 1 + 127) / 128;
  const long long need = (long long)nh * nsplit * (hs + 4);
  PLLM_REQUIRE(need <= NOALLOC_FLOATS,
               "%s: %d heads of %d at position %d need %lld floats of partials, more than the %lld of the static "
               "scratch (at most %lld positions for this shape)",
               name, nh, hs, pos, need, NOALLOC_FLOATS, NOALLOC_FLOATS / ((long long)nh * (hs + 4)) * 128);
  if (h1 == h0) return;
  float* part = noalloc_partials();
  if (!part) return;
  AttArgs a = {};
  a.out = dptr<float>(out);
  a.q = dptr<const float>(q);
  a.kc = dptr<const void>(kc);
  a.vc = dptr<const void>(vc);
  a.part = part;
  a.pos = pos;
  a.nh = nh;
  a.nkv = nkv;
  a.hs = hs;
  a.h0 = h0;
  a.h1 = h1;
  a.nsplit = (int)nsplit;
  a.split_len = 128;
  run_attention(name, a, true, false);
}

// ---- the forward driver's calls (the position in device memory)

// bytes of scratch pllm_attention_dev needs for a cache of capacity positions: the slices' partials, then a count a
// kv head (the scratch must be zero when first used; every call leaves the counts at zero)
static uint64_t partial_bytes(int nh, int hs, int capacity, int split_len) {
  const long long nsplit = (capacity + split_len - 1) / split_len;
  return ((uint64_t)nh * nsplit * (hs + 4) * sizeof(float) + 255) & ~255ull;
}
PLLM_API uint64_t pllm_attention_scratch_bytes(int32_t nh, int32_t hs, int32_t capacity, int32_t split_len) {
  return partial_bytes(nh, hs, capacity, split_len) + (uint64_t)nh * sizeof(int);
}

PLLM_API void pllm_attention_dev(uint64_t out, uint64_t q, uint64_t kc, uint64_t vc, uint64_t scratch, uint64_t pos_dev,
                                 int32_t capacity, int32_t nh, int32_t nkv, int32_t hs, int32_t half, float cap,
                                 int32_t split_len, int32_t pdl) {
  if (!check_heads("pllm_attention_dev", nh, nkv, hs, 0, nh)) return;
  PLLM_REQUIRE(capacity > 0 && split_len > 0 && split_len <= 2048, "pllm_attention_dev: capacity %d split %d",
               capacity, split_len);
  AttArgs a = {};
  a.out = dptr<float>(out);
  a.q = dptr<const float>(q);
  a.kc = dptr<const void>(kc);
  a.vc = dptr<const void>(vc);
  a.part = dptr<float>(scratch);
  a.pos_dev = dptr<const int>(pos_dev);
  a.nh = nh;
  a.nkv = nkv;
  a.hs = hs;
  a.h0 = 0;
  a.h1 = nh;
  a.split_len = split_len;
  a.nsplit = (capacity + split_len - 1) / split_len;
  a.cap = cap;
  a.counters = dptr<int>(scratch + partial_bytes(nh, hs, capacity, split_len));
  a.capacity = capacity;
  a.status = gemvk::status_word();
  run_attention("pllm_attention_dev", a, half != 0, pdl != 0);
}

// The forward driver's attention step, one launch: q / k head norms (null weights: none), RoPE at the position, this
// position's key and value into the cache, and the attention over positions 0..pos; q, k, v: the q/k/v product's
// output (nh, then nkv, then nkv heads of hs). The position is read from device memory (pos_dev).
PLLM_API void pllm_attention_step(uint64_t out, uint64_t qkv, uint64_t kc, uint64_t vc, uint64_t scratch,
                                  uint64_t pos_dev, int32_t capacity, int32_t nh, int32_t nkv, int32_t hs, int32_t half,
                                  float cap, int32_t split_len, uint64_t q_norm, uint64_t k_norm, uint64_t cos_t,
                                  uint64_t sin_t, int32_t rot, float eps, uint64_t bad, int32_t pdl) {
  if (!check_heads("pllm_attention_step", nh, nkv, hs, 0, nh)) return;
  PLLM_REQUIRE(capacity > 0 && split_len > 0 && split_len <= 2048 && hs % 2 == 0 && pos_dev,
               "pllm_attention_step: capacity %d split %d", capacity, split_len);
  AttArgs a = {};
  a.out = dptr<float>(out);
  a.q = dptr<const float>(qkv);
  a.kc = dptr<const void>(kc);
  a.vc = dptr<const void>(vc);
  a.part = dptr<float>(scratch);
  a.pos_dev = dptr<const int>(pos_dev);
  a.nh = nh;
  a.nkv = nkv;
  a.hs = hs;
  a.h0 = 0;
  a.h1 = nh;
  a.split_len = split_len;
  a.nsplit = (capacity + split_len - 1) / split_len;
  a.cap = cap;
  a.counters = dptr<int>(scratch + partial_bytes(nh, hs, capacity, split_len));
  a.capacity = capacity;
  a.status = gemvk::status_word();
  Fuse f = {};
  f.k = dptr<const float>(qkv) + (long long)nh * hs;
  f.v = f.k + (long long)nkv * hs;
  f.qn = dptr<const float>(q_norm);
  f.kn = dptr<const float>(k_norm);
  f.cos_t = dptr<const float>(cos_t);
  f.sin_t = dptr<const float>(sin_t);
  f.eps = eps;
  f.rot = rot;
  f.bad = dptr<int>(bad);
  run_attention("pllm_attention_step", a, half != 0, pdl != 0, &f);
}

// The same step for a batch of sequences in one launch (grid z a sequence): sequence z's q/k/v at qkv + z
// qkv_stride floats, its output at out + z out_stride floats, its caches at kc / vc + z cache_stride bytes, its
// position pos_dev[z], its scratch the z-th of batch regions of pllm_attention_scratch_bytes rounded up to 256 bytes;
// a float16 cache (each sequence its own positions: no cache row is shared)
PLLM_API void pllm_attention_step_batch(uint64_t out, int64_t out_stride, uint64_t qkv, int64_t qkv_stride,
                                        uint64_t kc, uint64_t vc, int64_t cache_stride, uint64_t scratch,
                                        uint64_t pos_dev, int32_t batch, int32_t capacity, int32_t nh, int32_t nkv,
                                        int32_t hs, float cap, int32_t split_len, uint64_t q_norm, uint64_t k_norm,
                                        uint64_t cos_t, uint64_t sin_t, int32_t rot, float eps, uint64_t bad,
                                        int32_t pdl) {
  if (!check_heads("pllm_attention_step_batch", nh, nkv, hs, 0, nh)) return;
  const uint64_t per = (pllm_attention_scratch_bytes(nh, hs, capacity, split_len) + 255) & ~255ull;
  PLLM_REQUIRE(capacity > 0 && split_len > 0 && split_len <= 2048 && hs % 2 == 0 && pos_dev && batch >= 1 &&
                   batch <= 65535 && out_stride >= (int64_t)nh * hs && qkv_stride >= (int64_t)(nh + 2 * nkv) * hs &&
                   cache_stride % 16 == 0 && cache_stride >= (int64_t)capacity * nkv * hs * 2 && per % 4 == 0,
               "pllm_attention_step_batch: batch %d capacity %d strides %lld %lld %lld", batch, capacity,
               (long long)out_stride, (long long)qkv_stride, (long long)cache_stride);
  AttArgs a = {};
  a.out = dptr<float>(out);
  a.q = dptr<const float>(qkv);
  a.kc = dptr<const void>(kc);
  a.vc = dptr<const void>(vc);
  a.part = dptr<float>(scratch);
  a.pos_dev = dptr<const int>(pos_dev);
  a.nh = nh;
  a.nkv = nkv;
  a.hs = hs;
  a.h0 = 0;
  a.h1 = nh;
  a.split_len = split_len;
  a.nsplit = (capacity + split_len - 1) / split_len;
  a.cap = cap;
  a.counters = dptr<int>(scratch + partial_bytes(nh, hs, capacity, split_len));
  a.batch = batch;
  a.z_out = out_stride;
  a.z_q = qkv_stride;
  a.z_kv = cache_stride;
  a.z_part = (long long)(per / 4);
  a.capacity = capacity;
  a.status = gemvk::status_word();
  Fuse f = {};
  f.k = dptr<const float>(qkv) + (long long)nh * hs;
  f.v = f.k + (long long)nkv * hs;
  f.qn = dptr<const float>(q_norm);
  f.kn = dptr<const float>(k_norm);
  f.cos_t = dptr<const float>(cos_t);
  f.sin_t = dptr<const float>(sin_t);
  f.eps = eps;
  f.rot = rot;
  f.bad = dptr<int>(bad);
  run_attention("pllm_attention_step_batch", a, true, pdl != 0, &f);
}

// 1: the forward driver's float16 attention by clusters (the default); 0: by slices and the last slice's combine.
// Returns the previous mode.
PLLM_API int32_t pllm_set_attention_mode(int32_t mode) {
  const int old = g_cluster_attention;
  if (mode == 0 || mode == 1) g_cluster_attention = mode;
  return old;
}

PLLM_API void pllm_qk_rope_cache(uint64_t q, uint64_t k, uint64_t v, uint64_t q_norm, uint64_t k_norm, uint64_t cos_t,
                                 uint64_t sin_t, uint64_t pos_dev, int32_t pos, uint64_t kc, uint64_t vc, int32_t nh,
                                 int32_t nkv, int32_t hs, int32_t rot, float eps, int32_t half, uint64_t bad,
                                 int32_t pdl) {
  PLLM_REQUIRE(nh > 0 && nkv > 0 && hs > 0 && hs <= 512 && hs % 2 == 0, "pllm_qk_rope_cache: nh %d nkv %d hs %d", nh,
               nkv, hs);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nh + 2 * nkv);
  cfg.blockDim = dim3(hs >= 128 ? 128 : 64);
  cfg.stream = pllm_stream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e;
  if (half)
    e = cudaLaunchKernelEx(&cfg, qk_rope_cache_kernel<true>, dptr<float>(q), dptr<const float>(k), dptr<const float>(v),
                           dptr<const float>(q_norm), dptr<const float>(k_norm), dptr<const float>(cos_t),
                           dptr<const float>(sin_t), dptr<const int>(pos_dev), (int)pos, dptr<void>(kc), dptr<void>(vc),
                           (int)nh, (int)nkv, (int)hs, (int)rot, eps, dptr<int>(bad), 0ll);
  else
    e = cudaLaunchKernelEx(&cfg, qk_rope_cache_kernel<false>, dptr<float>(q), dptr<const float>(k),
                           dptr<const float>(v), dptr<const float>(q_norm), dptr<const float>(k_norm),
                           dptr<const float>(cos_t), dptr<const float>(sin_t), dptr<const int>(pos_dev), (int)pos,
                           dptr<void>(kc), dptr<void>(vc), (int)nh, (int)nkv, (int)hs, (int)rot, eps, dptr<int>(bad),
                           0ll);
  if (e != cudaSuccess) pllm_fail(PLLM_ECUDA, "pllm_qk_rope_cache: %s", cudaGetErrorString(e));
}

// ---- prefill (many tokens at once)

// count tokens' q / k head norms (null weights: none), RoPE at positions p0.., and their keys and values into the
// cache: qkv rows stride floats apart (a token's nh q heads, nkv k heads, nkv v heads, as the q/k/v product writes)
PLLM_API void pllm_qk_rope_cache_rows(uint64_t qkv, int64_t stride, uint64_t q_norm, uint64_t k_norm, uint64_t cos_t,
                                      uint64_t sin_t, int32_t p0, int32_t count, uint64_t kc, uint64_t vc, int32_t nh,
                                      int32_t nkv, int32_t hs, int32_t rot, float eps, int32_t half, uint64_t bad) {
  PLLM_REQUIRE(nh > 0 && nkv > 0 && hs > 0 && hs <= 512 && hs % 2 == 0 && p0 >= 0 && count >= 0 &&
                   stride >= (int64_t)(nh + 2 * nkv) * hs,
               "pllm_qk_rope_cache_rows: nh %d nkv %d hs %d p0 %d count %d", nh, nkv, hs, p0, count);
  if (!count) return;
  const dim3 grid(nh + 2 * nkv, count);
  const int threads = hs >= 128 ? 128 : 64;
  float* q = dptr<float>(qkv);
  const float* k = q + (long long)nh * hs;
  const float* v = k + (long long)nkv * hs;
  if (half)
    qk_rope_cache_kernel<true><<<grid, threads, 0, pllm_stream()>>>(
        q, k, v, dptr<const float>(q_norm), dptr<const float>(k_norm), dptr<const float>(cos_t),
        dptr<const float>(sin_t), nullptr, p0, dptr<void>(kc), dptr<void>(vc), nh, nkv, hs, rot, eps, dptr<int>(bad),
        (long long)stride);
  else
    qk_rope_cache_kernel<false><<<grid, threads, 0, pllm_stream()>>>(
        q, k, v, dptr<const float>(q_norm), dptr<const float>(k_norm), dptr<const float>(cos_t),
        dptr<const float>(sin_t), nullptr, p0, dptr<void>(kc), dptr<void>(vc), nh, nkv, hs, rot, eps, dptr<int>(bad),
        (long long)stride);
  PLLM_LAUNCHED("pllm_qk_rope_cache_rows");
}

// count tokens (positions p0..) attend causally over a float16 cache that holds positions 0 .. p0 + count - 1: q
// from qkv rows (qstride floats apart, the nh q heads first), out rows ostride floats apart (nh x hs)
PLLM_API void pllm_attention_prefill(uint64_t out, int64_t ostride, uint64_t qkv, int64_t qstride, uint64_t kc,
                                     uint64_t vc, int32_t p0, int32_t count, int32_t nh, int32_t nkv, int32_t hs) {
  if (!check_heads("pllm_attention_prefill", nh, nkv, hs, 0, nh)) return;
  PLLM_REQUIRE(hs <= 128 && p0 >= 0 && count >= 0 && !(kc & 15) && !(vc & 15),
               "pllm_attention_prefill: hs %d (at most 128), p0 %d count %d, 16-byte aligned caches", hs, p0, count);
  if (!count) return;
  const int kvm = nh / nkv;
  const size_t rowb = (size_t)hs * 2 + 16;
  const size_t smem = 2 * PF_ROWS * rowb + 4 * PF_KEYS * rowb;
  const int qt = PF_ROWS / kvm;
  const dim3 grid(nkv, (count + qt - 1) / qt);
  cudaError_t e = cudaSuccess;
  auto run = [&](auto kernel) {
    cudaError_t r = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (r != cudaSuccess) return r;
    kernel<<<grid, PF_THREADS, smem, pllm_stream()>>>(dptr<float>(out), (long long)ostride, dptr<const float>(qkv),
                                                     (long long)qstride, dptr<const uint16_t>(kc),
                                                     dptr<const uint16_t>(vc), p0, count, nkv, hs);
    return cudaGetLastError();
  };
  switch (kvm) {
    case 1: e = run(attention_prefill_kernel<1>); break;
    case 2: e = run(attention_prefill_kernel<2>); break;
    case 4: e = run(attention_prefill_kernel<4>); break;
    default: e = run(attention_prefill_kernel<8>); break;
  }
  if (e != cudaSuccess) pllm_fail(PLLM_ECUDA, "pllm_attention_prefill: %s", cudaGetErrorString(e));
}
