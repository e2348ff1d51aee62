// attention.cu: RoPE, the cache write, and one token's attention over the cache (kernels/kernel/attention.ts).
//   rope                       attention.ts:7-20
//   attention, attention_f16   attention.ts:28-36 (attentionOf :87-211)
//   attention_capped, attention_f16_capped   attention.ts:40-45
// The cache is the reference's layout: a layer's keys (and values) [position][kv heads * head size], float32 or the
// float16 bits halves.ts writes. Grouped-query: q head h reads kv head h / (nh / nkv).
//
// B200 form: split-KV ("flash decoding"). A CTA takes one kv head and a slice of the positions for all of that head's
// query heads (the keys and values of the slice are read once for kvMul heads): scores in shared memory, a softmax
// of the slice (its max and sum), and the weighted values. A second small kernel combines the slices' partial
// results (max, sum, weighted values) per head. With one slice the first kernel writes the output itself.
// The numbers differ from the reference's in the order of the float32 sums and in exp (CUDA's expf in place of the
// reference's table-free one): the outputs agree within float32 rounding (the tests hold them to 1e-5 relative).
//
// The forward driver's calls read the position from device memory (pos_dev), so that one CUDA graph serves every
// position; their grid covers the cache's capacity and the slices past the position return at once.
#include "pllm_common.cuh"

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
};


// grid (nkv, nsplit): one kv head's slice of positions for its KVM query heads. The slice is taken TILE positions at
// a time: every thread first issues its 16-byte loads of the tile's keys and values (all of them in flight at once),
// into shared memory (rows padded by 16 bytes: conflict-free 16-byte reads of a row by consecutive threads), then the
// scores (a thread a position and head pair), an online softmax of the slice (running max and sum, the partial
// output rescaled), and the weighted values (a thread a head dimension).
constexpr int TILE = 64;

template <bool HALF>
__device__ __forceinline__ float kv_elem(const uint8_t* row, int d) {
  if (HALF) return half_bits_to_float(reinterpret_cast<const uint16_t*>(row)[d]);
  return reinterpret_cast<const float*>(row)[d];
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
__device__ __forceinline__ void split_half(float x, __half& hi, __half& lo) {
  hi = __float2half_rn(x);
  lo = __float2half_rn(x - __half2float(hi));
}

// a head of hs floats in shared memory normalized (w: null for none) and turned at pos by one warp (no block-wide
// barrier: the heads of a CTA go one a warp, side by side)
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

template <bool HALF, int KVM, bool FUSE>
__global__ void __launch_bounds__(ATT_THREADS) attention_split_kernel(const AttArgs a, const Fuse f) {
  extern __shared__ __align__(16) uint8_t att_smem[];
  constexpr int E = HALF ? 2 : 4;
  constexpr int HP = 8;                              // heads padded to the products' n = 8
  const int hs = a.hs;
  const int rowb = hs * E + 16;                      // a padded row of the tile, bytes (16-byte rows, no conflicts)
  const int tileb = TILE * rowb;
  uint8_t* ring = att_smem;                          // [2 buffers][K tile, V tile]: 4 x tileb bytes
  float* sq = reinterpret_cast<float*>(ring + 4 * tileb);  // [KVM][hs]
  float* sp = sq + KVM * hs;                         // [KVM][TILE] scores, then probabilities
  float* sx = sp + KVM * TILE;                       // [2][hs] (FUSE) this position's key and value
  __half* sqh = reinterpret_cast<__half*>(sx + 2 * hs);  // [HP][hs] q's high halves (HALF), then its low halves
  __half* sql = sqh + HP * hs;
  __half* sph = sql + HP * hs;                       // [HP][TILE] probabilities' high halves, then low halves
  __half* spl = sph + HP * TILE;
  __shared__ float sM[KVM], sL[KVM], sScale[KVM];
  // the position: written by the host before the step's first kernel, so readable before the dependency wait
  const int pos = a.pos_dev ? *a.pos_dev : a.pos;
  const int count = pos + 1;
  const int kvh = blockIdx.x, split = blockIdx.y;
  const int nsplit = a.pos_dev ? (count + a.split_len - 1) / a.split_len : a.nsplit;
  if (split >= nsplit) return;
  const int p0 = split * a.split_len;
  const int p1 = min(count, p0 + a.split_len);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t4 = lane & 3;            // an mma fragment's row group and column pair
  const int kvdim = a.nkv * hs, hbase = kvh * KVM;
  const float isq = 1.0f / sqrtf((float)hs);
  const int chunks = hs * E / 16;                    // 16-byte pieces a row
  const uint8_t* kbase = reinterpret_cast<const uint8_t*>(a.kc) + (long long)kvh * hs * E;
  const uint8_t* vbase = reinterpret_cast<const uint8_t*>(a.vc) + (long long)kvh * hs * E;
  // a tile's keys and values by asynchronous 16-byte copies, all in flight at once (positions before this token's:
  // not the previous kernel's output); rows past the tile's length zeroed (a probability of 0 must meet a 0)
  auto load_tile = [&](int t0, int buf) {
    uint8_t* sK = ring + (size_t)(2 * buf) * tileb;
    uint8_t* sV = sK + tileb;
    const int len = min(TILE, p1 - t0);
    for (int e = tid; e < TILE * chunks; e += ATT_THREADS) {
      const int t = e / chunks, c = e % chunks;
      if (t < len) {
        const long long off = (long long)(t0 + t) * kvdim * E + c * 16;
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
    if (holds_pos) {  // this position's key and value into the cache
      int local = 0;
      for (int e = tid; e < 2 * hs; e += ATT_THREADS) {
        const int d = e % hs;
        uint8_t* cache = reinterpret_cast<uint8_t*>(const_cast<void*>(e < hs ? a.kc : a.vc)) + (long long)pos * kvdim * E +
                         ((long long)kvh * hs + d) * E;
        if (HALF) *reinterpret_cast<uint16_t*>(cache) = float_to_half_bits(sx[e], &local);
        else *reinterpret_cast<float*>(cache) = sx[e];
      }
      if (local && f.bad) atomicAdd(f.bad, local);
    }
  }
  if (HALF) {  // q as two float16 halves a value, the padded heads zero
    for (int e = tid; e < HP * hs; e += ATT_THREADS) {
      const int j = e / hs;
      __half hi = __float2half_rn(0.0f), lo = hi;
      if (j < KVM) split_half(sq[e], hi, lo);
      sqh[e] = hi;
      sql[e] = lo;
    }
    for (int e = tid; e < HP * TILE; e += ATT_THREADS) {
      sph[e] = __float2half_rn(0.0f);
      spl[e] = __float2half_rn(0.0f);
    }
  }
  // the running output. HALF: mma fragments of O^T (dims x heads), m-blocks of 16 dims warp, warp + 4, ...;
  // else a thread a dimension d = tid + ATT_THREADS i of every head
  constexpr int DMAX = 2;   // hs <= 256
  constexpr int MBMAX = 4;  // hs / 16 / ATT_WARPS
  float acc[KVM][DMAX];
  float oc[MBMAX][4];
#pragma unroll
  for (int j = 0; j < KVM; j++)
#pragma unroll
    for (int i = 0; i < DMAX; i++) acc[j][i] = 0.0f;
#pragma unroll
  for (int m = 0; m < MBMAX; m++)
#pragma unroll
    for (int c = 0; c < 4; c++) oc[m][c] = 0.0f;
  const int nmb = hs / 16;
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
      for (int e = tid; e < 2 * hs; e += ATT_THREADS) {
        const int d = e % hs;
        uint8_t* tile = (e < hs ? sK : sV) + (size_t)(pos - t0) * rowb + d * E;
        int dummy = 0;
        if (HALF) *reinterpret_cast<uint16_t*>(tile) = float_to_half_bits(sx[e], &dummy);
        else *reinterpret_cast<float*>(tile) = sx[e];
      }
      __syncthreads();
    }
    // 2. scores
    if (HALF) {  // a warp 16 positions: S (positions x heads) = K (positions x dims) . q^T, the halves' two products
      float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const uint8_t* arow = sK + (16 * warp + (lane & 7) + ((lane >> 3) & 1) * 8) * rowb + (lane >> 4) * 16;
      for (int kk = 0; kk < nmb; kk++) {
        uint32_t af[4];
        ldsm_x4(af, arow + kk * 32);
        const int qo = g * hs + 16 * kk + 2 * t4;
        mma16816(c, af, *reinterpret_cast<const uint32_t*>(sqh + qo), *reinterpret_cast<const uint32_t*>(sqh + qo + 8));
        mma16816(c, af, *reinterpret_cast<const uint32_t*>(sql + qo), *reinterpret_cast<const uint32_t*>(sql + qo + 8));
      }
#pragma unroll
      for (int r = 0; r < 4; r++) {
        const int t = 16 * warp + g + (r >> 1) * 8, j = 2 * t4 + (r & 1);
        if (j < KVM) {
          float v = -INFINITY;
          if (t < len) {
            v = c[r] * isq;
            if (a.cap > 0.0f) v = a.cap * tanhf(v / a.cap);
          }
          sp[j * TILE + t] = v;
        }
      }
    } else {  // a thread a (position, head) pair
      for (int e = tid; e < KVM * TILE; e += ATT_THREADS) {
        const int t = e % TILE, j = e / TILE;
        float sc = -INFINITY;
        if (t < len) {
          const uint8_t* row = sK + t * rowb;
          const float* qj = sq + j * hs;
          sc = 0.0f;
          for (int c = 0; c < chunks; c++) {
            const int4 w = *reinterpret_cast<const int4*>(row + c * 16);
            const uint32_t u[4] = {(uint32_t)w.x, (uint32_t)w.y, (uint32_t)w.z, (uint32_t)w.w};
#pragma unroll
            for (int k = 0; k < 4; k++) sc = fmaf(qj[c * 4 + k], __uint_as_float(u[k]), sc);
          }
          sc *= isq;
          if (a.cap > 0.0f) sc = a.cap * tanhf(sc / a.cap);
        }
        sp[j * TILE + t] = sc;
      }
    }
    __syncthreads();
    // 3. the online softmax: a warp a head
    for (int j = warp; j < KVM; j += ATT_WARPS) {
      float m = -INFINITY;
      for (int t = lane; t < len; t += 32) m = fmaxf(m, sp[j * TILE + t]);
      m = warp_max(m);
      const float mnew = fmaxf(sM[j], m);
      float l = 0.0f;
      for (int t = lane; t < TILE; t += 32) {
        const float p = t < len ? expf(sp[j * TILE + t] - mnew) : 0.0f;
        sp[j * TILE + t] = p;
        if (HALF) split_half(p, sph[j * TILE + t], spl[j * TILE + t]);
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
    // 4. the weighted values
    if (HALF) {  // O^T (dims x heads) += V^T (dims x positions) . P^T (positions x heads), the halves' two products
      const float s0 = 2 * t4 < KVM ? sScale[2 * t4] : 1.0f, s1 = 2 * t4 + 1 < KVM ? sScale[2 * t4 + 1] : 1.0f;
#pragma unroll
      for (int mi = 0; mi < MBMAX; mi++) {
        const int mb = warp + ATT_WARPS * mi;
        if (mb >= nmb) break;
        oc[mi][0] *= s0;
        oc[mi][1] *= s1;
        oc[mi][2] *= s0;
        oc[mi][3] *= s1;
        const uint8_t* vrow = sV + ((lane & 7) + ((lane >> 4) & 1) * 8) * rowb + (16 * mb + ((lane >> 3) & 1) * 8) * 2;
#pragma unroll
        for (int ks = 0; ks < TILE / 16; ks++) {
          uint32_t af[4];
          ldsm_x4_trans(af, vrow + ks * 16 * rowb);
          const int po = g * TILE + 16 * ks + 2 * t4;
          mma16816(oc[mi], af, *reinterpret_cast<const uint32_t*>(sph + po), *reinterpret_cast<const uint32_t*>(sph + po + 8));
          mma16816(oc[mi], af, *reinterpret_cast<const uint32_t*>(spl + po), *reinterpret_cast<const uint32_t*>(spl + po + 8));
        }
      }
    } else {  // a thread a dimension
#pragma unroll
      for (int i = 0; i < DMAX; i++) {
        const int d = tid + ATT_THREADS * i;
        if (d >= hs) continue;
#pragma unroll
        for (int j = 0; j < KVM; j++) acc[j][i] *= sScale[j];
        for (int t = 0; t < len; t++) {
          const float v = kv_elem<HALF>(sV + t * rowb, d);
#pragma unroll
          for (int j = 0; j < KVM; j++) acc[j][i] = fmaf(sp[j * TILE + t], v, acc[j][i]);
        }
      }
    }
    // the tile after next into this buffer, once every warp is done with it
    if (t0 + 2 * TILE < p1) {
      __syncthreads();
      load_tile(t0 + 2 * TILE, buf);
    }
  }
  // 5. the slice's output (one slice: the head's output itself)
  auto put = [&](int j, int d, float v) {
    const int h = hbase + j;
    if (j >= KVM || h < a.h0 || h >= a.h1) return;
    if (nsplit == 1) {
      a.out[(long long)h * hs + d] = v / sL[j];
    } else {
      float* part = a.part + ((long long)h * a.nsplit + split) * (hs + 4);
      part[d] = v;
      if (d == 0) {
        part[hs] = sM[j];
        part[hs + 1] = sL[j];
      }
    }
  };
  if (HALF) {
#pragma unroll
    for (int mi = 0; mi < MBMAX; mi++) {
      const int mb = warp + ATT_WARPS * mi;
      if (mb >= nmb) break;
      put(2 * t4, 16 * mb + g, oc[mi][0]);
      put(2 * t4 + 1, 16 * mb + g, oc[mi][1]);
      put(2 * t4, 16 * mb + g + 8, oc[mi][2]);
      put(2 * t4 + 1, 16 * mb + g + 8, oc[mi][3]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < DMAX; i++) {
      const int d = tid + ATT_THREADS * i;
      if (d >= hs) continue;
#pragma unroll
      for (int j = 0; j < KVM; j++) put(j, d, acc[j][i]);
    }
  }
  if (nsplit == 1 || !a.counters) return;
  // 6. the last slice of this kv head to finish combines every slice's partials (no CTA waits for another: the
  // others are done when the count reaches nsplit), and sets the count back to zero for the next call. The partials
  // of the kv head's query heads are contiguous: copied into shared memory by asynchronous 16-byte copies, as many
  // slices at once as the tile ring holds (every copy of a chunk in flight together).
  __shared__ int last;
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(&a.counters[kvh], 1) == nsplit - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const int row = hs + 4;                                    // floats a slice's partial (16-byte rows)
  const int room = (int)((4 * (size_t)tileb) / ((size_t)KVM * row * 4));  // slices a chunk
  float* stage = reinterpret_cast<float*>(ring);
  float* sw = sp;  // [KVM][nsplit] weights exp(m_s - M), in the scores' room (the host sizes it for nsplit)
  float o[KVM][DMAX];
#pragma unroll
  for (int j = 0; j < KVM; j++)
#pragma unroll
    for (int i = 0; i < DMAX; i++) o[j][i] = 0.0f;
  for (int c0 = 0; c0 < nsplit; c0 += room) {
    const int cn = min(room, nsplit - c0);
    const int per4 = cn * row / 4;                           // 16-byte pieces a head's chunk
    __syncthreads();  // the previous chunk is read
    for (int e = tid; e < KVM * per4; e += ATT_THREADS) {
      const int j = e / per4, f4 = e % per4;
      cp_async16(stage + 4 * e, a.part + ((long long)(hbase + j) * a.nsplit + c0) * row + 4 * f4);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    cp_async_wait_all();
    __syncthreads();
    if (c0 == 0) {  // the maxima and sums of every slice (the first chunk holds them when room >= nsplit; else from L2)
      for (int j = warp; j < KVM; j += ATT_WARPS) {
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
    for (int i = 0; i < DMAX; i++) {
      const int d = tid + ATT_THREADS * i;
      if (d >= hs) continue;
#pragma unroll
      for (int j = 0; j < KVM; j++)
        for (int s2 = 0; s2 < cn; s2++) o[j][i] = fmaf(stage[(j * cn + s2) * row + d], sw[j * nsplit + c0 + s2], o[j][i]);
    }
  }
#pragma unroll
  for (int i = 0; i < DMAX; i++) {
    const int d = tid + ATT_THREADS * i;
    if (d >= hs) continue;
#pragma unroll
    for (int j = 0; j < KVM; j++) {
      const int h = hbase + j;
      if (h >= a.h0 && h < a.h1) a.out[(long long)h * hs + d] = o[j][i] / sL[j];
    }
  }
  if (tid == 0) a.counters[kvh] = 0;
}

// a block a head: the slices' partials combined
__global__ void attention_combine_kernel(const AttArgs a) {
  pdl_wait();
  const int pos = a.pos_dev ? *a.pos_dev : a.pos;
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

template <bool HALF, int KVM>
cudaError_t launch_split_kvm(const AttArgs& a, const Fuse* f, size_t smem, dim3 grid, bool pdl) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(ATT_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = pllm_stream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
if (f) {
    auto k = attention_split_kernel<HALF, KVM, true>;
    if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return cudaLaunchKernelEx(&cfg, k, a, *f);
  }
  const Fuse none = {};
  auto k = attention_split_kernel<HALF, KVM, false>;
  if (smem > 48 * 1024) cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  return cudaLaunchKernelEx(&cfg, k, a, none);
}

template <bool HALF>
cudaError_t launch_split(const AttArgs& a, const Fuse* f, int kvm, size_t smem, dim3 grid, bool pdl) {
  switch (kvm) {
    case 1: return launch_split_kvm<HALF, 1>(a, f, smem, grid, pdl);
    case 2: return launch_split_kvm<HALF, 2>(a, f, smem, grid, pdl);
    case 4: return launch_split_kvm<HALF, 4>(a, f, smem, grid, pdl);
    case 8: return launch_split_kvm<HALF, 8>(a, f, smem, grid, pdl);
    default: return cudaErrorInvalidValue;
  }
}

void run_attention(const char* name, AttArgs a, bool half, bool pdl, const Fuse* f = nullptr) {
  const int kvm = a.nh / a.nkv;
  const size_t rowb = (size_t)a.hs * (half ? 2 : 4) + 16;
  // the scores' room also holds the slices' weights in the combine (kvm * nsplit floats)
  const size_t scores = (size_t)kvm * (a.nsplit > TILE ? a.nsplit : TILE) * 4;
  const size_t halves = half ? (2 * 8 * (size_t)a.hs + 2 * 8 * TILE) * 2 : 0;
  const size_t smem = 4 * TILE * rowb + (size_t)kvm * a.hs * 4 + scores + 2 * (size_t)a.hs * 4 + halves;
  const dim3 grid(a.nkv, a.nsplit);
  cudaError_t e = half ? launch_split<true>(a, f, kvm, smem, grid, pdl) : launch_split<false>(a, f, kvm, smem, grid, pdl);
  if (e != cudaSuccess) {
    pllm_fail(PLLM_ECUDA, "%s: launch failed: %s", name, cudaGetErrorString(e));
    return;
  }
  if ((a.nsplit > 1 || a.pos_dev) && !a.counters) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.h1 - a.h0);
    cfg.blockDim = dim3(a.hs >= 128 ? 128 : 64);
    cfg.stream = pllm_stream();
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
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

// The forward driver's step between the q/k/v product and the attention: per head the RMSNorm of q and k (Qwen3's
// q_norm / k_norm, forward/attention.ts:140-143; skipped where the weight is null), RoPE at the position
// (attention.ts:7-20 with the tables' row of pos), and the key and value into the cache at pos (float16 by
// halves.ts's rounding, or float32). Blocks: nh query heads, then nkv key heads, then nkv value heads.
template <bool HALF>
__global__ void qk_rope_cache_kernel(float* q, const float* k, const float* v, const float* qn, const float* kn,
                                     const float* cos_t, const float* sin_t, const int* pos_dev, int pos, void* kc,
                                     void* vc, int nh, int nkv, int hs, int rot, float eps, int* bad) {
  pdl_wait();
  if (pos_dev) pos = *pos_dev;
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
                           (int)nh, (int)nkv, (int)hs, (int)rot, eps, dptr<int>(bad));
  else
    e = cudaLaunchKernelEx(&cfg, qk_rope_cache_kernel<false>, dptr<float>(q), dptr<const float>(k),
                           dptr<const float>(v), dptr<const float>(q_norm), dptr<const float>(k_norm),
                           dptr<const float>(cos_t), dptr<const float>(sin_t), dptr<const int>(pos_dev), (int)pos,
                           dptr<void>(kc), dptr<void>(vc), (int)nh, (int)nkv, (int)hs, (int)rot, eps, dptr<int>(bad));
  if (e != cudaSuccess) pllm_fail(PLLM_ECUDA, "pllm_qk_rope_cache: %s", cudaGetErrorString(e));
}
