// gemv_tma.cu: the decode product as a bulk-copy pipeline (the forward driver's and the registry's int8 products at
// one to sixteen tokens, int6 and ternary products at one).
//
// One CTA an SM, warp-specialized: a producer warp streams the CTA's rows of weights and their scales from HBM into
// a ring of shared-memory stages with cp.async.bulk (the TMA's bulk engine; completion counted on an mbarrier per
// stage, L2 evict-first: each weight byte is read once), and eight consumer warps take a row each of every stage:
// dp4a of the row's groups of 32 against the activations (shared memory, made by the consumers in the prologue),
// each group's exact int32 times the product of its two scales, summed in float32, reduced across the warp.
//
// The weights do not depend on the kernel ahead of this one in the stream, so the producer starts streaming before
// the programmatic-dependent-launch wait; only the consumers wait (griddepcontrol.wait) before reading the
// activations. Every wait on an mbarrier is bounded: past the bound the kernel records PLLM_ETIMEOUT in the device
// status word and returns (the host reads it with pllm_device_status).
//
// A stage holds TR = 8 rows x KS columns (KS = K, or K cut into equal chunks of at most 8192): rows whole are one
// contiguous copy of 8 x K bytes (and one of 8 x K/32 scales); rows cut into chunks are a copy a row. Consumer warp w
// takes row w of every stage (for one token of rows of at most 4096, a lane's activation groups held in registers).
//
// The rows are dealt as tiles of 8 from a ticket counter, not as fixed shares: each CTA's producer takes the next
// tile's ticket while the current tile streams, so the CTAs that start early (on SMs the kernel ahead leaves first)
// stream more of the matrix and none waits at the end for a late one's fixed share. Until its consumers have their
// activations a CTA takes no more than its even share of the tiles (Dealer): one that starts early would fill its
// whole ring while the kernel ahead still runs, then consume those tiles one after another while the CTAs that start
// later find none (measured on the 4096 x 4096 product after attention: 6 tiles on 68 CTAs, none on 18). A tile is
// all its stages in a row
// (EPI_SWIGLU: its w1 rows, then the same rows of w3; K cut into chunks: a stage a chunk), and the producer writes the
// tile's first row and row count into the stage's header before the copies' barrier completes, so a consumer warp
// reads it after its wait, with no barrier among the consumers. Every CTA's producer takes exactly one ticket past the
// tiles; the one that takes the last of those (tiles + grid - 1) sets the counter back to zero for the launch that
// next uses it. Rows cut into chunks (K > 8192) keep fixed shares: their tiles are two stages or more, and the last
// tile dealt ends the launch later than even shares do (measured at K = 12288).
#include "gemv_common.cuh"
#include <atomic>

__device__ int g_pllm_status = 0;  // a bounded wait gave up (PLLM_ETIMEOUT), read by pllm_device_status

// the launches' ticket counters: a launch takes the next of them in turn (host side), so two launches share one only
// TICKET_SLOTS launches apart on a device, long after the first has finished
constexpr int TICKET_SLOTS = 1024;
__device__ unsigned g_tickets[TICKET_SLOTS];

namespace {

using namespace gemvk;

constexpr int NC = 8;                 // consumer warps
constexpr int TR = NC;                // row slots a stage (a row a consumer warp)
constexpr int TRP = TR;               // the product kernel's tile rows
constexpr int TMA_THREADS = (NC + 1) * 32;
constexpr long long WAIT_BOUND = 1ll << 26;  // polls of an mbarrier before giving up (seconds: never in a run that works)

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
// true once the phase of the given parity has completed; false (and the status word set) past the bound
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
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
  atomicExch(&g_pllm_status, PLLM_ETIMEOUT);
  return false;
}
__device__ __forceinline__ void bulk_copy(void* dst, const void* src, unsigned bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(NC * 32) : "memory"); }
struct ConsumerSync {
  __device__ __forceinline__ void operator()() const { consumer_sync(); }
};

struct TmaPlan {
  int stages;       // S
  int ks;           // columns a chunk
  int chunks;       // K / ks
  int stage_bytes;  // TR * ks * 1.125, 128-aligned
  int act_bytes;    // activations and their scales, 128-aligned
  int slot;         // this launch's ticket counter (g_tickets)
  int tickets;      // 1: tiles dealt by tickets; 0: each CTA its own share of the rows (rows cut into chunks)
  int nred;         // the batched form's buffers of the warps' parts (stages + 2)
  int rw;           // the ternary form's rows a consumer warp (a tile NC rw rows)
};

// The ticket dealing of one CTA's producer (see the file's head). started: set by the consumers once they have their
// activations.
struct Dealer {
  unsigned* ticket;
  unsigned fair, taken;
  const volatile int* started;
  __device__ Dealer(unsigned* t, unsigned tiles, const int* st)
      : ticket(t), fair((tiles + gridDim.x - 1) / gridDim.x), taken(0), started(st) {}
  // the next ticket; past an even share, not before the consumers have started (a bounded wait: a hint only)
  __device__ __forceinline__ unsigned take() {
    if (taken >= fair)
      for (long long i = 0; !*started && i < WAIT_BOUND; i++) __nanosleep(32);
    taken++;
    return atomicAdd(ticket, 1u);
  }
};

// this CTA's rows: [lo, hi) of [r0, r1), near-equal shares
__device__ __forceinline__ void cta_rows(const GemvArgs& a, long long& lo, long long& hi) {
  const long long rows = a.r1 - a.r0, G = gridDim.x, c = blockIdx.x;
  const long long base = rows / G, rem = rows % G;
  lo = a.r0 + c * base + (c < rem ? c : rem);
  hi = lo + base + (c < rem ? 1 : 0);
}

// a group of 32 of one row (its two 16-byte halves at w, read in the lane's order: no bank conflicts) against the
// activations' halves read in the same order: the group's integer (the same sum in any order)
__device__ __forceinline__ int group_dot(const uint8_t* w, int swz, const int4 xa, const int4 xb) {
  const int4 wa = *reinterpret_cast<const int4*>(w + 16 * swz);
  const int4 wb = *reinterpret_cast<const int4*>(w + 16 * (swz ^ 1));
  int g0 = __dp4a(wa.x, xa.x, 0), g1 = __dp4a(wb.x, xb.x, 0);
  g0 = __dp4a(wa.y, xa.y, g0);
  g1 = __dp4a(wb.y, xb.y, g1);
  g0 = __dp4a(wa.z, xa.z, g0);
  g1 = __dp4a(wb.z, xb.z, g1);
  g0 = __dp4a(wa.w, xa.w, g0);
  g1 = __dp4a(wb.w, xb.w, g1);
  return g0 + g1;
}

// The producer (one thread): the tiles' stages into the ring, dealt by tickets or as this CTA's share (see the file's
// head). PAD: each row at KS + 16 bytes from the one before in the stage (one copy a row: the batched tensor-core
// consumer's fragment reads are then free of bank conflicts), the scales after TRP such rows.
template <int PHASES, bool PAD>
__device__ __forceinline__ void produce(const GemvArgs& a, const TmaPlan& p, uint64_t* full, uint64_t* empty, int* hdr,
                                        uint8_t* stage0, const int* started) {
  const int S = p.stages, KS = p.ks, chunks = p.chunks, K = a.K, ng = K / 32;
  const int RS = PAD ? KS + 16 : KS;
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  const unsigned tiles = (unsigned)((a.r1 - a.r0 + TRP - 1) / TRP);
  unsigned* ticket = g_tickets + p.slot;
  long long lo = a.r0, hi = a.r1;  // the rows this CTA streams: all of them by tickets, or its own share
  if (!p.tickets) cta_rows(a, lo, hi);
  Dealer deal(ticket, tiles, started);
  unsigned next = p.tickets ? deal.take() : 0u;
  long long it = 0;
  for (long long ts = lo;;) {
    long long t;
    if (p.tickets) {
      if (next >= tiles) break;
      t = a.r0 + (long long)next * TRP;
      next = deal.take();  // the following tile's ticket, on its way while this tile streams
    } else {
      if (ts >= hi) break;
      t = ts;
      ts += TRP;
    }
    const int n = (int)min((long long)TRP, hi - t);
    for (int ph = 0; ph < PHASES; ph++) {
      const long long row0 = t + (ph ? a.pair : 0);
      for (int c = 0; c < chunks; c++, it++) {
        const int slot = (int)(it % S);
        if (!mbar_wait(&empty[slot], ((unsigned)(it / S) & 1) ^ 1)) return;
        uint8_t* w = stage0 + (size_t)slot * p.stage_bytes;
        float* sc = reinterpret_cast<float*>(w + (size_t)TRP * RS);
        // the tile's first row (from r0) and its rows, seen by the consumers once the stage's barrier completes
        // (the expect_tx arrive releases it)
        hdr[slot] = (int)(((t - a.r0) << 4) | n);
        mbar_expect_tx(&full[slot], (unsigned)(n * (KS + KS / 8)));
        if (chunks == 1 && !PAD) {
          bulk_copy(w, a.wq + row0 * K, (unsigned)(n * K), &full[slot], policy);
          bulk_copy(sc, reinterpret_cast<const float*>(a.ws) + row0 * ng, (unsigned)(n * ng * 4), &full[slot], policy);
        } else {
          for (int r = 0; r < n; r++)
            bulk_copy(w + (size_t)r * RS, a.wq + (row0 + r) * K + (long long)c * KS, (unsigned)KS, &full[slot], policy);
          if (chunks == 1) {
            bulk_copy(sc, reinterpret_cast<const float*>(a.ws) + row0 * ng, (unsigned)(n * ng * 4), &full[slot],
                      policy);
          } else {
            for (int r = 0; r < n; r++)
              bulk_copy(sc + (size_t)r * (KS / 32),
                        reinterpret_cast<const float*>(a.ws) + (row0 + r) * ng + (long long)c * (KS / 32),
                        (unsigned)(KS / 8), &full[slot], policy);
          }
        }
      }
    }
  }
  // the end: a stage without rows
  const int slot = (int)(it % S);
  if (!mbar_wait(&empty[slot], ((unsigned)(it / S) & 1) ^ 1)) return;
  hdr[slot] = -1;
  mbar_arrive(&full[slot]);
  if (p.tickets && next == tiles + gridDim.x - 1) atomicExch(ticket, 0u);  // the last ticket of the launch
}

// a finished row's value of token t: stored, added, or sent to the ranks' exchange slots
template <int EPI>
__device__ __forceinline__ void emit(const GemvArgs& a, const Xchg& xg, int t, long long row, float v) {
  float* o = a.out + t * a.out_stride + row;
  if (EPI == EPI_SEND) {
    const unsigned mark = xchg_mark(xg);
    for (int r = 0; r < xg.world; r++) st_slot(xg.dst[r] + row, v, mark);
  } else if (EPI == EPI_ADD) {
    add_once(o, v);
  } else {
    *o = v;
  }
}

template <int MT, int PRO, int EPI>
__global__ void __launch_bounds__(TMA_THREADS, 1) gemv_tma_kernel(const GemvArgs a, const TmaPlan p, const Xchg xg) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int S = p.stages, KS = p.ks, chunks = p.chunks, K = a.K, ng = K / 32;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + S;
  int* hdr = reinterpret_cast<int*>(smem + 16 * S);  // [S] a stage's tile: its first row from r0 x 16 + its rows; -1: the end
  int* started = hdr + S;                            // the consumers have their activations
  uint8_t* act = smem + ((20 * S + 4 + 127) & ~127);
  int8_t* sq = reinterpret_cast<int8_t*>(act);
  float* ss = reinterpret_cast<float*>(act + (size_t)MT * K);
  uint8_t* stage0 = act + p.act_bytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // EPI_SWIGLU: a tile's w1 rows, then the same rows of w3 (at + pair); warp w makes row w of both, so the w1 result
  // waits in a register
  constexpr int PHASES = EPI == EPI_SWIGLU ? 2 : 1;
  const int per_tile = PHASES * chunks;  // stages a tile

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NC);
    }
    *started = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == NC) {  // ---- the producer
    if (lane == 0) produce<PHASES, false>(a, p, full, empty, hdr, stage0, started);
    return;
  }

  // ---- the consumers (a wait that gives up ends the warp: there is no barrier among the consumers past the prologue)
  pdl_wait();
  load_activations<F_Q8, MT, PRO, ConsumerSync>(a, sq, ss, nullptr, &xg);
  consumer_sync();
  if (threadIdx.x == 0) *reinterpret_cast<volatile int*>(started) = 1;
  pdl_launch_dependents();
  const int swz = (lane >> 2) & 1;  // which half of its 32 bytes a lane reads first: no bank conflicts
  // one token and rows of at most 32 x RG groups in one chunk: a lane's activation groups (the same for every row) and
  // their scales held in registers, so that a row's shared-memory reads are its weights only
  constexpr int RG = 4;
  const bool reg = MT == 1 && chunks == 1 && KS / 32 <= 32 * RG;
  int4 ra[RG], rb[RG];
  float rx[RG];
#pragma unroll
  for (int k = 0; k < RG; k++) {
    const int u = lane + 32 * k;
    ra[k] = rb[k] = make_int4(0, 0, 0, 0);
    rx[k] = 0.0f;
    if (reg && u < KS / 32) {
      ra[k] = *reinterpret_cast<const int4*>(sq + (size_t)u * 32 + 16 * swz);
      rb[k] = *reinterpret_cast<const int4*>(sq + (size_t)u * 32 + 16 * (swz ^ 1));
      rx[k] = ss[u];
    }
  }
  float h1 = 0.0f;  // EPI_SWIGLU: this lane's w1 result of the tile's row
  long long it = 0;
  for (;;) {
    float acc[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) acc[m] = 0.0f;
    for (int k = 0; k < per_tile; k++, it++) {
      const int slot = (int)(it % S);
      if (!mbar_wait(&full[slot], (unsigned)(it / S) & 1)) return;
      const int tile = hdr[slot];
      if (tile < 0) return;  // no more tiles (only ever the first stage of a tile)
      const int c = k % chunks, ph = k / chunks;
      const long long row = a.r0 + (tile >> 4) + warp;
      const bool mine = warp < (tile & 15);
      if (mine) {
        const uint8_t* w = stage0 + (size_t)slot * p.stage_bytes + (size_t)warp * KS;
        const float* sc = reinterpret_cast<const float*>(stage0 + (size_t)slot * p.stage_bytes + (size_t)TRP * KS) +
                          (size_t)warp * (KS / 32);
        const int u0 = c * (KS / 32);
        // the groups in the order u = lane, lane + 32, ...
        if (MT == 1 && reg) {
#pragma unroll
          for (int k2 = 0; k2 < RG; k2++) {
            const int u = lane + 32 * k2;
            if (u >= KS / 32) break;
            const int G = group_dot(w + u * 32, swz, ra[k2], rb[k2]);
            acc[0] = fmaf((float)G, __fmul_rn(sc[u], rx[k2]), acc[0]);
          }
        } else {
          for (int u = lane; u < KS / 32; u += 32) {
            const float s = sc[u];
#pragma unroll
            for (int m = 0; m < MT; m++) {
              const int8_t* x = sq + (size_t)m * K + (size_t)(u0 + u) * 32;
              const int4 xa = *reinterpret_cast<const int4*>(x + 16 * swz);
              const int4 xb = *reinterpret_cast<const int4*>(x + 16 * (swz ^ 1));
              const int G = group_dot(w + u * 32, swz, xa, xb);
              acc[m] = fmaf((float)G, __fmul_rn(s, ss[m * ng + u0 + u]), acc[m]);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (c != chunks - 1 || !mine) continue;
      // the row of this phase is done
#pragma unroll
      for (int m = 0; m < MT; m++) acc[m] = warp_sum(acc[m]);
      float v = acc[0];
#pragma unroll
      for (int m = 1; m < MT; m++)
        if (lane == m) v = acc[m];
#pragma unroll
      for (int m = 0; m < MT; m++) acc[m] = 0.0f;
      if (lane >= MT || lane >= a.count) continue;
      if (EPI == EPI_SWIGLU) {
        if (ph == 0) h1 = v;
        else a.out[lane * a.out_stride + row] = (h1 / (1.0f + expf(-h1))) * v;
      } else {
        emit<EPI>(a, xg, lane, row, v);
      }
    }
  }
}

// ---- the batched form (3..16 tokens, the registry's tiles and a batch of sequences): each group of 32 of a stage's
// rows is one tensor-core product (mma.sync m16n8k32, int8 x int8 -> int32, 16 tokens x 8 rows), whose int32 are the
// exact group sums (the same integers as every other form; tokens past count are zeros), each scaled by ws x xs and
// summed in float32. The consumer warps split a stage's groups (warp w: groups w, w + 8, ...), so each holds a part of
// the tile's 16 x 8 sums; at the end of a tile's phase each posts its part in shared memory and the last to post adds
// them (in warp order) and writes the outputs. Activations: ASMEM, all tokens in shared memory (rows padded by
// 16 bytes: conflict-free fragment reads), made by the prologue; else (K too long for shared memory) the caller's
// quantized activations read from global memory (L2) fragment by fragment.
constexpr int MB = 16;                      // tokens of the batched form

__device__ __forceinline__ void mma_s8(int c[4], const uint32_t a[4], const uint32_t b[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
__device__ __forceinline__ void ldsm_x4(uint32_t r[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x2(uint32_t r[2], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(smem_u32(p)));
}
// an exact int32 of magnitude below 2^22 as float32: its bits added to those of 1.5 x 2^23, that float less 1.5 x 2^23
__device__ __forceinline__ float exact_float(int v) {
  return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.0f);
}

// The batched kernel's shared memory: the barriers, headers and the phase-ends' arrival counts in the first 512
// bytes, then nred buffers of the warps' parts (NC x 128 floats each), nred buffers of w1's results (EPI_SWIGLU, 128
// floats each), the activations, the stages.
constexpr int MMA_HEAD = 512;
constexpr int RED_FLOATS = NC * 128;

// one group of 32 of the stage (its u-th): the tokens' fragment (shared memory, or the caller's activations in global
// memory), the weights' fragment, the tensor-core product, its exact int32 scaled into the lane's four sums
template <bool ASMEM>
__device__ __forceinline__ void mma_group(float acc[4], const int8_t* sq, int AS, const float* sst, int uu, int a_tok,
                                          int a_off, int g, const uint8_t* xg0, const uint8_t* xg1, const float* xs0,
                                          const float* xs1, bool tok0, bool tok1, unsigned bias4, const uint8_t* brow,
                                          float w0, float w1, int t4, uint32_t af[4], uint32_t bf[2], float& x0,
                                          float& x1, bool load) {
  if (load) {
    if (ASMEM) {
      ldsm_x4(af, sq + (size_t)a_tok * AS + (size_t)uu * 32 + a_off);
      x0 = sst[uu * MB + g];
      x1 = sst[uu * MB + g + 8];
    } else {
      const long long o = (long long)uu * 32 + 4 * t4;
      af[0] = tok0 ? __vsub4(__ldg(reinterpret_cast<const unsigned*>(xg0 + o)), bias4) : 0u;
      af[1] = tok1 ? __vsub4(__ldg(reinterpret_cast<const unsigned*>(xg1 + o)), bias4) : 0u;
      af[2] = tok0 ? __vsub4(__ldg(reinterpret_cast<const unsigned*>(xg0 + o + 16)), bias4) : 0u;
      af[3] = tok1 ? __vsub4(__ldg(reinterpret_cast<const unsigned*>(xg1 + o + 16)), bias4) : 0u;
      x0 = tok0 ? __ldg(xs0 + uu) : 0.0f;
      x1 = tok1 ? __ldg(xs1 + uu) : 0.0f;
    }
    ldsm_x2(bf, brow);
    return;
  }
  int cf[4] = {0, 0, 0, 0};
  mma_s8(cf, af, bf);
  acc[0] = fmaf(exact_float(cf[0]), __fmul_rn(w0, x0), acc[0]);
  acc[1] = fmaf(exact_float(cf[1]), __fmul_rn(w1, x0), acc[1]);
  acc[2] = fmaf(exact_float(cf[2]), __fmul_rn(w0, x1), acc[2]);
  acc[3] = fmaf(exact_float(cf[3]), __fmul_rn(w1, x1), acc[3]);
}

template <int PRO, int EPI, bool ASMEM>
__global__ void __launch_bounds__(TMA_THREADS, 1) gemv_tma_mma_kernel(const GemvArgs a, const TmaPlan p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int S = p.stages, KS = p.ks, chunks = p.chunks, K = a.K, ng = K / 32, RS = KS + 16, AS = K + 16;
  const int NRED = p.nred;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + S;
  int* hdr = reinterpret_cast<int*>(smem + 16 * S);
  int* cnt = reinterpret_cast<int*>(smem + 20 * S);  // [NRED] the warps arrived at a phase-end
  int* started = cnt + NRED;                         // the consumers have their activations
  float* red = reinterpret_cast<float*>(smem + MMA_HEAD);  // [NRED][NC][128]
  float* hsave = red + NRED * RED_FLOATS;                     // [NRED][128]
  uint8_t* act = reinterpret_cast<uint8_t*>(hsave + NRED * 128);
  int8_t* sq = reinterpret_cast<int8_t*>(act);                         // ASMEM: [MB][AS]
  float* ss = reinterpret_cast<float*>(act + (size_t)MB * AS);         //        [MB][ng]
  float* sst = ss + MB * ng;                                           //        [ng][MB]: by group
  uint8_t* stage0 = act + p.act_bytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  constexpr int PHASES = EPI == EPI_SWIGLU ? 2 : 1;

  if (tid == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NC);
    }
    for (int i = 0; i < NRED; i++) cnt[i] = 0;
    *started = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == NC) {
    if (lane == 0) produce<PHASES, true>(a, p, full, empty, hdr, stage0, started);
    return;
  }
  pdl_wait();
  if (ASMEM) {
    load_activations<F_Q8, MB, PRO, ConsumerSync>(a, sq, ss, nullptr, nullptr, (size_t)AS);
    consumer_sync();
    for (int i = tid; i < MB * ng; i += NC * 32) sst[(i % ng) * MB + i / ng] = ss[i];
    consumer_sync();
  }
  if (tid == 0) *reinterpret_cast<volatile int*>(started) = 1;
  pdl_launch_dependents();
  const int g = lane >> 2, t4 = lane & 3;
  // ldmatrix rows: A (tokens (lane & 7) + 8 ((lane >> 3) & 1), bytes 16 (lane >> 4) of a group), B (weight rows lane & 7,
  // bytes 16 ((lane >> 3) & 1))
  const int a_tok = (lane & 7) + 8 * ((lane >> 3) & 1), a_off = 16 * (lane >> 4);
  const int b_row = lane & 7, b_off = 16 * ((lane >> 3) & 1);
  // ASMEM off: this lane's tokens g and g + 8 in the caller's activations (q - 64 where they are biased)
  const uint8_t* xg0 = a.xq + (long long)g * a.xq_stride;
  const uint8_t* xg1 = a.xq + (long long)(g + 8) * a.xq_stride;
  const float* xs0 = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(a.xs) + (long long)g * a.xs_stride);
  const float* xs1 =
      reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(a.xs) + (long long)(g + 8) * a.xs_stride);
  const bool tok0 = g < a.count, tok1 = g + 8 < a.count;
  const unsigned bias4 = a.bias ? 0x40404040u : 0u;
  long long it = 0, pe = 0;  // stages taken, phase-ends passed (the same sequence in every warp)
  for (;;) {
    int tile = 0;
    for (int ph = 0; ph < PHASES; ph++, pe++) {
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int c = 0; c < chunks; c++, it++) {
        const int slot = (int)(it % S);
        if (!mbar_wait(&full[slot], (unsigned)(it / S) & 1)) return;  // every consumer warp gives up at this stage
        tile = hdr[slot];
        if (tile < 0) return;  // no more tiles (only ever the first stage of a tile)
        const uint8_t* w = stage0 + (size_t)slot * p.stage_bytes;
        const float* sc = reinterpret_cast<const float*>(w + (size_t)TRP * RS);
        const int gs = KS / 32, u0 = c * gs;
        const float* ws0 = sc + (2 * t4) * gs;
        const float* ws1 = ws0 + gs;
        const uint8_t* brow = w + (size_t)b_row * RS + b_off;
        // two groups an iteration: both groups' fragments loaded before either product
        for (int u = warp; u < gs; u += 2 * NC) {
          const bool two = u + NC < gs;
          uint32_t af0[4], af1[4], bf0[2], bf1[2];
          float x00 = 0.0f, x01 = 0.0f, x10 = 0.0f, x11 = 0.0f;
          mma_group<ASMEM>(acc, sq, AS, sst, u0 + u, a_tok, a_off, g, xg0, xg1, xs0, xs1, tok0, tok1, bias4,
                           brow + (size_t)u * 32, 0.0f, 0.0f, t4, af0, bf0, x00, x01, true);
          if (two)
            mma_group<ASMEM>(acc, sq, AS, sst, u0 + u + NC, a_tok, a_off, g, xg0, xg1, xs0, xs1, tok0, tok1, bias4,
                             brow + (size_t)(u + NC) * 32, 0.0f, 0.0f, t4, af1, bf1, x10, x11, true);
          mma_group<ASMEM>(acc, sq, AS, sst, 0, a_tok, a_off, g, xg0, xg1, xs0, xs1, tok0, tok1, bias4, brow,
                           ws0[u], ws1[u], t4, af0, bf0, x00, x01, false);
          if (two)
            mma_group<ASMEM>(acc, sq, AS, sst, 0, a_tok, a_off, g, xg0, xg1, xs0, xs1, tok0, tok1, bias4, brow,
                             ws0[u + NC], ws1[u + NC], t4, af1, bf1, x10, x11, false);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
      }
      // the tile's phase is done: this warp's part posted; the last warp to post adds the parts in warp order and
      // writes the outputs (no warp waits for another). A warp runs at most S stages ahead of the slowest, so the
      // nred = S + 2 buffers are not reused while read.
      const int b = (int)(pe % NRED);
      float* rb = red + b * RED_FLOATS;
      *reinterpret_cast<float4*>(rb + warp * 128 + 4 * lane) = make_float4(acc[0], acc[1], acc[2], acc[3]);
      __syncwarp();
      int last = 0;
      if (lane == 0) {
        __threadfence_block();
        last = atomicAdd(&cnt[b], 1) == NC - 1;
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) continue;
      __threadfence_block();
      for (int e = lane; e < 128; e += 32) {
        float v = 0.0f;
#pragma unroll
        for (int w2 = 0; w2 < NC; w2++) v += rb[w2 * 128 + e];
        const int el = e >> 2, i = e & 3;
        const int token = (el >> 2) + (i >= 2 ? 8 : 0), r = 2 * (el & 3) + (i & 1);
        if (EPI == EPI_SWIGLU && ph == 0) {
          hsave[b * 128 + e] = v;  // w1's result, read by the phase that follows (its last warp)
          continue;
        }
        if (r < (tile & 15) && token < a.count) {
          const long long row = a.r0 + (tile >> 4) + r;
          float* o = a.out + token * a.out_stride + row;
          if (EPI == EPI_SWIGLU) {
            const float h1 = hsave[(int)((pe - 1) % NRED) * 128 + e];
            *o = (h1 / (1.0f + expf(-h1))) * v;
          } else if (EPI == EPI_ADD) {
            add_once(o, v);
          } else {
            *o = v;
          }
        }
      }
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        cnt[b] = 0;
      }
    }
  }
}

template <int PRO, int EPI, bool ASMEM>
bool launch_mma(const GemvArgs& a, const TmaPlan& p, size_t smem, bool pdl) {
  auto kernel = gemv_tma_mma_kernel<PRO, EPI, ASMEM>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return false;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)gemv_tma_grid(a.r1 - a.r0, EPI));
  cfg.blockDim = dim3(TMA_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = pllm_stream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, a, p);
  if (e != cudaSuccess) pllm_fail(PLLM_ECUDA, "gemv_tma (batched) launch: %s", cudaGetErrorString(e));
  return true;
}

// ---- ternary weights at one token (the 27B-class decoder's products): the same pipeline, a stage TRP rows of K / 4
// bytes of 2-bit codes (ternary.ts:25-33: weight j's code w + 1 at bits 2 (j & 3) of byte j / 4) and then the rows'
// float16 scales a group of 128; tiles dealt by tickets. The consumers unpack the codes in registers against the
// activations in the interleave's layout (matmul.ts:106-146: byte 16 p + c of a block of 64 is activation 4 c + p, so
// (word >> 2 p) & 0x03030303 holds four codes whose activations are four consecutive bytes; ternary_group), each
// group of 32's exact sum of codes times activations plus the group's minus-sum (the + 1 of the codes taken out) times
// its scale, times the group of 128's scale (relaxed/signs.ts:28-55). A unit of 128 activations is 8 chunks of 16
// bytes, chunk c of unit u stored at slot c ^ (u & 7): the lanes' reads of consecutive units do not share banks.
constexpr int T2_STAGES = 16;

// four unsigned bytes of a times four signed bytes of b, plus c (dp4a.u32.s32)
__device__ __forceinline__ int dp4a_us(unsigned a, int b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// a tile's whole rows a stage: the rows' codes, then their scales (ternary: K / 4 code bytes and a float16 scale a
// group of 128; int6: K / 32 x 24 code bytes and a float32 scale a group of 32)
template <int FMT, int PHASES>
__device__ __forceinline__ void produce_rows(const GemvArgs& a, const TmaPlan& p, uint64_t* full, uint64_t* empty,
                                             int* hdr, uint8_t* stage0, const int* started) {
  const int S = p.stages, K = a.K, T = NC * p.rw;
  const int cb = FMT == F_Q6 ? K / 32 * 24 : K / 4;        // a row's code bytes
  const int sb = FMT == F_Q6 ? K / 32 * 4 : K / 128 * 2;  // and its scale bytes
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  const unsigned tiles = (unsigned)((a.r1 - a.r0 + T - 1) / T);
  unsigned* ticket = g_tickets + p.slot;
  Dealer deal(ticket, tiles, started);
  unsigned next = deal.take();
  long long it = 0;
  while (next < tiles) {
    const long long t = a.r0 + (long long)next * T;
    next = deal.take();
    const int n = (int)min((long long)T, a.r1 - t);
    for (int ph = 0; ph < PHASES; ph++, it++) {
      const long long row0 = t + (ph ? a.pair : 0);
      const int slot = (int)(it % S);
      if (!mbar_wait(&empty[slot], ((unsigned)(it / S) & 1) ^ 1)) return;
      uint8_t* w = stage0 + (size_t)slot * p.stage_bytes;
      hdr[slot] = (int)(((t - a.r0) << 6) | n);
      mbar_expect_tx(&full[slot], (unsigned)(n * (cb + sb)));
      bulk_copy(w, a.wq + row0 * cb, (unsigned)(n * cb), &full[slot], policy);
      bulk_copy(w + (size_t)T * cb, reinterpret_cast<const uint8_t*>(a.ws) + row0 * sb, (unsigned)(n * sb),
                &full[slot], policy);
    }
  }
  const int slot = (int)(it % S);
  if (!mbar_wait(&empty[slot], ((unsigned)(it / S) & 1) ^ 1)) return;
  hdr[slot] = -1;
  mbar_arrive(&full[slot]);
  if (next == tiles + gridDim.x - 1) atomicExch(ticket, 0u);
}

template <int PRO, int EPI>
__global__ void __launch_bounds__(TMA_THREADS, 1) gemv_tma_t2_kernel(const GemvArgs a, const TmaPlan p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int S = p.stages, K = a.K, ng = K / 32, units = K / 128, cb = K / 4;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + S;
  int* hdr = reinterpret_cast<int*>(smem + 16 * S);
  int* started = hdr + S;  // the consumers have their activations
  uint8_t* act = smem + ((20 * T2_STAGES + 4 + 127) & ~127);
  int8_t* sq = reinterpret_cast<int8_t*>(act);            // [K] the prologue's activations, in order
  uint8_t* si = act + K;                                   // [K] interleaved, chunks swizzled
  float* ss = reinterpret_cast<float*>(act + 2 * (size_t)K);  // [ng] scales
  int* sm = reinterpret_cast<int*>(ss + ng);                  // [ng] minus-sums
  uint8_t* stage0 = act + p.act_bytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  constexpr int PHASES = EPI == EPI_SWIGLU ? 2 : 1;
  if (tid == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NC);
    }
    *started = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == NC) {
    if (lane == 0) produce_rows<F_T2, PHASES>(a, p, full, empty, hdr, stage0, started);
    return;
  }
  pdl_wait();
  if (PRO == PRO_Q) {  // the caller's interleaved activations, their scales, then their minus-sums (interleave())
    for (int e = tid; e < K / 16; e += NC * 32) {
      const int u = e >> 3, c = e & 7;
      *reinterpret_cast<int4*>(si + (size_t)u * 128 + 16 * (c ^ (u & 7))) = reinterpret_cast<const int4*>(a.xq)[e];
    }
    for (int i = tid; i < ng; i += NC * 32) {
      ss[i] = a.xs[i];
      sm[i] = reinterpret_cast<const int*>(a.xs + ng)[i];
    }
  } else {  // RMSNorm / quantize_x of float32 x, then the interleave and each group's minus-sum here
    load_activations<F_Q8, 1, PRO, ConsumerSync>(a, sq, ss, nullptr, nullptr);
    consumer_sync();
    for (int b = tid; b < K / 64; b += NC * 32) {
      uint32_t v[16];
#pragma unroll
      for (int k = 0; k < 4; k++) {
        const int4 q = reinterpret_cast<const int4*>(sq + 64 * (size_t)b)[k];
        v[4 * k] = (uint32_t)q.x;
        v[4 * k + 1] = (uint32_t)q.y;
        v[4 * k + 2] = (uint32_t)q.z;
        v[4 * k + 3] = (uint32_t)q.w;
      }
      int s0 = 0, s1 = 0;
#pragma unroll
      for (int k = 0; k < 8; k++) {
        s0 = __dp4a((int)v[k], 0x01010101, s0);
        s1 = __dp4a((int)v[8 + k], 0x01010101, s1);
      }
      sm[2 * b] = -s0;
      sm[2 * b + 1] = -s1;
      // plane p, byte c = activation 4 c + p = byte p of word c: plane word q from byte p of words 4 q .. 4 q + 3
      const int u = b >> 1, h = b & 1;
#pragma unroll
      for (int pl = 0; pl < 4; pl++) {
        const unsigned sel = (unsigned)pl | ((unsigned)(pl + 4) << 4);
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; q++)
          o[q] = __byte_perm(__byte_perm(v[4 * q], v[4 * q + 1], sel), __byte_perm(v[4 * q + 2], v[4 * q + 3], sel),
                             0x5410);
        const int c = 4 * h + pl;
        *reinterpret_cast<uint4*>(si + (size_t)u * 128 + 16 * (c ^ (u & 7))) = make_uint4(o[0], o[1], o[2], o[3]);
      }
    }
  }
  consumer_sync();
  if (tid == 0) *reinterpret_cast<volatile int*>(started) = 1;
  pdl_launch_dependents();
  constexpr int RWM = 4;  // the most rows a warp
  const int rw = p.rw, T = NC * rw;
  float h1[RWM] = {0.0f, 0.0f, 0.0f, 0.0f};  // EPI_SWIGLU: this warp's rows' w1 results
  long long it = 0;
  for (;;) {
    for (int ph = 0; ph < PHASES; ph++, it++) {
      const int slot = (int)(it % S);
      if (!mbar_wait(&full[slot], (unsigned)(it / S) & 1)) return;
      const int tile = hdr[slot];
      if (tile < 0) return;
      const int mine = min(rw, (tile & 63) - warp * rw);  // this warp's rows of the tile
      float acc[RWM] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (mine > 0) {
        const uint8_t* w = stage0 + (size_t)slot * p.stage_bytes + (size_t)warp * rw * cb;
        const uint16_t* d16 = reinterpret_cast<const uint16_t*>(stage0 + (size_t)slot * p.stage_bytes +
                                                                (size_t)T * cb) + (size_t)warp * rw * units;
        // half units of 64 weights (16 code bytes; one block of the interleave), lane after lane along the row: the
        // block's activations read once for the warp's rows
        for (int hu = lane; hu < 2 * units; hu += 32) {
          const int u = hu >> 1, h = hu & 1;
          int4 av[4];
#pragma unroll
          for (int pl = 0; pl < 4; pl++)
            av[pl] = *reinterpret_cast<const int4*>(si + (size_t)u * 128 + 16 * ((4 * h + pl) ^ (u & 7)));
          const int m0 = sm[4 * u + 2 * h], m1 = sm[4 * u + 2 * h + 1];
          const float x0 = ss[4 * u + 2 * h], x1 = ss[4 * u + 2 * h + 1];
#pragma unroll
          for (int r = 0; r < RWM; r++) {
            if (r >= mine) break;
            const uint4 cw = *reinterpret_cast<const uint4*>(w + (size_t)r * cb + (size_t)u * 32 + 16 * h);
            // plane p's codes left in place (times 4^p, unsigned bytes up to 192) against the signed activations: 4^p
            // times the plane's sum, exactly; the planes' sums shifted back and added
            int q0[4], q1[4];
#pragma unroll
            for (int pl = 0; pl < 4; pl++) {
              const unsigned m = 0x03030303u << (2 * pl);
              q0[pl] = dp4a_us(cw.x & m, av[pl].x, 0);
              q0[pl] = dp4a_us(cw.y & m, av[pl].y, q0[pl]);
              q1[pl] = dp4a_us(cw.z & m, av[pl].z, 0);
              q1[pl] = dp4a_us(cw.w & m, av[pl].w, q1[pl]);
            }
            const int g0 = q0[0] + (q0[1] >> 2) + (q0[2] >> 4) + (q0[3] >> 6);
            const int g1 = q1[0] + (q1[1] >> 2) + (q1[2] >> 4) + (q1[3] >> 6);
            const float d = half_bits_to_float(d16[(size_t)r * units + u]);
            acc[r] += __fmul_rn(__fmul_rn((float)(g0 + m0), x0), d) + __fmul_rn(__fmul_rn((float)(g1 + m1), x1), d);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
#pragma unroll
      for (int r = 0; r < RWM; r++) {
        if (r >= mine) break;
        const float v = warp_sum(acc[r]);
        if (lane != 0) continue;
        const long long row = a.r0 + (tile >> 6) + warp * rw + r;
        if (EPI == EPI_SWIGLU) {
          if (ph == 0) h1[r] = v;
          else a.out[row] = (h1[r] / (1.0f + expf(-h1[r]))) * v;
        } else if (EPI == EPI_ADD) {
          add_once(a.out + row, v);
        } else {
          a.out[row] = v;
        }
      }
    }
  }
}

template <int PRO, int EPI>
bool launch_t2(const GemvArgs& a, const TmaPlan& p, size_t smem, bool pdl) {
  auto kernel = gemv_tma_t2_kernel<PRO, EPI>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return false;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)gemv_tma_grid(a.r1 - a.r0, EPI));
  cfg.blockDim = dim3(TMA_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = pllm_stream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, a, p);
  if (e != cudaSuccess) pllm_fail(PLLM_ECUDA, "gemv_tma (ternary) launch: %s", cudaGetErrorString(e));
  return true;
}

// ---- int6 weights at one token (matmul.ts:227, relaxed/six.ts:16): the same pipeline, a stage NC rw whole rows of
// K / 32 x 24 bytes of codes (a group of 32: the low nibbles of its 32 values in 16 bytes, their top two bits in 8)
// and then the rows' float32 scales a group of 32; tiles dealt by tickets. A lane takes a row's groups lane, lane +
// 32, ... in order and widens each group's 24 bytes to eight words of int8 (widen6_regs: 4 v) against the group's
// activations: the register kernel's order of every sum, so the same bits as matmul_q6 / q6r there.
template <int PRO, int EPI>
__global__ void __launch_bounds__(TMA_THREADS, 1) gemv_tma_q6_kernel(const GemvArgs a, const TmaPlan p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int S = p.stages, K = a.K, ng = K / 32, cb = ng * 24;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + S;
  int* hdr = reinterpret_cast<int*>(smem + 16 * S);
  int* started = hdr + S;  // the consumers have their activations
  uint8_t* act = smem + ((20 * T2_STAGES + 4 + 127) & ~127);
  int8_t* sq = reinterpret_cast<int8_t*>(act);          // [K] signed activations
  float* ss = reinterpret_cast<float*>(act + (size_t)K);  // [ng] their scales
  uint8_t* stage0 = act + p.act_bytes;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  constexpr int PHASES = EPI == EPI_SWIGLU ? 2 : 1;
  if (tid == 0) {
    for (int s = 0; s < S; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NC);
    }
    *started = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (warp == NC) {
    if (lane == 0) produce_rows<F_Q6, PHASES>(a, p, full, empty, hdr, stage0, started);
    return;
  }
  pdl_wait();
  load_activations<F_Q6, 1, PRO, ConsumerSync>(a, sq, ss, nullptr, nullptr);
  consumer_sync();
  if (tid == 0) *reinterpret_cast<volatile int*>(started) = 1;
  pdl_launch_dependents();
  constexpr int RWM = 4;  // the most rows a warp
  const int rw = p.rw, T = NC * rw;
  float h1[RWM] = {0.0f, 0.0f, 0.0f, 0.0f};  // EPI_SWIGLU: this warp's rows' w1 results
  long long it = 0;
  for (;;) {
    for (int ph = 0; ph < PHASES; ph++, it++) {
      const int slot = (int)(it % S);
      if (!mbar_wait(&full[slot], (unsigned)(it / S) & 1)) return;
      const int tile = hdr[slot];
      if (tile < 0) return;
      const int mine = min(rw, (tile & 63) - warp * rw);  // this warp's rows of the tile
      float acc[RWM] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (mine > 0) {
        const uint8_t* w = stage0 + (size_t)slot * p.stage_bytes + (size_t)warp * rw * cb;
        const float* d32 = reinterpret_cast<const float*>(stage0 + (size_t)slot * p.stage_bytes + (size_t)T * cb) +
                           (size_t)warp * rw * ng;
        // two groups a step (g and g + 32: independent loads and products, added in order); the groups' activations
        // read once for the warp's rows
        for (int g = lane; g < ng; g += 64) {
          const bool two = g + 32 < ng;
          const int h = two ? g + 32 : g;
          const int4 a0 = *reinterpret_cast<const int4*>(sq + 32 * (size_t)g);
          const int4 a1 = *reinterpret_cast<const int4*>(sq + 32 * (size_t)g + 16);
          const int4 b0 = *reinterpret_cast<const int4*>(sq + 32 * (size_t)h);
          const int4 b1 = *reinterpret_cast<const int4*>(sq + 32 * (size_t)h + 16);
          const float xs = ss[g], xt = ss[h];
#pragma unroll
          for (int r = 0; r < RWM; r++) {
            if (r >= mine) break;
            const uint8_t* c = w + (size_t)r * cb + 24 * (size_t)g;
            const uint8_t* e = w + (size_t)r * cb + 24 * (size_t)h;
            const uint2 v0 = *reinterpret_cast<const uint2*>(c), v1 = *reinterpret_cast<const uint2*>(c + 8),
                        v2 = *reinterpret_cast<const uint2*>(c + 16);
            const uint2 u0 = *reinterpret_cast<const uint2*>(e), u1 = *reinterpret_cast<const uint2*>(e + 8),
                        u2 = *reinterpret_cast<const uint2*>(e + 16);
            const float s0 = d32[(size_t)r * ng + g], s1 = d32[(size_t)r * ng + h];
            uint32_t wd[8], wu[8];
            widen6_regs(v0.x, v0.y, v1.x, v1.y, v2.x, v2.y, wd);
            widen6_regs(u0.x, u0.y, u1.x, u1.y, u2.x, u2.y, wu);
            const int G = dot32_words(wd, a0, a1), H = dot32_words(wu, b0, b1);
            const float f = fmaf((float)G, __fmul_rn(s0, xs), acc[r]);
            acc[r] = two ? fmaf((float)H, __fmul_rn(s1, xt), f) : f;
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
#pragma unroll
      for (int r = 0; r < RWM; r++) {
        if (r >= mine) break;
        const float v = warp_sum(acc[r]);
        if (lane != 0) continue;
        const long long row = a.r0 + (tile >> 6) + warp * rw + r;
        if (EPI == EPI_SWIGLU) {
          if (ph == 0) h1[r] = v;
          else a.out[row] = (h1[r] / (1.0f + expf(-h1[r]))) * v;
        } else if (EPI == EPI_ADD) {
          add_once(a.out + row, v);
        } else {
          a.out[row] = v;
        }
      }
    }
  }
}

template <int PRO, int EPI>
bool launch_q6(const GemvArgs& a, const TmaPlan& p, size_t smem, bool pdl) {
  auto kernel = gemv_tma_q6_kernel<PRO, EPI>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return false;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)gemv_tma_grid(a.r1 - a.r0, EPI));
  cfg.blockDim = dim3(TMA_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = pllm_stream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, a, p);
  if (e != cudaSuccess) pllm_fail(PLLM_ECUDA, "gemv_tma (int6) launch: %s", cudaGetErrorString(e));
  return true;
}

template <int MT, int PRO, int EPI>
bool launch(const GemvArgs& a, const TmaPlan& p, size_t smem, bool pdl, const Xchg& xg) {
  auto kernel = gemv_tma_kernel<MT, PRO, EPI>;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return false;
  const long long grid = gemv_tma_grid(a.r1 - a.r0, EPI);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(TMA_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = pllm_stream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, a, p, xg);
  if (e != cudaSuccess) {
    pllm_fail(PLLM_ECUDA, "gemv_tma launch: %s", cudaGetErrorString(e));
    return true;  // failed, but not for want of a fit: do not fall back
  }
  return true;
}

}  // namespace

namespace gemvk {

// the stage budget: a stage ring of about this many bytes (a smaller one leaves room on the SM for the next
// kernel's CTA); the default takes what one CTA may have
int g_tma_budget = 180 * 1024;  // (measured best of 160..226 KB on the Qwen3-8B step)
// 0: the bulk-copy kernel wherever it applies; 1: the register-streaming kernel only (for comparisons)
int g_gemv_mode = 0;

// the device address of the status word on the current device (looked up once a device)
int* status_word() {
  static int* addr[64] = {nullptr};
  std::lock_guard<std::mutex> hold(pllm_lookup_lock());
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    pllm_fail(PLLM_ECUDA, "gemv_tma: no current device");
    return nullptr;
  }
  if (!addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_pllm_status);
    if (e != cudaSuccess) {
      pllm_fail(PLLM_ECUDA, "gemv_tma: the status word: %s", cudaGetErrorString(e));
      return nullptr;
    }
    addr[dev] = static_cast<int*>(p);
  }
  return addr[dev];
}

// a device's launches take its ticket counters in turn (from any host thread)
unsigned next_ticket_slot(int dev) {
  static std::atomic<unsigned> next_slot[64];
  return next_slot[dev & 63].fetch_add(1u, std::memory_order_relaxed);
}

int gemv_tma_grid(long long rows, int epi) {
  (void)epi;  // a tile is TRP rows of one matrix in every form (EPI_SWIGLU: of w1, then of w3)
  const long long tiles = (rows + TRP - 1) / TRP;
  const long long sms = pllm_num_sms();
  return (int)(tiles < sms ? tiles : sms);
}

// The batched form (3..16 tokens): stages of at most 4096 columns (rows padded), the activations in shared memory
// where they fit beside two stages, else (the caller's quantized activations only) read from global memory.
bool gemv_tma_batched(const GemvArgs& a, int pro, int epi, bool pdl) {
  const int K = a.K;
  if (epi > EPI_SWIGLU || ((uintptr_t)a.xq & 3)) return false;
  TmaPlan p = {};
  p.chunks = (K + 4095) / 4096;
  while (K % (p.chunks * 128)) p.chunks++;
  p.ks = K / p.chunks;
  p.stage_bytes = (TRP * (p.ks + 16) + TRP * (p.ks / 32) * 4 + 127) & ~127;
  const int most = 227 * 1024;
  const int per_red = (RED_FLOATS + 128) * 4;  // a buffer of the warps' parts and one of w1's results
  int act = (int)(((size_t)MB * (K + 16) + 2 * (size_t)MB * (K / 32) * 4 + 127) & ~127);
  const bool asmem = MMA_HEAD + 4 * per_red + act + 2 * p.stage_bytes <= most;
  if (!asmem) {
    if (pro != PRO_Q || (a.xq_stride & 3) || (a.xs_stride & 3)) return false;
    act = 0;
  }
  p.act_bytes = act;
  int S = (most - MMA_HEAD - 2 * per_red - act) / (p.stage_bytes + per_red);  // S stages and S + 2 buffers
  if (S > 8) S = 8;
  if (S < 2) return false;
  p.stages = S;
  p.nred = S + 2;
  const size_t smem = (size_t)MMA_HEAD + (size_t)p.nred * per_red + act + (size_t)S * p.stage_bytes;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  p.slot = (int)(next_ticket_slot(dev) % TICKET_SLOTS);
  p.tickets = p.chunks == 1;
#define CASE(P, E) \
  if (pro == P && epi == E) return asmem ? launch_mma<P, E, true>(a, p, smem, pdl) : launch_mma<P, E, false>(a, p, smem, pdl);
  CASE(PRO_Q, EPI_STORE) CASE(PRO_Q, EPI_ADD) CASE(PRO_Q, EPI_SWIGLU)
#undef CASE
#define CASE(P, E) \
  if (pro == P && epi == E) return asmem ? launch_mma<P, E, true>(a, p, smem, pdl) : false;
  CASE(PRO_RMS, EPI_STORE) CASE(PRO_RMS, EPI_ADD) CASE(PRO_RMS, EPI_SWIGLU)
  CASE(PRO_QUANT, EPI_STORE) CASE(PRO_QUANT, EPI_ADD) CASE(PRO_QUANT, EPI_SWIGLU)
#undef CASE
  return false;
}

// The ternary form at one token: whole rows a stage (K / 4 code bytes and K / 128 float16 scales a row, the scales'
// rows whole 16-byte pieces), up to 16 stages.
bool gemv_tma_t2(const GemvArgs& a, int pro, int epi, bool pdl) {
  const int K = a.K, units = K / 128;
  if (K % 128 || K > 65536 || (units * 2) % 16 || epi > EPI_SWIGLU || ((uintptr_t)a.wq & 15) || ((uintptr_t)a.ws & 15))
    return false;
  if (pro == PRO_Q && (((uintptr_t)a.xq & 15) || ((uintptr_t)a.xs & 15))) return false;
  TmaPlan p = {};
  p.chunks = 1;
  p.ks = K;
  const int row_bytes = K / 4 + units * 2;
  p.rw = 45056 / (NC * row_bytes);  // a stage of about 44 KB: up to 4 rows a warp (the shorter rows)
  if (p.rw > 4) p.rw = 4;
  if (p.rw < 1) p.rw = 1;
  p.stage_bytes = (NC * p.rw * row_bytes + 127) & ~127;
  p.act_bytes = (int)((2 * (size_t)K + 2 * (size_t)(K / 32) * 4 + 127) & ~127);
  const int head = (20 * T2_STAGES + 4 + 127) & ~127;
  int S = (227 * 1024 - head - p.act_bytes) / p.stage_bytes;
  if (S > T2_STAGES) S = T2_STAGES;
  if (S < 2) return false;
  p.stages = S;
  const size_t smem = (size_t)head + p.act_bytes + (size_t)S * p.stage_bytes;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  p.slot = (int)(next_ticket_slot(dev) % TICKET_SLOTS);
  p.tickets = 1;
#define CASE(P, E) \
  if (pro == P && epi == E) return launch_t2<P, E>(a, p, smem, pdl);
  CASE(PRO_Q, EPI_STORE) CASE(PRO_Q, EPI_ADD) CASE(PRO_Q, EPI_SWIGLU)
  CASE(PRO_RMS, EPI_STORE) CASE(PRO_RMS, EPI_ADD) CASE(PRO_RMS, EPI_SWIGLU)
  CASE(PRO_QUANT, EPI_STORE) CASE(PRO_QUANT, EPI_ADD) CASE(PRO_QUANT, EPI_SWIGLU)
#undef CASE
  return false;
}

// The int6 form at one token: whole rows a stage (K / 32 x 24 code bytes and K / 32 float32 scales a row), up to 16
// stages.
bool gemv_tma_q6(const GemvArgs& a, int pro, int epi, bool pdl) {
  const int K = a.K, ng = K / 32;
  if (K % 128 || K > 65536 || epi > EPI_SWIGLU || ((uintptr_t)a.wq & 15) || ((uintptr_t)a.ws & 15)) return false;
  // below ~32 M weights the register kernel is as fast or faster (measured, one launch after another: 4096 x 4096
  // 6.0-6.4 us against 8.3, 1024 x 1024 the same; from 12,288 x 4096 up the bulk-copy form is 10-12 % faster)
  if ((long long)(a.r1 - a.r0) * K < (1ll << 25)) return false;
  if (pro == PRO_Q && (((uintptr_t)a.xq & 15) || ((uintptr_t)a.xs & 15))) return false;
  TmaPlan p = {};
  p.chunks = 1;
  p.ks = K;
  const int row_bytes = ng * 24 + ng * 4;
  p.rw = 90112 / (NC * row_bytes);  // a stage of about 88 KB, up to 4 rows a warp (measured: 4.0 TB/s at 16,384 x
  if (p.rw > 4) p.rw = 4;            // 4096 against 3.1 with 28 KB stages of a row a warp)
  if (p.rw < 1) p.rw = 1;
  p.stage_bytes = (NC * p.rw * row_bytes + 127) & ~127;
  p.act_bytes = (int)(((size_t)K + (size_t)ng * 4 + 127) & ~127);
  const int head = (20 * T2_STAGES + 4 + 127) & ~127;
  int S = (227 * 1024 - head - p.act_bytes) / p.stage_bytes;
  if (S > T2_STAGES) S = T2_STAGES;
  if (S < 2) return false;
  p.stages = S;
  const size_t smem = (size_t)head + p.act_bytes + (size_t)S * p.stage_bytes;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  p.slot = (int)(next_ticket_slot(dev) % TICKET_SLOTS);
  p.tickets = 1;
#define CASE(P, E) \
  if (pro == P && epi == E) return launch_q6<P, E>(a, p, smem, pdl);
  CASE(PRO_Q, EPI_STORE) CASE(PRO_Q, EPI_ADD) CASE(PRO_Q, EPI_SWIGLU)
  CASE(PRO_RMS, EPI_STORE) CASE(PRO_RMS, EPI_ADD) CASE(PRO_RMS, EPI_SWIGLU)
  CASE(PRO_QUANT, EPI_STORE) CASE(PRO_QUANT, EPI_ADD) CASE(PRO_QUANT, EPI_SWIGLU)
#undef CASE
  return false;
}

// The bulk-copy product for int8 weights at 1 to 16 tokens and int6 and ternary weights at one; false where it does not
// apply
// (the caller then takes the register-streaming kernel).
bool gemv_tma(const GemvArgs& a, int fmt, int pro, int epi, bool pdl, const Xchg* xg) {
  const bool tp = pro == PRO_RMS_SUM || epi == EPI_SEND;
  if (tp != (xg != nullptr)) return false;
  if (fmt == F_T2 && !tp && a.count == 1 && g_gemv_mode != 1) return gemv_tma_t2(a, pro, epi, pdl);
  if (fmt == F_Q6 && !tp && a.count == 1 && g_gemv_mode != 1) return gemv_tma_q6(a, pro, epi, pdl);
  if (g_gemv_mode == 1 || fmt != F_Q8 || a.count < 1 || (tp && a.count != 1)) return false;
  const int K = a.K;
  if (K % 128 || ((uintptr_t)a.wq & 15) || ((uintptr_t)a.ws & 15)) return false;
  if (a.count > 2) {  // the batched form, in passes of 16 tokens (each pass streams the rows again)
    for (int t0 = 0; t0 < a.count; t0 += MB) {
      GemvArgs b = a;
      b.count = a.count - t0 < MB ? a.count - t0 : MB;
      b.out = a.out + t0 * a.out_stride;
      b.xq = a.xq + t0 * a.xq_stride;
      b.xs = reinterpret_cast<const float*>(reinterpret_cast<const uint8_t*>(a.xs) + t0 * a.xs_stride);
      b.x = a.x + t0 * a.x_stride;
      if (!gemv_tma_batched(b, pro, epi, pdl)) {
        if (t0 == 0) return false;  // the register kernel instead
        pllm_fail(PLLM_ECUDA, "gemv_tma: a pass of the batched form did not launch");
        return true;
      }
    }
    return true;
  }
  TmaPlan p = {};
  p.chunks = (K + 8191) / 8192;
  while (K % (p.chunks * 128)) p.chunks++;
  p.ks = K / p.chunks;
  const int MT = a.count;
  p.stage_bytes = (TRP * p.ks + TRP * (p.ks / 32) * 4 + 127) & ~127;
  p.act_bytes = (int)((MT * (size_t)K + MT * (size_t)(K / 32) * 4 + 127) & ~127);
  const int head = (20 * 8 + 4 + 127) & ~127;  // the barriers, headers and started flag of up to 8 stages
  int S = (g_tma_budget - p.act_bytes - head) / p.stage_bytes;
  if (S > 8) S = 8;
  if (S < 2) return false;
  p.stages = S;
  const size_t smem = (size_t)head + p.act_bytes + (size_t)S * p.stage_bytes;
  if (smem > 227 * 1024) return false;
  Xchg x = {};
  if (xg) {
    x = *xg;
    x.status = status_word();
    if (!x.status) return true;  // failed (recorded), not for want of a fit
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
  p.slot = (int)(next_ticket_slot(dev) % TICKET_SLOTS);
  // rows cut into chunks make tiles of two stages or more, the last of which ends the launch late: fixed shares there
  p.tickets = p.chunks == 1;
#define CASE(M, P, E) \
  if (MT == M && pro == P && epi == E) return launch<M, P, E>(a, p, smem, pdl, x);
  CASE(1, PRO_Q, EPI_STORE) CASE(1, PRO_Q, EPI_ADD) CASE(1, PRO_Q, EPI_SWIGLU)
  CASE(1, PRO_RMS, EPI_STORE) CASE(1, PRO_RMS, EPI_ADD) CASE(1, PRO_RMS, EPI_SWIGLU)
  CASE(1, PRO_QUANT, EPI_STORE) CASE(1, PRO_QUANT, EPI_ADD) CASE(1, PRO_QUANT, EPI_SWIGLU)
  CASE(2, PRO_Q, EPI_STORE) CASE(2, PRO_RMS, EPI_STORE) CASE(2, PRO_QUANT, EPI_ADD) CASE(2, PRO_RMS, EPI_SWIGLU)
  CASE(1, PRO_RMS_SUM, EPI_STORE) CASE(1, PRO_RMS_SUM, EPI_SWIGLU) CASE(1, PRO_QUANT, EPI_SEND)
#undef CASE
  return false;
}

}  // namespace gemvk

// a bounded device-side wait gave up since the last call (PLLM_ETIMEOUT), or 0; reading it clears it
PLLM_API int32_t pllm_device_status() {
  int v = 0, zero = 0;
  cudaMemcpyFromSymbol(&v, g_pllm_status, sizeof v);
  if (v) {
    cudaMemcpyToSymbol(g_pllm_status, &zero, sizeof zero);
    // a product that gave up may not have put its ticket counter back to zero: every counter starts over
    static const unsigned zeros[TICKET_SLOTS] = {0};
    cudaMemcpyToSymbol(g_tickets, zeros, sizeof zeros);
  }
  return v;
}

// which decode-product kernel: 0 the bulk-copy pipeline where it applies (int8, 1 or 2 tokens), 1 the
// register-streaming kernel always. Returns the previous mode.
PLLM_API int32_t pllm_set_gemv_mode(int32_t mode) {
  const int old = gemvk::g_gemv_mode;
  if (mode == 0 || mode == 1) gemvk::g_gemv_mode = mode;
  return old;
}

// the bytes of shared memory the bulk-copy product's stage ring may take (default 180 KB); a smaller ring leaves
// room on each SM for the next kernel's CTA to start streaming early. Returns the previous value.
PLLM_API int32_t pllm_set_stage_budget(int32_t bytes) {
  const int old = gemvk::g_tma_budget;
  if (bytes >= 32 * 1024 && bytes <= 227 * 1024) gemvk::g_tma_budget = bytes;
  return old;
}
