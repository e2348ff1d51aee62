// exchange.cu: the tensor-parallel decode step's reductions over NVLink (no counterpart in the reference, whose engine
// splits a product's rows across the CPU threads of one memory: src/runtime/forward/threads.ts). One process a GPU;
// each rank holds its share of every matrix (q/k/v and w1/w3 by rows, wo and w2 by K, the classifier by vocab rows),
// and a layer has two reductions, after wo and after w2: dim floats from every rank, summed.
//
// A rank's exchange region (one cudaMalloc, mapped into every other rank by CUDA IPC):
//   slots [2 parities][world][dim] x 8 bytes: rank s's partial of the reduction at [parity][s], each value with the
//         reduction's mark in the upper 4 bytes (one 8-byte store: a reader sees the pair whole or the old one)
//   step  uint32: this rank's steps (pllm_tp_step, the first kernel of a step)
// The k-th reduction of a parity in a step has the mark (step - 1) layers + k + 1; a reader takes a slot once its mark
// is that (no fence, no counter: the same scheme as a low-latency all-reduce). The reductions of a step alternate
// parities (wo: 0, w2: 1), so a rank can only write a parity's slots again after every rank has read them: its next
// write there follows its own reduction of the other parity, which needs this rank's next partial, made after this
// rank's read. The sends and the sums are in the bulk-copy product's epilogue and prologue (gemv_tma.cu: EPI_SEND,
// PRO_RMS_SUM); waits are bounded (2 s, then PLLM_ETIMEOUT in the device status word).
#include <string.h>

#include "pllm_common.cuh"
#include "gemv_common.cuh"

using gemvk::Xchg;

namespace {

struct Tp {
  int world, rank, dim, layers;
  size_t step_off, bytes;
  uint8_t* local;
  uint8_t* peer[gemvk::TP_MAX];  // every rank's region as this process sees it (peer[rank] = local)
};

size_t recv_off(const Tp& t, int parity, int src) { return ((size_t)parity * t.world + src) * t.dim * 8; }

__global__ void tp_step_kernel(unsigned* step) { *step += 1u; }

Tp* tp_of(uint64_t h, const char* name) {
  Tp* t = reinterpret_cast<Tp*>((uintptr_t)h);
  if (!t) pllm_fail(PLLM_EINVAL, "%s: no exchange", name);
  return t;
}

}  // namespace

// A rank's exchange for world ranks of dim floats and layers layers (its region zeroed); 0 on failure.
PLLM_API uint64_t pllm_tp_open(int32_t world, int32_t rank, int32_t dim, int32_t layers) {
  PLLM_REQUIRE_RET(world >= 1 && world <= gemvk::TP_MAX && rank >= 0 && rank < world && dim > 0 && dim % 32 == 0 &&
                       layers > 0,
                   0, "pllm_tp_open: world %d rank %d dim %d layers %d", world, rank, dim, layers);
  Tp* t = new Tp();
  t->world = world;
  t->rank = rank;
  t->dim = dim;
  t->layers = layers;
  t->step_off = (recv_off(*t, 2, 0) + 255) & ~(size_t)255;
  t->bytes = t->step_off + 256;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, t->bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, t->bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    pllm_fail(PLLM_ECUDA, "pllm_tp_open: %s", cudaGetErrorString(e));
    if (p) cudaFree(p);
    delete t;
    return 0;
  }
  t->local = static_cast<uint8_t*>(p);
  t->peer[rank] = t->local;
  if (!gemvk::status_word()) {  // the products' waits report there; looked up here, outside any capture
    pllm_tp_close((uint64_t)(uintptr_t)t);
    return 0;
  }
  return (uint64_t)(uintptr_t)t;
}

// The region's IPC handle (64 bytes at out), for the other ranks' pllm_tp_connect; 0 or an error code.
PLLM_API int32_t pllm_tp_handle(uint64_t tp, void* out) {
  Tp* t = tp_of(tp, "pllm_tp_handle");
  if (!t || !out) return PLLM_EINVAL;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, t->local);
  if (e != cudaSuccess) {
    pllm_fail(PLLM_ECUDA, "pllm_tp_handle: %s", cudaGetErrorString(e));
    return PLLM_ECUDA;
  }
  memcpy(out, &h, sizeof h);
  return 0;
}

// Every rank's handle (world x 64 bytes, in rank order): the other ranks' regions mapped into this process.
PLLM_API int32_t pllm_tp_connect(uint64_t tp, const void* handles) {
  Tp* t = tp_of(tp, "pllm_tp_connect");
  if (!t || !handles) return PLLM_EINVAL;
  for (int r = 0; r < t->world; r++) {
    if (r == t->rank || t->peer[r]) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)r * sizeof h, sizeof h);
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      pllm_fail(PLLM_ECUDA, "pllm_tp_connect: rank %d: %s", r, cudaGetErrorString(e));
      return PLLM_ECUDA;
    }
    t->peer[r] = static_cast<uint8_t*>(p);
  }
  return 0;
}

// Unmaps the other ranks' regions and frees this one (after every rank is done with the exchange).
PLLM_API void pllm_tp_close(uint64_t tp) {
  Tp* t = reinterpret_cast<Tp*>((uintptr_t)tp);
  if (!t) return;
  for (int r = 0; r < t->world; r++)
    if (r != t->rank && t->peer[r]) cudaIpcCloseMemHandle(t->peer[r]);
  cudaFree(t->local);
  delete t;
}

// The first kernel of a tensor-parallel step: the step counter the reductions' marks are made from.
PLLM_API void pllm_tp_step(uint64_t tp) {
  Tp* t = tp_of(tp, "pllm_tp_step");
  if (!t) return;
  tp_step_kernel<<<1, 1, 0, pllm_stream()>>>(reinterpret_cast<unsigned*>(t->local + t->step_off));
  PLLM_LAUNCHED("pllm_tp_step");
}

// The decode product of a tensor-parallel step (int8, one token, rows 0..rows): pllm_gemv's pro 1 / 2 and epi 0 / 2,
// plus pro 3 (x + every rank's partial of reduction use, then RMSNorm and quantize_x; the sum to x_out) and epi 3
// (the rows sent to every rank as its partial of reduction use). use: the reduction's index in the step (wo of layer
// l: 2 l, w2 of layer l: 2 l + 1).
PLLM_API void pllm_gemv_tp(uint64_t out, uint64_t x, uint64_t x_out, uint64_t norm, float eps, int32_t bias,
                           uint64_t wq, uint64_t ws, int32_t n, int32_t rows, int32_t pro, int32_t epi, int64_t pair,
                           int32_t pdl, uint64_t tp, int32_t use) {
  using namespace gemvk;
  PLLM_REQUIRE(pro >= PRO_RMS && pro <= PRO_RMS_SUM && (epi == EPI_STORE || epi == EPI_SWIGLU || epi == EPI_SEND),
               "pllm_gemv_tp: pro %d epi %d", pro, epi);
  PLLM_REQUIRE(n > 0 && n % 128 == 0 && rows > 0 && (bias == 0 || bias == 64), "pllm_gemv_tp: n %d rows %d bias %d",
               n, rows, bias);
  GemvArgs a = {};
  a.out = dptr<float>(out);
  a.x = dptr<const float>(x);
  a.norm = dptr<const float>(norm);
  a.eps = eps;
  a.bias = bias;
  a.wq = dptr<const uint8_t>(wq);
  a.ws = dptr<const void>(ws);
  a.K = n;
  a.r0 = 0;
  a.r1 = rows;
  a.count = 1;
  a.pair = pair;
  const bool exchanged = pro == PRO_RMS_SUM || epi == EPI_SEND;
  Xchg xg = {};
  if (exchanged) {
    Tp* t = tp_of(tp, "pllm_gemv_tp");
    if (!t) return;
    PLLM_REQUIRE(use >= 0 && use < 2 * t->layers, "pllm_gemv_tp: reduction %d of %d", use, 2 * t->layers);
    const int parity = use & 1;
    for (int r = 0; r < t->world; r++)
      PLLM_REQUIRE(t->peer[r], "pllm_gemv_tp: rank %d is not connected", r);
    if (epi == EPI_SEND) {
      PLLM_REQUIRE(rows == t->dim, "pllm_gemv_tp: a sent product has dim (%d) rows, not %d", t->dim, rows);
      for (int r = 0; r < t->world; r++)
        xg.dst[r] = reinterpret_cast<unsigned long long*>(t->peer[r] + recv_off(*t, parity, t->rank));
    }
    if (pro == PRO_RMS_SUM) {
      PLLM_REQUIRE(n == t->dim && x_out && x_out != x,
                   "pllm_gemv_tp: a summed input is dim (%d) floats, not %d, into another buffer", t->dim, n);
      xg.src = reinterpret_cast<const unsigned long long*>(t->local + recv_off(*t, parity, 0));
      xg.x_out = dptr<float>(x_out);
    }
    xg.step = reinterpret_cast<const unsigned*>(t->local + t->step_off);
    xg.world = t->world;
    xg.per_step = (unsigned)t->layers;
    xg.k = (unsigned)(use >> 1);
  }
  if (!gemv_tma(a, F_Q8, pro, epi, pdl != 0, exchanged ? &xg : nullptr))
    pllm_fail(PLLM_EINVAL, "pllm_gemv_tp: the bulk-copy product does not take this call (pro %d epi %d n %d)", pro,
              epi, n);
}
