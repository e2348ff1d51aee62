/*
 * pllm.h -- the C ABI of libpllm.so: takano32/pyodide-llm's kernel registry on a B200 (sm_100a).
 *
 * The registry functions keep the reference's names, argument order and argument meaning exactly (the exports of
 * kernels/kernel.ts:23-43 and kernels/kernel_relaxed.ts:14-16, typed by src/runtime/jobs.ts:82-142 `Arguments`, with
 * the address positions of src/runtime/jobs.ts:56-74 `ADDRESSES`). An address there (a WASM `usize`) is a
 * `uint64_t` device pointer here; `i32` and `f32` stay `int32_t` and `float`. So a bun:ffi / ctypes binding of the
 * reference's table binds this library unchanged: FFIType.u64 for an address, i32 and f32 for the rest.
 *
 * Differences from the reference's contract, all at the boundary:
 *  - Memory: every address is device memory of the current device (pllm_alloc or any CUDA allocation). The
 *    kernels allocate nothing in a call (as kernels/README.md:365-370 requires of the reference's). The library
 *    keeps this state of its own, each per device: the status word of to_f16 / finite_f16 (one int32, made on the
 *    first call), the scratch of argmax and sample (a few words), the bounded waits' status word and the bulk-copy
 *    product's 1,024 tile-ticket counters (pllm_device_status), and the 4 MiB partials array of
 *    pllm_attention_f16_noalloc.
 *  - Threads: as the reference's threads.ts:90-133 shares a kernel's rows among threads, many host threads may call
 *    the kernels at once (on disjoint outputs, each on its own stream: the current stream is a thread's own). The
 *    calls that wait for a result in the library's scratch (argmax, sample, to_f16, finite_f16) take turns; each
 *    bulk-copy product launch takes its own ticket counter.
 *  - Ordering: a call enqueues its kernel on the calling thread's current stream (pllm_set_stream; default: the
 *    legacy stream 0) and returns; calls on one stream run in order. Only to_f16, finite_f16, argmax and sample
 *    (which return a number) wait for the stream.
 *  - Errors: the reference does not check its arguments (built --noAssert, kernels/build.py:13). Here a call whose
 *    arguments the reference's kernel could not take (n not whole groups, r0 > r1, a null or misaligned address)
 *    launches nothing and sets the sticky error that pllm_last_error returns; a failed launch sets it too.
 *  - Alignment: int8 and ternary weights 32-byte aligned, binary 16, int6 8; quantized activations, their scales
 *    and a tile's frame 16 bytes (pllm_alloc returns 256-byte aligned memory).
 *  - Relaxed products (matmul_q8r, matmul_q6r, matmul_q8r_tile): the corrections wc are accepted and not read: the
 *    activations' bias of 64 is taken off as they are loaded, which gives the same exact integer dot(w, q - 64) that
 *    wc (int8_sums / six_sums of the same weights) gives the reference.
 *  - Numbers: every group's int32 sum is the reference's to the bit (pllm_group_sums returns them). Float32 outputs
 *    of the products and attention agree with the reference's within float32 rounding of a different summation order
 *    (and of CUDA's expf against the reference's table-free exp); quantize_x, interleave, int8_sums, six_sums,
 *    to_f16, from_f16, finite_f16, delta_rule are the reference's to the bit.
 */
#ifndef PLLM_H
#define PLLM_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ===== the registry: activations (kernels/kernel/quantize.ts, kernels/kernel/matmul.ts) ===== */
/* replaces quantize_x, kernels/kernel/quantize.ts:124 (jobs.ts:113): per group of 32, scale = max|x| / qmax,
 * q = sat8(rne(x / scale) + bias); bias 0 (qmax 127, signed) or 64 (qmax 63, stored 1..127) */
void quantize_x(uint64_t xq, uint64_t xs, uint64_t x, int32_t n, int32_t bias);
/* replaces interleave, kernels/kernel/matmul.ts:129 (jobs.ts:105): the ternary / binary products' layout, in place;
 * after the n / 32 scales at xs, n / 32 int32 minus-sums */
void interleave(uint64_t xq, uint64_t xs, int32_t n);
/* replaces int8_sums, kernels/kernel/matmul.ts:50 (jobs.ts:103) */
void int8_sums(uint64_t out, uint64_t w, int32_t groups);
/* replaces six_sums, kernels/kernel/matmul.ts:38 (jobs.ts:102) */
void six_sums(uint64_t out, uint64_t w, int32_t groups);

/* ===== the registry: products ===== */
/* replaces matmul_q8, kernels/kernel/matmul.ts:77 (jobs.ts:104) */
void matmul_q8(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n, int32_t r0, int32_t r1);
/* replaces matmul_q8r, kernels/relaxed/int8.ts:17 (jobs.ts:124) */
void matmul_q8r(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, uint64_t wc, int32_t n, int32_t r0,
                int32_t r1);
/* replaces matmul_q8r_tile, kernels/relaxed/int8.ts:147 (jobs.ts:125): count tokens, xq / xs frame bytes apart,
 * outputs os bytes apart */
void matmul_q8r_tile(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, uint64_t wc, int32_t n,
                     int32_t r0, int32_t r1, int32_t count, int32_t os, int32_t frame);
/* replaces matmul_q6, kernels/kernel/matmul.ts:227 (jobs.ts:107) */
void matmul_q6(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n, int32_t r0, int32_t r1);
/* replaces matmul_q6r, kernels/relaxed/six.ts:16 (jobs.ts:126) */
void matmul_q6r(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, uint64_t wc, int32_t n, int32_t r0,
                int32_t r1);
/* replaces matmul_t2, kernels/kernel/matmul.ts:218 (jobs.ts:106); three must be 3 */
void matmul_t2(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n, int32_t r0, int32_t r1,
               int32_t three);
/* replaces matmul_t2r, kernels/relaxed/signs.ts:117 (jobs.ts:127) */
void matmul_t2r(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n, int32_t r0, int32_t r1,
                int32_t three);
/* replaces matmul_t2r_tile, kernels/relaxed/signs.ts:120 (jobs.ts:128) */
void matmul_t2r_tile(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n, int32_t r0,
                     int32_t r1, int32_t count, int32_t os, int32_t frame, int32_t three);
/* replaces matmul_b1, kernels/kernel/matmul.ts:222 (jobs.ts:138); two must be 2 */
void matmul_b1(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n, int32_t r0, int32_t r1,
               int32_t two);
/* replaces matmul_b1r, kernels/relaxed/signs.ts:123 (jobs.ts:139) */
void matmul_b1r(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n, int32_t r0, int32_t r1,
                int32_t two);
/* replaces matmul_b1r_tile, kernels/relaxed/signs.ts:126 (jobs.ts:140) */
void matmul_b1r_tile(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n, int32_t r0,
                     int32_t r1, int32_t count, int32_t os, int32_t frame, int32_t two);
/* replaces matmul_f32, kernels/kernel/matmul.ts:13 (jobs.ts:101) */
void matmul_f32(uint64_t xout, uint64_t x, uint64_t w, int32_t n, int32_t r0, int32_t r1);

/* ===== the registry: attention and float16 (kernels/kernel/attention.ts, kernels/kernel/halves.ts) ===== */
/* replaces rope, kernels/kernel/attention.ts:7 (jobs.ts:93) */
void rope(uint64_t v, uint64_t fcr, uint64_t fci, int32_t nh, int32_t hs, int32_t rot);
/* replaces attention, kernels/kernel/attention.ts:28 (jobs.ts:94); att: nh (pos + 1) floats of scratch, whose
 * contents after the call are not the probabilities */
void attention(uint64_t out, uint64_t q, uint64_t kc, uint64_t vc, uint64_t att, int32_t pos, int32_t nh, int32_t nkv,
               int32_t hs, int32_t h0, int32_t h1);
/* replaces attention_f16, kernels/kernel/attention.ts:34 (jobs.ts:95) */
void attention_f16(uint64_t out, uint64_t q, uint64_t kc, uint64_t vc, uint64_t att, int32_t pos, int32_t nh,
                   int32_t nkv, int32_t hs, int32_t h0, int32_t h1);
/* replaces attention_capped, kernels/kernel/attention.ts:40 (jobs.ts:96) */
void attention_capped(uint64_t out, uint64_t q, uint64_t kc, uint64_t vc, uint64_t att, int32_t pos, int32_t nh,
                      int32_t nkv, int32_t hs, int32_t h0, int32_t h1, float cap);
/* replaces attention_f16_capped, kernels/kernel/attention.ts:43 (jobs.ts:97) */
void attention_f16_capped(uint64_t out, uint64_t q, uint64_t kc, uint64_t vc, uint64_t att, int32_t pos, int32_t nh,
                          int32_t nkv, int32_t hs, int32_t h0, int32_t h1, float cap);
/* replaces to_f16, kernels/kernel/halves.ts:35 (jobs.ts:98): returns how many inputs were not finite (waits) */
int32_t to_f16(uint64_t out, uint64_t x, int32_t n);
/* replaces from_f16, kernels/kernel/halves.ts:72 (jobs.ts:99) */
void from_f16(uint64_t out, uint64_t x, int32_t n);
/* replaces finite_f16, kernels/kernel/halves.ts:82 (jobs.ts:100): 1 if all finite, else 0 (waits) */
int32_t finite_f16(uint64_t x, int32_t n);

/* ===== the registry: from the logits to a token (kernels/kernel/sample.ts) */
/* replaces argmax, sample.ts:6-10 (jobs.ts:116): the first index of the largest of n floats (a NaN never wins; one at
 * index 0 is the answer, as the reference's walk); waits (the library's own small scratch: concurrent host calls take
 * turns) */
int32_t argmax(uint64_t x, int32_t n);
/* replaces penalize, sample.ts:16-30 (jobs.ts:117): each distinct token of tokens[0..count) once: a positive logit
 * divided by penalty, another multiplied by it, then presence (if > 0) taken off */
void penalize(uint64_t logits, uint64_t tokens, int32_t count, float penalty, float presence);
/* replaces sample, sample.ts:248-337 (kernels.py's restype i32): the token drawn from softmax(logits / temperature) by
 * random in [0, 1), of the topk most probable (0: all), then of their nucleus (0 < topp < 1), then without those below
 * minp times the most probable (0: none); -1 where the largest logit is not a finite number. probs, index: device
 * scratch of n floats and n int32. Waits (the library's own scratch: concurrent host calls take turns) */
int32_t sample(uint64_t logits, int32_t n, float temperature, float topp, double random, uint64_t probs,
               uint64_t index, int32_t topk, float minp);

/* ===== the registry: llama.cpp's blocks of 256 weights (kernels/blocks.ts:11-13, kernels/blocks_relaxed.ts:5-6;
 * kernels/blocks/types.ts): Q2_K 10, Q4_K 12, IQ2_XXS 16, IQ2_XS 17, IQ3_XXS 18, IQ1_S 19, IQ3_S 21, IQ2_S 22,
 * IQ4_XS 23, IQ1_M 29 (type: the type's number in a GGUF); rows of whole blocks (n a multiple of 256); tab: sb_tables'
 * area. Every group's integers are the reference's; the float32 row within rounding of its order. */
/* replaces sb_tables, blocks/types.ts:294: the tables (34,992 bytes at area) from the checkpoint's codebooks row;
 * returns the bytes */
int32_t sb_tables(uint64_t area, uint64_t codebooks);
/* replaces sums_x, blocks/token.ts:160: after the n / 32 scales at xs, the int16 sums of each 16 activations of xq,
 * then of each 8 */
void sums_x(uint64_t xs, uint64_t xq, int32_t n);
/* replaces matmul_sb, blocks/token.ts:133, and matmul_sbr, :138 (the same numbers): one token, rows r0..r1 */
void matmul_sb(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t w, uint64_t tab, int32_t n, int32_t r0, int32_t r1,
               int32_t type);
void matmul_sbr(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t w, uint64_t tab, int32_t n, int32_t r0, int32_t r1,
                int32_t type);
/* replaces matmul_sbr_tile, blocks/tile.ts:149, and matmul_sbw_tile (the same numbers; its scratch is not needed):
 * count tokens, activations and xs frame bytes apart, outputs os bytes apart */
void matmul_sbr_tile(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t w, uint64_t tab, int32_t n, int32_t r0,
                     int32_t r1, int32_t count, int32_t os, int32_t frame, int32_t type);
void matmul_sbw_tile(uint64_t xout, uint64_t xq, uint64_t xs, uint64_t w, uint64_t tab, int32_t n, int32_t r0,
                     int32_t r1, int32_t count, int32_t os, int32_t frame, int32_t type, uint64_t scratch);
/* replaces signed_dots, blocks/tile.ts: out[l] = sum over i < 4 of a[4 l + i] b[4 l + i], signed bytes by signed
 * bytes (exact here for every a and b) */
void signed_dots(uint64_t out, uint64_t a, uint64_t b);
/* replaces sb_row, blocks/row.ts:60: a row of n weights as float32 (each as the reference's reader makes it) */
void sb_row(uint64_t out, uint64_t w, uint64_t tab, int32_t n, int32_t type);

/* ===== the registry: vector glue and stateful layers (kernels/kernel/activations.ts, kernels/kernel/stateful.ts) */
/* replaces rmsnorm, kernels/kernel/activations.ts:8 (jobs.ts:83) */
void rmsnorm(uint64_t out, uint64_t x, uint64_t w, int32_t n, float eps);
/* replaces swiglu, kernels/kernel/activations.ts:77 (jobs.ts:86) */
void swiglu(uint64_t out, uint64_t h1, uint64_t h3, int32_t n);
/* replaces add_inplace, kernels/kernel/activations.ts:156 (jobs.ts:90) */
void add_inplace(uint64_t x, uint64_t y, int32_t n);
/* replaces gate, kernels/kernel/stateful.ts:12 (jobs.ts:120) */
void gate(uint64_t out, uint64_t x, uint64_t g, int32_t n);
/* replaces convolve, kernels/kernel/stateful.ts:49 (jobs.ts:121) */
void convolve(uint64_t out, uint64_t taps, uint64_t rows, int32_t n, int32_t count);
/* replaces short_conv, kernels/kernel/stateful.ts:70 (jobs.ts:122) */
void short_conv(uint64_t out, uint64_t taps, uint64_t rows, uint64_t b, int32_t n, int32_t count);
/* replaces delta_rule, kernels/kernel/stateful.ts:96 (jobs.ts:123) */
void delta_rule(uint64_t out, uint64_t state, uint64_t next, uint64_t c, uint64_t work, int32_t kh, int32_t kd,
                int32_t vd, int32_t vh, int32_t h0, int32_t h1);

/* ===== device, memory, streams, graphs, errors (no counterpart in the reference: its kernels worked in one WASM
 * memory the engine owned, src/runtime/forward/engine.ts:147-163) ===== */
int32_t pllm_init(int32_t device);                     /* select the device (sm_100 only) and make its context */
int32_t pllm_last_error(char *buf, int32_t len);       /* the sticky error code (0: none) and its message */
void pllm_clear_error(void);
int32_t pllm_num_sms_of_device(void);
uint64_t pllm_alloc(uint64_t bytes);                   /* device memory, 256-byte aligned; 0 on failure */
void pllm_free(uint64_t p);
uint64_t pllm_alloc_host(uint64_t bytes);              /* pinned host memory */
void pllm_free_host(uint64_t p);
void pllm_h2d(uint64_t dst, const void *src, uint64_t bytes);   /* on the current stream */
void pllm_d2h(void *dst, uint64_t src, uint64_t bytes);
void pllm_d2d(uint64_t dst, uint64_t src, uint64_t bytes);
void pllm_memset(uint64_t dst, int32_t value, uint64_t bytes);
uint64_t pllm_stream_create(void);
void pllm_stream_destroy(uint64_t s);
void pllm_set_stream(uint64_t s);                      /* the calling thread's; 0: the legacy default stream */
uint64_t pllm_get_stream(void);
int32_t pllm_sync(void);                               /* wait for the current stream */
int32_t pllm_device_sync(void);
int32_t pllm_graph_begin(void);                        /* record the calls that follow on the current stream */
uint64_t pllm_graph_end(void);                         /* an executable graph of them (0 on failure) */
int32_t pllm_graph_launch(uint64_t exec);
void pllm_graph_destroy(uint64_t exec);
uint64_t pllm_event_create(void);
void pllm_event_record(uint64_t e);
float pllm_event_ms(uint64_t a, uint64_t b);           /* waits for b */
void pllm_event_destroy(uint64_t e);
const char *pllm_version(void);

/* ===== additions for a device-memory engine (no counterpart in the reference: its engine touched the memory from
 * JavaScript between kernel calls, src/runtime/forward/tensors.ts:154-160, forward/cache.ts:117-141) ===== */
/* the exact int32 sums of every (row, group of 32) of rows [r0, r1) against one token: the accumulators every
 * product scales. fmt 0 int8, 1 int6, 2 ternary, 3 binary; bias 0 or 64 (int8 / int6) */
void pllm_group_sums(uint64_t out, uint64_t xq, uint64_t xs, uint64_t wq, int32_t fmt, int32_t n, int32_t r0, int32_t r1,
                     int32_t bias);
/* count tokens quantized (x a frame of n floats apart, xq n bytes, xs n / 32 floats) */
void pllm_quantize_tokens(uint64_t xq, uint64_t xs, uint64_t x, int32_t n, int32_t bias, int32_t count);
/* to_f16 without waiting: the count of non-finite inputs is added to the device int32 at bad */
void pllm_to_f16_async(uint64_t out, uint64_t x, int32_t n, uint64_t bad);
/* rmsnorm of rows rows of n floats, stride floats apart, one weight (Qwen3's per-head q / k norms) */
void pllm_rmsnorm_rows(uint64_t out, uint64_t x, uint64_t w, int32_t n, float eps, int32_t rows, int64_t stride);
/* the reference engine's memory touches between kernel calls (JavaScript over its WASM memory, double precision then
 * stored as float32), as device kernels: */
/* an LFM2 convolution layer's step between its products (convolution.ts:51-60), a batch of sequences: per sequence z
 * (its rows at rows + z rows_stride, its [B | C | z] at mixed + z mixed_stride, its output at out + z out_stride,
 * floats) the rows move up one (at position pos_dev[z] == 0 from zeros, as clear() leaves them; pos_dev 0: never),
 * the newest row is B z, and out = C sum_j taps[j] rows[j]: shift_rows then short_conv, to the bit; count <= 8 */
void pllm_conv_step(uint64_t out, int64_t out_stride, uint64_t taps, uint64_t rows, int64_t rows_stride,
                    uint64_t mixed, int64_t mixed_stride, int32_t n, int32_t count, uint64_t pos_dev, int32_t batch);
/* linear.ts:160-161, convolution.ts:57: rows 1..count-1 of n floats move up one row (copyWithin); the last stays */
void pllm_shift_rows(uint64_t rows, int32_t n, int32_t count);
/* linear.ts:151-158: per value head h, work[h] = 1 / (1 + exp(-work[h])) (beta) and work[vh + h] = exp(decays[h]
 * softplus(work[vh + h] + dt_bias[h])) (decay), softplus(s) = s past 20, else log1p(exp(s)) */
void pllm_delta_gates(uint64_t work, uint64_t decays, uint64_t dt_bias, int32_t vh);
/* engine.ts:452-455: count rows of n floats (stride floats apart) times the float at scale (a layer's layerScale) */
void pllm_scale_rows(uint64_t x, int32_t n, int32_t count, int64_t stride, uint64_t scale);
/* engine.ts:467-470: x = cap tanh(x / cap), the quotient, its tanh and the product each rounded to float32 */
void pllm_softcap(uint64_t x, int32_t n, float cap);
/* count tokens' int8 embedding rows (tokens: device int32[count], or 0 to take token), as tensors.ts:154-160 */
void pllm_embed_q8(uint64_t x, uint64_t emb, uint64_t scales, uint64_t tokens, int32_t token, int32_t dim, int32_t count,
                   int64_t stride);
/* the fused decode product: fmt as pllm_group_sums; pro 0 quantized input (xq / xs), 1 RMSNorm(x, norm) then
 * quantize_x, 2 quantize_x(x); epi 0 store, 1 add into out (the residual), 2 silu(row) * row + pair (the gated FFN);
 * count tokens (strides: out and x in floats, xq and xs in bytes); pdl 1: launched as a programmatic dependent */
void pllm_gemv(uint64_t out, int64_t out_stride, uint64_t xq, uint64_t xs, int64_t xq_stride, int64_t xs_stride,
               uint64_t x, int64_t x_stride, uint64_t norm, float eps, int32_t bias, uint64_t wq, uint64_t ws,
               int32_t fmt, int32_t n, int32_t r0, int32_t r1, int32_t count, int32_t pro, int32_t epi, int64_t pair,
               int32_t pdl);
/* argmax into device memory (out: one int32) without waiting: the forward driver's greedy step; scratch: 16 bytes of
 * device memory, zero before the first call (every call leaves it at zero); a scratch's calls must not overlap */
void pllm_argmax_dev(uint64_t out, uint64_t x, int32_t n, uint64_t scratch);
/* the tensor-parallel greedy step (no counterpart in the reference: one memory holds its vocabulary): a rank's slice of
 * n logits starting at token offset gives its largest as a 64-bit key (ordered float bits, complement of the global
 * token) at key; the integer max of the ranks' keys (an all-reduce) names argmax's token over the whole vocabulary,
 * and pllm_key_token_dev turns it into the token (one int32 at out); scratch as pllm_argmax_dev's */
void pllm_argmax_key_dev(uint64_t key, uint64_t x, int32_t n, int64_t offset, uint64_t scratch);
void pllm_key_token_dev(uint64_t out, uint64_t key);
/* sample into device memory (out: one int32) without waiting, the random number a double at random_dev (written
 * before the launch runs: a recorded step's) */
void pllm_sample_dev(uint64_t out, uint64_t logits, int32_t n, float temperature, float topp, uint64_t random_dev,
                     uint64_t probs, uint64_t index, int32_t topk, float minp);
/* q / k head norms (null weights: none), RoPE at the position, and k / v into the cache at it; the position is
 * read from device memory at pos_dev (or pos if pos_dev is 0), so one recorded graph serves every position */
void pllm_qk_rope_cache(uint64_t q, uint64_t k, uint64_t v, uint64_t q_norm, uint64_t k_norm, uint64_t cos_t,
                        uint64_t sin_t, uint64_t pos_dev, int32_t pos, uint64_t kc, uint64_t vc, int32_t nh,
                        int32_t nkv, int32_t hs, int32_t rot, float eps, int32_t half, uint64_t bad, int32_t pdl);
/* the forward driver's attention step in one launch: the q / k head norms (null weights: none), RoPE at the device
 * position, this position's key and value into the cache, and the attention over positions 0..pos; qkv: the q/k/v
 * product's output (nh, nkv, nkv heads of hs); scratch: pllm_attention_scratch_bytes, zero before its first use */
void pllm_attention_step(uint64_t out, uint64_t qkv, uint64_t kc, uint64_t vc, uint64_t scratch, uint64_t pos_dev,
                         int32_t capacity, int32_t nh, int32_t nkv, int32_t hs, int32_t half, float cap,
                         int32_t split_len, uint64_t q_norm, uint64_t k_norm, uint64_t cos_t, uint64_t sin_t, int32_t rot,
                         float eps, uint64_t bad, int32_t pdl);
/* the same step for a batch of sequences in one launch: sequence z's q/k/v at qkv + z qkv_stride floats, its output at
 * out + z out_stride floats, its float16 caches at kc / vc + z cache_stride bytes, its position pos_dev[z], its
 * scratch the z-th of batch regions of pllm_attention_scratch_bytes rounded up to 256 (zero before their first use) */
void pllm_attention_step_batch(uint64_t out, int64_t out_stride, uint64_t qkv, int64_t qkv_stride, uint64_t kc,
                               uint64_t vc, int64_t cache_stride, uint64_t scratch, uint64_t pos_dev, int32_t batch,
                               int32_t capacity, int32_t nh, int32_t nkv, int32_t hs, float cap, int32_t split_len,
                               uint64_t q_norm, uint64_t k_norm, uint64_t cos_t, uint64_t sin_t, int32_t rot,
                               float eps, uint64_t bad, int32_t pdl);
/* attention at the device position over a cache of capacity positions; scratch: pllm_attention_scratch_bytes */
uint64_t pllm_attention_scratch_bytes(int32_t nh, int32_t hs, int32_t capacity, int32_t split_len);
void pllm_attention_dev(uint64_t out, uint64_t q, uint64_t kc, uint64_t vc, uint64_t scratch, uint64_t pos_dev,
                        int32_t capacity, int32_t nh, int32_t nkv, int32_t hs, int32_t half, float cap,
                        int32_t split_len, int32_t pdl);

/* count tokens of delta_rule's recurrence in one launch (a prompt's block, no counterpart in the reference, whose
 * engine calls delta_rule a token at a time, forward/linear.ts:99-183): token t's inputs at c + t c_stride floats,
 * its gates / delta at work + t work_stride, its outputs at out + t out_stride; state read once, the state after the
 * last token written to next once; every token's numbers delta_rule's to the bit. vd % 16 == 0, 16-byte aligned
 * states */
void pllm_delta_rule_block(uint64_t out, int64_t out_stride, uint64_t state, uint64_t next, uint64_t c,
                           int64_t c_stride, uint64_t work, int64_t work_stride, int32_t count, int32_t kh, int32_t kd,
                           int32_t vd, int32_t vh, int32_t h0, int32_t h1);

/* a bounded device-side wait (an mbarrier of the bulk-copy product) gave up since the last call: PLLM_ETIMEOUT (3);
 * or the attention step read a position from device memory outside its cache (held at the cache's edge, so that
 * nothing is read or written outside it): PLLM_ERANGE (5); else 0. Reading it clears it (and, after a wait that gave
 * up, puts the products' tile counters back to zero) */
int32_t pllm_device_status(void);
/* which decode-product kernel: 0 the bulk-copy pipeline where it applies (int8 weights at 1 to 16 tokens; int6
 * weights at one token in products of 2^25 weights and more; ternary weights at one token), 1 the register-streaming
 * kernel always; returns the previous mode */
int32_t pllm_set_gemv_mode(int32_t mode);
/* the shared-memory bytes the bulk-copy product's ring of stages may take (32 KB..227 KB; default 180 KB) */
int32_t pllm_set_stage_budget(int32_t bytes);
/* how the forward driver's float16 attention (pllm_attention_dev, pllm_attention_step) combines its parts: 1 (the
 * default) one thread-block cluster a kv head over the whole cache, combined in distributed shared memory; 0 slices
 * of split_len positions whose partials the last slice combines through the scratch; returns the previous mode */
int32_t pllm_set_attention_mode(int32_t mode);

/* ---- prefill on the tensor cores (the reference's tile products, matmul_q8r_tile / q8rTile, relaxed/int8.ts:89-166,
 * at a tile of 128 tokens): tcgen05 kind::i8 one group of 32 at a time, each group's exact int32 scaled in float32 */
/* out (M x N, ldo floats a row) = the int8 product of xq (M x K signed int8), xs (M x K/32), wq (w_rows x K) with its
 * scales transposed in ws_t (K/32 x w_rows); epi 0 store, 1 add into out, 2 silu(w1 row) x (w3 row) with w1's rows
 * 0..N and w3's from pair; K % 128 == 0, N % 128 == 0 (epi 2: N % 64 == 0) */
void pllm_gemm_q8(uint64_t out, int64_t ldo, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws_t, int32_t M, int32_t N,
                  int32_t K, int64_t w_rows, int32_t epi, int64_t pair);
/* rows of n floats (x_stride apart): RMSNorm with norm (0: none) then quantize_x with bias, as signed int8 (the bias
 * taken off) and n / 32 scales a row */
void pllm_norm_quantize_rows(uint64_t xq, uint64_t xs, uint64_t x, int64_t x_stride, uint64_t norm, float eps,
                             int32_t n, int32_t rows, int32_t bias);
/* dst[g][r] = src[r][g] for rows x groups scales */
void pllm_transpose_scales(uint64_t dst, uint64_t src, int64_t rows, int32_t groups);
/* count tokens' q / k head norms (null weights: none), RoPE at positions p0.., their keys and values into the cache;
 * qkv rows stride floats apart (nh q heads, nkv k heads, nkv v heads) */
void pllm_qk_rope_cache_rows(uint64_t qkv, int64_t stride, uint64_t q_norm, uint64_t k_norm, uint64_t cos_t,
                             uint64_t sin_t, int32_t p0, int32_t count, uint64_t kc, uint64_t vc, int32_t nh,
                             int32_t nkv, int32_t hs, int32_t rot, float eps, int32_t half, uint64_t bad);
/* count tokens at positions p0.. attend causally over a float16 cache holding positions 0 .. p0 + count - 1 (q from
 * qkv rows qstride floats apart; out rows ostride floats apart); hs <= 128 */
void pllm_attention_prefill(uint64_t out, int64_t ostride, uint64_t qkv, int64_t qstride, uint64_t kc, uint64_t vc,
                            int32_t p0, int32_t count, int32_t nh, int32_t nkv, int32_t hs);

/* ---- tensor-parallel decode over NVLink (no counterpart in the reference, whose engine splits rows across the
 * CPU threads of one memory, src/runtime/forward/threads.ts): one process a GPU, a layer's two reductions (after wo
 * and after w2) by peer stores into every rank's exchange region (mapped by CUDA IPC) and bounded waits */
/* a rank's exchange of world ranks (<= 8), dim floats a reduction, layers layers; 0 on failure */
uint64_t pllm_tp_open(int32_t world, int32_t rank, int32_t dim, int32_t layers);
/* the exchange region's IPC handle (64 bytes at out) for the other ranks; 0 or an error code */
int32_t pllm_tp_handle(uint64_t tp, void* out);
/* every rank's handle (world x 64 bytes, rank order): maps the other ranks' regions; 0 or an error code */
int32_t pllm_tp_connect(uint64_t tp, const void* handles);
/* unmaps the other ranks' regions and frees this one (once every rank is done) */
void pllm_tp_close(uint64_t tp);
/* the first kernel of a step: counts the steps the reductions' marks are made from */
void pllm_tp_step(uint64_t tp);
/* a tensor-parallel step's int8 product of one token, rows 0..rows: pro 1 RMSNorm + quantize_x, 2 quantize_x, 3 x +
 * every rank's partial of reduction use (in rank order) written to x_out, then RMSNorm + quantize_x; epi 0 store, 2
 * the gated FFN's silu(row) * row + pair, 3 the rows sent to every rank as this rank's partial of reduction use (wo of
 * layer l: use 2 l; w2: 2 l + 1). A wait for the other ranks gives up after 2 s (pllm_device_status: 3). */
void pllm_gemv_tp(uint64_t out, uint64_t x, uint64_t x_out, uint64_t norm, float eps, int32_t bias, uint64_t wq,
                  uint64_t ws, int32_t n, int32_t rows, int32_t pro, int32_t epi, int64_t pair, int32_t pdl,
                  uint64_t tp, int32_t use);

/* ---- a decode step in the reference's own order of float32 operations (no counterpart in the reference's registry:
 * its kernels have one order each, which these restate on the device so that a forward's logits are the reference
 * kernels' to the bit; the default kernels above agree with them within rounding). Exponentials: the Cephes expf
 * that kernels/kernel/math.ts:28-58 follows. */
/* x (n floats; mode 2: h1 then h3, 2 n floats) as it is (mode 0), through rmsnorm with norm (mode 1,
 * activations.ts:8-20) or swiglu (mode 2, activations.ts:77-90), then quantize_x with bias into xq / xs (n <= 49152);
 * out (0: none) gets the float32 vector that was quantized */
void pllm_exact_prepare(uint64_t xq, uint64_t xs, uint64_t out, uint64_t x, uint64_t norm, int32_t n, float eps,
                        int32_t bias, int32_t mode);
/* rows 0..rows of an int8 product of one token in matmul_q8's order (relaxed 0, matmul.ts:77-104: xq signed) or
 * matmul_q8r's (relaxed 1, relaxed/int8.ts:17-50: xq the bias-64 bytes); add (0: none) makes out[r] = add[r] + row
 * (add may be out) */
void pllm_exact_product(uint64_t out, uint64_t add, uint64_t xq, uint64_t xs, uint64_t wq, uint64_t ws, int32_t n,
                        int32_t rows, int32_t relaxed);
/* qkv (nh q, nkv k, nkv v heads of hs floats): the q / k head norms (null weights: none), rope (attention.ts:7-20)
 * at the position (pos_dev: device int32, or pos where pos_dev is 0), the key and value into the cache (to_f16 where
 * half, counting non-finite values into the device int32 at bad) */
void pllm_exact_qk_rope_cache(uint64_t qkv, uint64_t q_norm, uint64_t k_norm, uint64_t cos_t, uint64_t sin_t,
                              uint64_t pos_dev, int32_t pos, uint64_t kc, uint64_t vc, int32_t nh, int32_t nkv,
                              int32_t hs, float eps, int32_t half, uint64_t bad);
/* attentionOf (attention.ts:87-211) of nh heads over positions 0..pos (pos_dev or pos) of a cache of capacity
 * positions; att: nh x capacity floats of scratch (the scaled scores afterwards); cap > 0: attention_capped's
 * scores; hs % 16 == 0, nh / nkv <= 8, the kv head's probabilities in shared memory (refused beyond it) */
void pllm_exact_attention(uint64_t out, uint64_t q, uint64_t kc, uint64_t vc, uint64_t att, uint64_t pos_dev,
                          int32_t pos, int32_t capacity, int32_t nh, int32_t nkv, int32_t hs, int32_t half, float cap);

/* attention_f16 for callers that cannot allocate device memory (no counterpart in the reference): the same
 * arguments without att; the slices' partials live in a 4 MiB device array of the library's own, held by every GPU
 * that loads the library until exit, shared by all calls (overlapping calls race), with nothing that must start at
 * zero. Refused with an error where nh x ceil((pos + 1) / 128) x (hs + 4) floats exceed 1,048,576. The first call on
 * a device looks up the array's address: make it before any stream capture. */
void pllm_attention_f16_noalloc(uint64_t out, uint64_t q, uint64_t kc, uint64_t vc, int32_t pos, int32_t nh,
                                int32_t nkv, int32_t hs, int32_t h0, int32_t h1);

/* ===== seeded synthetic weights made on the device, for benchmarks and tests of model-sized shapes (no counterpart
 * in the reference, whose tests make synthetic checkpoints in NumPy, tests/made_up.py:30) ===== */
/* n float32 values N(mean, std) of (seed, index) */
void pllm_synth_f32(uint64_t out, int64_t n, uint64_t seed, float mean, float std);
/* rows x cols int8 weights: N(0, std) quantized group by group as engine/packing.py:40-45 quantizes */
void pllm_synth_q8(uint64_t wq, uint64_t ws, int64_t rows, int32_t cols, uint64_t seed, float std);
/* the block rows x cols at (row0, col0) of the matrix pllm_synth_q8 makes with full_cols columns (the same bytes):
 * a tensor-parallel rank's share of a synthetic matrix */
void pllm_synth_q8_block(uint64_t wq, uint64_t ws, int64_t rows, int32_t cols, uint64_t seed, float std, int64_t row0,
                         int64_t col0, int64_t full_cols);
/* rows x cols ternary weights uniform on {-1, 0, +1} (packing.py:106-109's codes) and a float16 scale a row,
 * N(mean, std) rounded to float16, repeated for each group of 128 */
void pllm_synth_t2(uint64_t wq, uint64_t ws, int64_t rows, int32_t cols, uint64_t seed, float mean, float std);

#ifdef __cplusplus
}
#endif
#endif
