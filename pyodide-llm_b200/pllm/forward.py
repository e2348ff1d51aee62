"""A decoder's forward pass on the device: the B200 counterpart of src/runtime/forward/engine.ts's createForward
(run() :421-475; the attention layer forward/attention.ts:171-197; the gated FFN forward/ffn.ts:25-35) for the
Llama / Qwen3 families of int8 models (Qwen3: q_norm / k_norm, forward/attention.ts:140-143).

The engine's public calls are the reference's (engine.ts:549-702): forward(token, pos, need_logits) and
forward_many(tokens, pos). What differs is where the memory is: the weights, the cache and the activations stay in
device memory, and one decode step is recorded once as a CUDA graph of the library's kernels (the token and the
position are read by the kernels from device memory, so the same graph serves every position). A step is:

    embed (pllm_embed_q8: the int8 row times its scales, tensors.ts:154-160)
    per layer:
      q, k, v   = one product over the three matrices' rows, its input RMSNorm + quantize_x fused (pllm_gemv pro 1)
      q/k norms, RoPE at pos, k and v into the cache, attention over 0..pos (pllm_attention_step: split-KV)
      x += wo . quantize_x(attention)      (pllm_gemv pro 2, epi 1: the residual add fused)
      hb = silu(w1 . h) * (w3 . h), h = quantize_x(RMSNorm(x))  (pllm_gemv pro 1, epi 2: w1's and w3's rows in one)
      x += w2 . quantize_x(hb)            (pllm_gemv pro 2, epi 1)
    logits = wcls . quantize_x(RMSNorm(x))

With an exchange (pllm.tp.Exchange: tensor parallelism, one process a GPU) each rank holds its share of the matrices
(pllm.tp.Shard) and its heads' cache; wo and w2 send their partials to every rank (pllm_gemv_tp epi 3) instead of
adding them to x, and the next product sums them into x in its prologue (pro 3), x alternating between two buffers
(the prologue's CTAs all read one while the first writes the other). The logits are the rank's vocab rows.

Every product's group sums are the reference kernels' exact integers; the float32 around them agrees with the
reference's within rounding of other summation orders, which a deep random net carries through quantize_x's rounding
boundaries (the tests: 2e-2 of the largest logit at two layers of the Qwen3-8B widths). Engine(exact=True) runs every
step in the reference kernels' own order of float32 operations instead (pllm_exact_*): the oracle's logits to the bit.
"""
import os
from dataclasses import dataclass

import numpy as np

from .device import Buffer, Pinned, init
from .lib import L, check
from .tp import Shard

F_Q8, F_T2 = 0, 2
PRO_Q, PRO_RMS, PRO_QUANT, PRO_RMS_SUM = 0, 1, 2, 3
EPI_STORE, EPI_ADD, EPI_SWIGLU, EPI_SEND = 0, 1, 2, 3


@dataclass
class Config:
    dim: int
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_size: int
    vocab: int
    seq_len: int
    qk_norm: bool = False
    rope_theta: float = 10000.0
    eps: float = 1e-5
    relaxed: bool = False     # matmul_q8r's activations (bias 64, qmax 63) in place of matmul_q8's (qmax 127)
    half_kv: bool = True      # a float16 cache (to_f16 / attention_f16), as engine.ts:191 chooses for int8 models
    weights: str = "q8"       # the matrices' format: "q8" int8 groups of 32, "t2" packed ternary (ternary.ts)
    kinds: str = ""           # an LFM2's layers, a letter each: "c" a convolution layer, "a" attention ("": all "a")
    taps: int = 3             # a convolution layer's taps (conv_L_cache)

    def kind(self, l):
        return self.kinds[l] if self.kinds else "a"

    @property
    def qdim(self):
        return self.heads * self.head_size

    @property
    def kvdim(self):
        return self.kv_heads * self.head_size

    @property
    def bytes_per_weight(self):
        """int8: the value and 4 / 32 of a float32 scale; ternary: 2 bits and 2 / 128 of a float16 scale."""
        return 1.125 if self.weights == "q8" else 0.25 + 2 / 128

    def weight_bytes(self):
        """The bytes a decode step reads of the matrices (values and scales)."""
        attn = (self.qdim + 2 * self.kvdim) * self.dim + self.dim * self.qdim
        conv = 3 * self.dim * self.dim + self.dim * self.dim
        total = sum((conv if self.kind(l) == "c" else attn) + 3 * self.hidden * self.dim for l in range(self.layers))
        return int((total + self.vocab * self.dim) * self.bytes_per_weight)


# the BASELINE configurations (synthetic weights of these shapes)
STORIES15M = Config(dim=288, hidden=768, layers=6, heads=6, kv_heads=6, head_size=48, vocab=32000, seq_len=256)
QWEN3_8B = Config(dim=4096, hidden=12288, layers=36, heads=32, kv_heads=8, head_size=128, vocab=151936, seq_len=2560,
                  qk_norm=True, rope_theta=1e6, eps=1e-6)
# the LFM2-350M-shaped hybrid: 10 short-convolution layers (3 taps) among 6 grouped-query attention layers
# (16 q / 8 kv heads of 64, QK-norm), SwiGLU FFN 4608, 65536 vocab (the classifier the embedding's rows)
LFM2_350M = Config(dim=1024, hidden=4608, layers=16, heads=16, kv_heads=8, head_size=64, vocab=65536, seq_len=768,
                   qk_norm=True, rope_theta=1e6, eps=1e-5, kinds="ccaccaccacacacac", taps=3)
# the 27B-class ternary decoder (every matrix ternary, the classifier too); 1024 + 256 positions
TERNARY_27B = Config(dim=5120, hidden=21504, layers=62, heads=32, kv_heads=16, head_size=128, vocab=262144,
                     seq_len=1280, weights="t2")


def rope_tables(cfg):
    """cos / sin of every position's angle of every pair of a head (float64, then float32), as the reference's
    converter writes freq_cis_real / freq_cis_imag (engine/layers.py:372-377 rope_frequencies)."""
    freqs = 1.0 / cfg.rope_theta ** (np.arange(0, cfg.head_size, 2, dtype=np.float64) / cfg.head_size)
    angles = np.outer(np.arange(cfg.seq_len, dtype=np.float64), freqs)
    return np.cos(angles).astype(np.float32), np.sin(angles).astype(np.float32)


def quantize_rows(w):
    """float32 rows -> (int8, float32 scales a group of 32): engine/packing.py's quantize (= quantize_x bias 0)."""
    g = w.reshape(-1, 32)
    scales = (np.abs(g).max(axis=1) / np.float32(127.0)).astype(np.float32)
    inv = np.divide(np.float32(1.0), scales, out=np.zeros_like(scales), where=scales > 0)
    return np.rint(g * inv[:, None]).astype(np.int8).reshape(w.shape), scales.reshape(w.shape[:-1] + (-1,))


def pack_ternary(w):
    """int8 weights in {-1, 0, +1} (rows of k) -> codes w + 1 four to a byte, weight j at bits 2 (j & 3) of byte j / 4
    (kernels/ternary.ts:25-33, engine/packing.py:100-136)."""
    c = (w.astype(np.int16) + 1).astype(np.uint8).reshape(w.shape[:-1] + (-1, 4))
    return (c[..., 0] | (c[..., 1] << 2) | (c[..., 2] << 4) | (c[..., 3] << 6)).astype(np.uint8)


def widen_ternary(packed, scales16):
    """Packed ternary rows and their float16 scales a group of 128 -> the same weights as int8 groups of 32 (the code
    less 1) with their group of 128's scale each: the same integers of every group of 32 and the same products within
    float32 rounding (the checkpoint reader's widening, engine/packing.py:48-53 for the int6 analogue)."""
    p = packed.astype(np.uint8)
    codes = np.stack([(p >> (2 * j)) & 3 for j in range(4)], axis=-1).reshape(p.shape[:-1] + (-1,))
    w = (codes.astype(np.int16) - 1).astype(np.int8)
    s = np.repeat(scales16.view(np.float16).astype(np.float32), 4, axis=-1)
    return np.ascontiguousarray(w), np.ascontiguousarray(s)


def synthetic_host_weights(cfg, seed=0, std=0.02):
    """Host weights of a small model in the reference's int8 format (N(0, std) quantized; norms N(1, 0.1) as
    tests/made_up.py:42 makes them), or (cfg.weights "t2") packed ternary (codes uniform on {-1, 0, +1}, a row's
    scale N(std, std / 10) rounded to float16 for each of its groups of 128): a dict by the oracle's field names."""
    rng = np.random.default_rng(seed)
    Lr, d, h, q, kv = cfg.layers, cfg.dim, cfg.hidden, cfg.qdim, cfg.kvdim
    W = {}

    def mat(name, shape):
        if cfg.weights == "t2":
            w = rng.integers(-1, 2, shape).astype(np.int8)
            s = rng.normal(std, std / 10, shape[:-1] + (1,)).astype(np.float16)
            W["w" + name] = pack_ternary(w)
            W["s" + name] = np.repeat(s, shape[-1] // 128, axis=-1).view(np.uint16)
            return
        w, s = quantize_rows(rng.normal(0, std, shape).astype(np.float32))
        W["w" + name], W["s" + name] = w, s

    mat("q", (Lr, q, d))
    mat("k", (Lr, kv, d))
    mat("v", (Lr, kv, d))
    mat("o", (Lr, d, q))
    mat("1", (Lr, h, d))
    mat("2", (Lr, d, h))
    mat("3", (Lr, h, d))
    W["emb"], W["emb_s"] = quantize_rows(rng.normal(0, 1.0, (cfg.vocab, d)).astype(np.float32))
    mat("cls", (cfg.vocab, d))
    W["cls"], W["cls_s"] = W.pop("wcls"), W.pop("scls")
    W["att_norm"] = rng.normal(1, 0.1, (Lr, d)).astype(np.float32)
    W["ffn_norm"] = rng.normal(1, 0.1, (Lr, d)).astype(np.float32)
    W["final_norm"] = rng.normal(1, 0.1, d).astype(np.float32)
    W["q_norm"] = rng.normal(1, 0.1, (Lr, cfg.head_size)).astype(np.float32) if cfg.qk_norm else None
    W["k_norm"] = rng.normal(1, 0.1, (Lr, cfg.head_size)).astype(np.float32) if cfg.qk_norm else None
    W["cos_t"], W["sin_t"] = rope_tables(cfg)
    return W


class Engine:
    """One model's forward pass on the current device."""

    SPLIT = 128  # positions a slice of the split-KV attention (two tiles of 64 a CTA, double-buffered)

    def __init__(self, cfg, host=None, seed=0, device=0, graphs=True, pdl=True, exchange=None, exact=False, batch=1):
        """exact: every step in the reference kernels' own order of float32 operations (pllm_exact_*: the oracle's
        logits to the bit, several times slower); else the fused kernels (the same integers, float32 within
        rounding). One rank only.
        batch: sequences decoded together, a token each a step (forward_batch / next_tokens), each with its own cache
        and position: every product streams its weights once for all of them (up to 16 a pass), the attention takes
        them in one launch. One rank, the fused kernels, a float16 cache."""
        init(device)
        if exact and exchange:
            raise ValueError("the reference-order step runs on one rank")
        if batch > 1 and (exact or exchange or not cfg.half_kv):
            raise ValueError("a batch of sequences runs on one rank, with the fused kernels and a float16 cache")
        if cfg.weights not in ("q8", "t2") or (cfg.weights == "t2" and (exact or exchange or batch > 1)):
            raise ValueError("ternary matrices run the fused single-sequence step on one rank")
        self.hybrid = "c" in cfg.kinds
        if self.hybrid and (exact or exchange or cfg.weights != "q8" or not cfg.half_kv):
            raise ValueError("convolution layers run the fused int8 step on one rank (one sequence or a batch)")
        self.fmt = F_T2 if cfg.weights == "t2" else F_Q8
        self.exact = exact
        self.batch = nb = int(batch)
        self.xg = exchange
        self.device = device
        self.shard = s = Shard(cfg, exchange.rank, exchange.world) if exchange else Shard(cfg)
        if os.environ.get("PLLM_STAGE_BUDGET"):  # the bulk-copy product's stage ring, bytes (a tuning knob)
            L.pllm_set_stage_budget(int(os.environ["PLLM_STAGE_BUDGET"]))
        self.cfg, self.graphs = cfg, graphs
        self.pdl = pdl and not os.environ.get("PLLM_NO_PDL")  # (a switch for measuring what the early launches give)
        c = cfg
        self.rows_qkv = s.rows_qkv
        self.bias = 64 if c.relaxed else 0
        B = {}
        ng = lambda cols: cols // 32  # noqa: E731
        # the matrices (this rank's share), a layer's after another; q, k, v rows in one, w1 rows then w3 rows in one
        wb, sb = self.wb, self.sb
        B["wqkv"] = Buffer(c.layers * self.rows_qkv * wb(c.dim))
        B["sqkv"] = Buffer(c.layers * self.rows_qkv * sb(c.dim))
        B["wo"] = Buffer(c.layers * c.dim * wb(s.qdim))
        B["so"] = Buffer(c.layers * c.dim * sb(s.qdim))
        B["w13"] = Buffer(c.layers * 2 * s.hidden * wb(c.dim))
        B["s13"] = Buffer(c.layers * 2 * s.hidden * sb(c.dim))
        B["w2"] = Buffer(c.layers * c.dim * wb(s.hidden))
        B["s2"] = Buffer(c.layers * c.dim * sb(s.hidden))
        B["emb"] = Buffer(c.vocab * c.dim)
        B["emb_s"] = Buffer(c.vocab * ng(c.dim) * 4)
        B["cls"] = Buffer(s.vocab * wb(c.dim))
        B["cls_s"] = Buffer(s.vocab * sb(c.dim))
        if self.hybrid:  # a convolution layer's in (3 dim rows: B, C, x) and out matrices, its taps, its sequences' rows
            B["win"], B["swin"] = Buffer(c.layers * 3 * c.dim * c.dim), Buffer(c.layers * 3 * c.dim * c.dim // 8)
            B["wout"], B["swout"] = Buffer(c.layers * c.dim * c.dim), Buffer(c.layers * c.dim * c.dim // 8)
            B["taps"] = Buffer(c.layers * c.taps * c.dim * 4)
            B["rows"] = Buffer(c.layers * nb * c.taps * c.dim * 4).zero()
            B["mixed"] = Buffer(nb * 3 * c.dim * 4)
        B["att_norm"] = Buffer(c.layers * c.dim * 4)
        B["ffn_norm"] = Buffer(c.layers * c.dim * 4)
        B["final_norm"] = Buffer(c.dim * 4)
        B["q_norm"] = Buffer(c.layers * c.head_size * 4) if c.qk_norm else None
        B["k_norm"] = Buffer(c.layers * c.head_size * 4) if c.qk_norm else None
        B["cos_t"] = Buffer(c.seq_len * c.head_size // 2 * 4)
        B["sin_t"] = Buffer(c.seq_len * c.head_size // 2 * 4)
        E = 2 if c.half_kv else 4
        # the caches: [layer][sequence][position][kv heads x head size]
        B["kc"] = Buffer(c.layers * nb * c.seq_len * s.kvdim * E).zero()
        B["vc"] = Buffer(c.layers * nb * c.seq_len * s.kvdim * E).zero()
        # activations (a row a sequence)
        B["x"] = Buffer(nb * c.dim * 4)
        B["x1"] = Buffer(c.dim * 4) if exchange else None  # the residual's other buffer (tensor-parallel)
        B["qkv"] = Buffer(nb * self.rows_qkv * 4)
        self.att_stride = max(s.qdim, c.dim) if self.hybrid else s.qdim  # a convolution layer's output too
        B["att"] = Buffer(nb * self.att_stride * 4)
        B["hb"] = Buffer(nb * s.hidden * 4)
        B["logits"] = Buffer(nb * s.vocab * 4)
        B["tp"] = Buffer(8 * nb).zero()  # the tokens, then the positions, read by the kernels
        B["bad"] = Buffer(4).zero()     # non-finite keys / values written to a float16 cache (halves.ts:35)
        B["next"] = Buffer(4)           # the greedy step's token (pllm_argmax_dev) and its scratch
        B["amx"] = Buffer(16).zero()
        self.scratch_bytes = (L.pllm_attention_scratch_bytes(s.heads, c.head_size, c.seq_len, self.SPLIT) + 255) & ~255
        B["scratch"] = Buffer(nb * self.scratch_bytes).zero()
        if nb > 1:  # w2's input quantized for its product (K too long to quantize in shared memory for 16 tokens)
            B["hq"], B["hq_scales"] = Buffer(nb * s.hidden), Buffer(nb * s.hidden // 8)
            B["nexts"] = Buffer(4 * nb)
        if exact:  # the reference-order step's quantized activations, w1 / w3 rows and attention scores
            wide = max(c.dim, c.qdim, c.hidden)
            B["xq"], B["xs"] = Buffer(wide), Buffer(wide // 8)
            B["h13"], B["scores"] = Buffer(2 * c.hidden * 4), Buffer(c.heads * c.seq_len * 4)
        self.B = B
        if host is not None:
            self.load(host)
        else:
            self.synthesize(seed)
        self.stream = L.pllm_stream_create()
        self.tp_host = Pinned(2 * nb, np.int32)
        self.logits_host = Pinned(nb * s.vocab, np.float32)
        self.next_host = Pinned(nb, np.int32)
        self.graph = 0
        check("Engine")

    # ---- weights
    def wb(self, k):
        """Bytes of a row of k weights' values: int8 k, ternary k / 4 (four codes a byte)."""
        return k if self.fmt == F_Q8 else k // 4

    def sb(self, k):
        """Bytes of a row of k weights' scales: int8 a float32 a group of 32, ternary a float16 a group of 128."""
        return k // 8 if self.fmt == F_Q8 else k // 64

    def load(self, W):
        """Host weights (synthetic_host_weights' dict, the reference's int8 layout) into the device layout (this rank's
        share of them with an exchange)."""
        c, B = self.cfg, self.B
        if self.xg:
            W = self.shard.host_share(W)
        B["wqkv"].upload(np.concatenate([W["wq"], W["wk"], W["wv"]], axis=1))
        B["sqkv"].upload(np.concatenate([W["sq"], W["sk"], W["sv"]], axis=1))
        B["wo"].upload(W["wo"])
        B["so"].upload(W["so"])
        B["w13"].upload(np.concatenate([W["w1"], W["w3"]], axis=1))
        B["s13"].upload(np.concatenate([W["s1"], W["s3"]], axis=1))
        B["w2"].upload(W["w2"])
        B["s2"].upload(W["s2"])
        for k in ("emb", "emb_s", "cls", "cls_s", "att_norm", "ffn_norm", "final_norm", "cos_t", "sin_t"):
            B[k].upload(W[k])
        if self.hybrid:
            for k in ("win", "swin", "wout", "swout", "taps"):
                B[k].upload(W[k])
        if c.qk_norm:
            B["q_norm"].upload(W["q_norm"])
            B["k_norm"].upload(W["k_norm"])
        L.pllm_sync()
        check("load")

    def synthesize(self, seed):
        """Seeded synthetic weights made on the device: N(0, 0.02) int8 matrices (the embedding N(0, 1)), norms
        N(1, 0.1), the RoPE tables of the configuration."""
        c, B = self.cfg, self.B
        s = seed * 1000
        if self.fmt == F_T2:  # codes uniform on {-1, 0, +1}, a row's scale N(0.02, 0.002) rounded to float16
            for i, (w, sc, rows, cols) in enumerate([
                    ("wqkv", "sqkv", c.layers * self.rows_qkv, c.dim), ("wo", "so", c.layers * c.dim, c.qdim),
                    ("w13", "s13", c.layers * 2 * c.hidden, c.dim), ("w2", "s2", c.layers * c.dim, c.hidden),
                    ("cls", "cls_s", c.vocab, c.dim)]):
                L.pllm_synth_t2(B[w].ptr, B[sc].ptr, rows, cols, s + i, 0.02, 0.002)
        elif self.xg:
            self._synthesize_share(s)
        else:
            for i, (w, sc, rows, cols) in enumerate([
                    ("wqkv", "sqkv", c.layers * self.rows_qkv, c.dim), ("wo", "so", c.layers * c.dim, c.qdim),
                    ("w13", "s13", c.layers * 2 * c.hidden, c.dim), ("w2", "s2", c.layers * c.dim, c.hidden),
                    ("cls", "cls_s", c.vocab, c.dim)]):
                L.pllm_synth_q8(B[w].ptr, B[sc].ptr, rows, cols, s + i, 0.02)
        if self.hybrid:
            L.pllm_synth_q8(B["win"].ptr, B["swin"].ptr, c.layers * 3 * c.dim, c.dim, s + 5, 0.02)
            L.pllm_synth_q8(B["wout"].ptr, B["swout"].ptr, c.layers * c.dim, c.dim, s + 6, 0.02)
            L.pllm_synth_f32(B["taps"].ptr, c.layers * c.taps * c.dim, s + 7, 0.0, 0.3)
        L.pllm_synth_q8(B["emb"].ptr, B["emb_s"].ptr, c.vocab, c.dim, s + 10, 1.0)
        for i, k in enumerate(("att_norm", "ffn_norm", "final_norm", "q_norm", "k_norm")):
            if B[k] is not None:
                L.pllm_synth_f32(B[k].ptr, B[k].nbytes // 4, s + 20 + i, 1.0, 0.1)
        cos, sin = rope_tables(c)
        B["cos_t"].upload(cos)
        B["sin_t"].upload(sin)
        L.pllm_sync()
        check("synthesize")

    def _synthesize_share(self, s):
        """This rank's blocks of the matrices synthesize() makes whole (the same bytes: pllm_synth_q8_block)."""
        c, B, sh = self.cfg, self.B, self.shard
        blk = lambda w, sc, row, nrows, cols, row0, col0, full, seed: L.pllm_synth_q8_block(  # noqa: E731
            B[w].ptr + row * cols, B[sc].ptr + row * (cols // 32) * 4, nrows, cols, seed, 0.02, row0, col0, full)
        R = c.qdim + 2 * c.kvdim  # a layer's q/k/v rows in the whole model
        for l in range(c.layers):
            at = l * self.rows_qkv
            blk("wqkv", "sqkv", at, sh.qdim, c.dim, l * R + sh.q_rows().start, 0, c.dim, s)
            blk("wqkv", "sqkv", at + sh.qdim, sh.kvdim, c.dim, l * R + c.qdim + sh.kv_rows().start, 0, c.dim, s)
            blk("wqkv", "sqkv", at + sh.qdim + sh.kvdim, sh.kvdim, c.dim,
                l * R + c.qdim + c.kvdim + sh.kv_rows().start, 0, c.dim, s)
            at = l * 2 * sh.hidden
            blk("w13", "s13", at, sh.hidden, c.dim, l * 2 * c.hidden + sh.hidden_rows().start, 0, c.dim, s + 2)
            blk("w13", "s13", at + sh.hidden, sh.hidden, c.dim, l * 2 * c.hidden + c.hidden + sh.hidden_rows().start,
                0, c.dim, s + 2)
        blk("wo", "so", 0, c.layers * c.dim, sh.qdim, 0, sh.q_rows().start, c.qdim, s + 1)
        blk("w2", "s2", 0, c.layers * c.dim, sh.hidden, 0, sh.hidden_rows().start, c.hidden, s + 3)
        blk("cls", "cls_s", 0, sh.vocab, c.dim, sh.vocab_rows().start, 0, c.dim, s + 4)

    def host_weights(self):
        """The device weights back in the oracle's layout (for the CPU baseline and the checks); ternary matrices
        widened to int8 groups of 32 (widen_ternary: the same integers)."""
        c, B, sh = self.cfg, self.B, self.shard
        if self.fmt == F_T2:
            return self._host_weights_t2()
        d = lambda k, dt: B[k].download(dt)  # noqa: E731
        W = {}
        qkv = d("wqkv", np.int8).reshape(c.layers, self.rows_qkv, c.dim)
        sqkv = d("sqkv", np.float32).reshape(c.layers, self.rows_qkv, c.dim // 32)
        W["wq"], W["wk"], W["wv"] = np.split(qkv, [sh.qdim, sh.qdim + sh.kvdim], axis=1)
        W["sq"], W["sk"], W["sv"] = np.split(sqkv, [sh.qdim, sh.qdim + sh.kvdim], axis=1)
        W["wo"], W["so"] = d("wo", np.int8), d("so", np.float32)
        w13 = d("w13", np.int8).reshape(c.layers, 2 * sh.hidden, c.dim)
        s13 = d("s13", np.float32).reshape(c.layers, 2 * sh.hidden, c.dim // 32)
        W["w1"], W["w3"] = w13[:, :sh.hidden], w13[:, sh.hidden:]
        W["s1"], W["s3"] = s13[:, :sh.hidden], s13[:, sh.hidden:]
        W["w2"], W["s2"] = d("w2", np.int8), d("s2", np.float32)
        for k, dt in (("emb", np.int8), ("emb_s", np.float32), ("cls", np.int8), ("cls_s", np.float32),
                      ("att_norm", np.float32), ("ffn_norm", np.float32), ("final_norm", np.float32),
                      ("cos_t", np.float32), ("sin_t", np.float32)):
            W[k] = d(k, dt)
        W["q_norm"] = d("q_norm", np.float32) if c.qk_norm else None
        W["k_norm"] = d("k_norm", np.float32) if c.qk_norm else None
        if self.hybrid:
            W["win"] = d("win", np.int8).reshape(c.layers, 3 * c.dim, c.dim)
            W["swin"] = d("swin", np.float32).reshape(c.layers, 3 * c.dim, c.dim // 32)
            W["wout"] = d("wout", np.int8).reshape(c.layers, c.dim, c.dim)
            W["swout"] = d("swout", np.float32).reshape(c.layers, c.dim, c.dim // 32)
            W["taps"] = d("taps", np.float32).reshape(c.layers, c.taps, c.dim)
        return {k: (np.ascontiguousarray(v) if v is not None else None) for k, v in W.items()}

    def _host_weights_t2(self):
        c, B = self.cfg, self.B
        d = lambda k, dt: B[k].download(dt)  # noqa: E731
        W = {}

        def mat(key, skey, rows, k):
            return widen_ternary(d(key, np.uint8).reshape(rows, k // 4), d(skey, np.uint16).reshape(rows, k // 128))
        qkv, sqkv = mat("wqkv", "sqkv", c.layers * self.rows_qkv, c.dim)
        qkv, sqkv = qkv.reshape(c.layers, self.rows_qkv, -1), sqkv.reshape(c.layers, self.rows_qkv, -1)
        W["wq"], W["wk"], W["wv"] = np.split(qkv, [c.qdim, c.qdim + c.kvdim], axis=1)
        W["sq"], W["sk"], W["sv"] = np.split(sqkv, [c.qdim, c.qdim + c.kvdim], axis=1)
        W["wo"], W["so"] = mat("wo", "so", c.layers * c.dim, c.qdim)
        w13, s13 = mat("w13", "s13", c.layers * 2 * c.hidden, c.dim)
        w13, s13 = w13.reshape(c.layers, 2 * c.hidden, -1), s13.reshape(c.layers, 2 * c.hidden, -1)
        W["w1"], W["w3"] = w13[:, :c.hidden], w13[:, c.hidden:]
        W["s1"], W["s3"] = s13[:, :c.hidden], s13[:, c.hidden:]
        W["w2"], W["s2"] = mat("w2", "s2", c.layers * c.dim, c.hidden)
        W["cls"], W["cls_s"] = mat("cls", "cls_s", c.vocab, c.dim)
        for k, dt in (("emb", np.int8), ("emb_s", np.float32), ("att_norm", np.float32), ("ffn_norm", np.float32),
                      ("final_norm", np.float32), ("cos_t", np.float32), ("sin_t", np.float32)):
            W[k] = d(k, dt)
        W["q_norm"] = d("q_norm", np.float32) if c.qk_norm else None
        W["k_norm"] = d("k_norm", np.float32) if c.qk_norm else None
        return {k: (np.ascontiguousarray(v) if v is not None else None) for k, v in W.items()}

    # ---- one step
    def _gemv(self, out, wq, ws, rows, n, x, norm, pro, epi, pair=0, pdl=True):
        c = self.cfg
        L.pllm_gemv(out, 0, 0, 0, 0, 0, x, 0, norm, c.eps, self.bias, wq, ws, self.fmt, n, 0, rows, 1, pro, epi,
                    pair, int(pdl and self.pdl))

    @property
    def launches_per_step(self):
        """Kernels a step launches: the embedding, five a layer (the q/k/v product; the attention with the q / k
        norms, RoPE, the cache write and its slices' combine inside; the wo, w1/w3 and w2 products), the classifier."""
        if self.exact:
            return 3 + 11 * self.cfg.layers
        if self.batch > 1:  # the attention's slices combined by a second kernel where clusters do not take it
            return 2 + 6 * self.cfg.layers
        return 2 + 5 * self.cfg.layers + (1 if self.xg else 0)

    def _enqueue_exact_step(self, need_logits=True):
        """A step in the reference kernels' order of float32 operations (pllm_exact_*), as the oracle's forward
        (oracle/pllm_oracle.c or_forward) and the reference's engine.ts:421-475 run it: rmsnorm + quantize_x, the
        q/k/v products, the head norms, rope and the cache, attentionOf, quantize_x + wo (x +=), rmsnorm + quantize_x,
        w1 and w3, swiglu + quantize_x, w2 (x +=); the final norm and the classifier."""
        c, B = self.cfg, self.B
        tok, pos = B["tp"].ptr, B["tp"].ptr + 4
        E, half, rel = (2 if c.half_kv else 4), int(c.half_kv), int(c.relaxed)
        xq, xs, x = B["xq"].ptr, B["xs"].ptr, B["x"].ptr
        L.pllm_embed_q8(x, B["emb"].ptr, B["emb_s"].ptr, tok, 0, c.dim, 1, c.dim)
        for l in range(c.layers):
            L.pllm_exact_prepare(xq, xs, 0, x, B["att_norm"].ptr + l * c.dim * 4, c.dim, c.eps, self.bias, 1)
            L.pllm_exact_product(B["qkv"].ptr, 0, xq, xs, B["wqkv"].ptr + l * self.rows_qkv * c.dim,
                                 B["sqkv"].ptr + l * self.rows_qkv * (c.dim // 32) * 4, c.dim, self.rows_qkv, rel)
            kc = B["kc"].ptr + l * c.seq_len * c.kvdim * E
            vc = B["vc"].ptr + l * c.seq_len * c.kvdim * E
            qn = B["q_norm"].ptr + l * c.head_size * 4 if c.qk_norm else 0
            kn = B["k_norm"].ptr + l * c.head_size * 4 if c.qk_norm else 0
            L.pllm_exact_qk_rope_cache(B["qkv"].ptr, qn, kn, B["cos_t"].ptr, B["sin_t"].ptr, pos, 0, kc, vc, c.heads,
                                       c.kv_heads, c.head_size, c.eps, half, B["bad"].ptr)
            L.pllm_exact_attention(B["att"].ptr, B["qkv"].ptr, kc, vc, B["scores"].ptr, pos, 0, c.seq_len, c.heads,
                                   c.kv_heads, c.head_size, half, 0.0)
            L.pllm_exact_prepare(xq, xs, 0, B["att"].ptr, 0, c.qdim, c.eps, self.bias, 0)
            L.pllm_exact_product(x, x, xq, xs, B["wo"].ptr + l * c.dim * c.qdim,
                                 B["so"].ptr + l * c.dim * (c.qdim // 32) * 4, c.qdim, c.dim, rel)
            L.pllm_exact_prepare(xq, xs, 0, x, B["ffn_norm"].ptr + l * c.dim * 4, c.dim, c.eps, self.bias, 1)
            L.pllm_exact_product(B["h13"].ptr, 0, xq, xs, B["w13"].ptr + l * 2 * c.hidden * c.dim,
                                 B["s13"].ptr + l * 2 * c.hidden * (c.dim // 32) * 4, c.dim, 2 * c.hidden, rel)
            L.pllm_exact_prepare(xq, xs, 0, B["h13"].ptr, 0, c.hidden, c.eps, self.bias, 2)
            L.pllm_exact_product(x, x, xq, xs, B["w2"].ptr + l * c.dim * c.hidden,
                                 B["s2"].ptr + l * c.dim * (c.hidden // 32) * 4, c.hidden, c.dim, rel)
        if need_logits:
            L.pllm_exact_prepare(xq, xs, 0, x, B["final_norm"].ptr, c.dim, c.eps, self.bias, 1)
            L.pllm_exact_product(B["logits"].ptr, 0, xq, xs, B["cls"].ptr, B["cls_s"].ptr, c.dim, c.vocab, rel)

    def _enqueue_batch_step(self, need_logits=True):
        """A step of the batch's sequences: every product over all of them at once (the batched tensor-core form of
        pllm_gemv, count = batch), the attention of all of them in one launch (pllm_attention_step_batch: each
        sequence its own cache and position)."""
        c, B, nb = self.cfg, self.B, self.batch
        toks, poss = B["tp"].ptr, B["tp"].ptr + 4 * nb
        E, pdl = 2, int(self.pdl)
        x, qkv, att, hb = B["x"].ptr, B["qkv"].ptr, B["att"].ptr, B["hb"].ptr
        R = self.rows_qkv
        L.pllm_embed_q8(x, B["emb"].ptr, B["emb_s"].ptr, toks, 0, c.dim, nb, c.dim)

        def gemv(out, ldo, xin, ldx, norm, wq, ws, rows, k, pro, epi, pair=0, xq=0, xs=0, bias=None):
            L.pllm_gemv(out, ldo, xq, xs, k if xq else 0, k // 8 if xq else 0, xin, ldx, norm, c.eps,
                        self.bias if bias is None else bias, wq, ws, F_Q8, k, 0, rows, nb, pro, epi, pair, pdl)

        def quantized(xin, ldx, norm, k):
            """The batch's activations (RMSNorm with norm, or none: 0) quantized once, signed int8 (the bias taken
            off) into hq: a product over them loads them as they are, where every CTA of a product that quantizes in
            its own prologue makes all the batch's tokens again (measured at batch 16: the products' prologues took
            most of the step)."""
            L.pllm_norm_quantize_rows(B["hq"].ptr, B["hq_scales"].ptr, xin, ldx, norm, c.eps, k, nb, self.bias)
            return {"xq": B["hq"].ptr, "xs": B["hq_scales"].ptr, "bias": 0}
        self._quantized = quantized
        layer_cache = nb * c.seq_len * c.kvdim * E
        A, d = self.att_stride, c.dim
        for l in range(c.layers):
            if c.kind(l) == "c":  # the convolution layer of every sequence: its rows at rows + (l nb + z) taps dim
                gemv(B["mixed"].ptr, 3 * d, x, d, B["att_norm"].ptr + l * d * 4, B["win"].ptr + l * 3 * d * d,
                     B["swin"].ptr + l * 3 * d * (d // 32) * 4, 3 * d, d, PRO_RMS, EPI_STORE)
                L.pllm_conv_step(att, A, B["taps"].ptr + l * c.taps * d * 4, B["rows"].ptr + l * nb * c.taps * d * 4,
                                 c.taps * d, B["mixed"].ptr, 3 * d, d, c.taps, poss, nb)
                gemv(x, d, att, A, 0, B["wout"].ptr + l * d * d, B["swout"].ptr + l * d * (d // 32) * 4, d, d,
                     PRO_QUANT, EPI_ADD)
                self._enqueue_batch_ffn(l, gemv)
                continue
            gemv(qkv, R, 0, 0, 0, B["wqkv"].ptr + l * R * c.dim, B["sqkv"].ptr + l * R * (c.dim // 32) * 4, R,
                 c.dim, PRO_Q, EPI_STORE, **quantized(x, c.dim, B["att_norm"].ptr + l * c.dim * 4, c.dim))
            qn = B["q_norm"].ptr + l * c.head_size * 4 if c.qk_norm else 0
            kn = B["k_norm"].ptr + l * c.head_size * 4 if c.qk_norm else 0
            L.pllm_attention_step_batch(att, A, qkv, R, B["kc"].ptr + l * layer_cache,
                                        B["vc"].ptr + l * layer_cache, c.seq_len * c.kvdim * E, B["scratch"].ptr, poss,
                                        nb, c.seq_len, c.heads, c.kv_heads, c.head_size, 0.0, self.SPLIT, qn, kn,
                                        B["cos_t"].ptr, B["sin_t"].ptr, 0, c.eps, B["bad"].ptr, pdl)
            gemv(x, c.dim, 0, 0, 0, B["wo"].ptr + l * c.dim * c.qdim, B["so"].ptr + l * c.dim * (c.qdim // 32) * 4,
                 c.dim, c.qdim, PRO_Q, EPI_ADD, **quantized(att, A, 0, c.qdim))
            self._enqueue_batch_ffn(l, gemv)
        if need_logits:
            gemv(B["logits"].ptr, c.vocab, 0, 0, 0, B["cls"].ptr, B["cls_s"].ptr, c.vocab, c.dim, PRO_Q, EPI_STORE,
                 **quantized(x, c.dim, B["final_norm"].ptr, c.dim))

    def _enqueue_batch_ffn(self, l, gemv):
        """Layer l's gated FFN of the batch's sequences: the activations of each product quantized once first (w1/w3:
        RMSNorm and quantize_x; w2's K, the hidden width, then read from global memory by the batched product)."""
        c, B, nb = self.cfg, self.B, self.batch
        x, hb = B["x"].ptr, B["hb"].ptr
        gemv(hb, c.hidden, 0, 0, 0, B["w13"].ptr + l * 2 * c.hidden * c.dim,
             B["s13"].ptr + l * 2 * c.hidden * (c.dim // 32) * 4, c.hidden, c.dim, PRO_Q, EPI_SWIGLU, pair=c.hidden,
             **self._quantized(x, c.dim, B["ffn_norm"].ptr + l * c.dim * 4, c.dim))
        L.pllm_quantize_tokens(B["hq"].ptr, B["hq_scales"].ptr, hb, c.hidden, self.bias, nb)
        gemv(x, c.dim, 0, 0, 0, B["w2"].ptr + l * c.dim * c.hidden, B["s2"].ptr + l * c.dim * (c.hidden // 32) * 4,
             c.dim, c.hidden, PRO_Q, EPI_ADD, xq=B["hq"].ptr, xs=B["hq_scales"].ptr)

    def _enqueue_step(self, need_logits=True):
        if self.batch > 1:
            return self._enqueue_batch_step(need_logits)
        if self.exact:
            return self._enqueue_exact_step(need_logits)
        if self.xg:
            return self._enqueue_tp_step(need_logits)
        c, B = self.cfg, self.B
        tok, pos = B["tp"].ptr, B["tp"].ptr + 4
        E = 2 if c.half_kv else 4
        wb, sb = self.wb, self.sb
        L.pllm_embed_q8(B["x"].ptr, B["emb"].ptr, B["emb_s"].ptr, tok, 0, c.dim, 1, c.dim)
        for l in range(c.layers):
            if c.kind(l) == "c":
                self._enqueue_conv(l, pos)
                self._enqueue_ffn(l)
                continue
            wqkv = B["wqkv"].ptr + l * self.rows_qkv * wb(c.dim)
            sqkv = B["sqkv"].ptr + l * self.rows_qkv * sb(c.dim)
            self._gemv(B["qkv"].ptr, wqkv, sqkv, self.rows_qkv, c.dim, B["x"].ptr, B["att_norm"].ptr + l * c.dim * 4,
                       PRO_RMS, EPI_STORE)
            kc = B["kc"].ptr + l * c.seq_len * c.kvdim * E
            vc = B["vc"].ptr + l * c.seq_len * c.kvdim * E
            qn = B["q_norm"].ptr + l * c.head_size * 4 if c.qk_norm else 0
            kn = B["k_norm"].ptr + l * c.head_size * 4 if c.qk_norm else 0
            L.pllm_attention_step(B["att"].ptr, B["qkv"].ptr, kc, vc, B["scratch"].ptr, pos, c.seq_len, c.heads,
                                  c.kv_heads, c.head_size, int(c.half_kv), 0.0, self.SPLIT, qn, kn, B["cos_t"].ptr,
                                  B["sin_t"].ptr, 0, c.eps, B["bad"].ptr, int(self.pdl))
            self._gemv(B["x"].ptr, B["wo"].ptr + l * c.dim * wb(c.qdim), B["so"].ptr + l * c.dim * sb(c.qdim),
                       c.dim, c.qdim, B["att"].ptr, 0, PRO_QUANT, EPI_ADD)
            self._enqueue_ffn(l)
        if need_logits:
            self._gemv(B["logits"].ptr, B["cls"].ptr, B["cls_s"].ptr, c.vocab, c.dim, B["x"].ptr, B["final_norm"].ptr,
                       PRO_RMS, EPI_STORE)

    def _enqueue_ffn(self, l):
        """Layer l's gated FFN of one sequence: x += w2 . quantize_x(silu(w1 . h) * (w3 . h)), h = RMSNorm(x)."""
        c, B, wb, sb = self.cfg, self.B, self.wb, self.sb
        self._gemv(B["hb"].ptr, B["w13"].ptr + l * 2 * c.hidden * wb(c.dim), B["s13"].ptr + l * 2 * c.hidden * sb(c.dim),
                   c.hidden, c.dim, B["x"].ptr, B["ffn_norm"].ptr + l * c.dim * 4, PRO_RMS, EPI_SWIGLU, pair=c.hidden)
        self._gemv(B["x"].ptr, B["w2"].ptr + l * c.dim * wb(c.hidden), B["s2"].ptr + l * c.dim * sb(c.hidden), c.dim,
                   c.hidden, B["hb"].ptr, 0, PRO_QUANT, EPI_ADD)

    def _enqueue_conv(self, l, pos):
        """An LFM2 convolution layer of one sequence (forward/convolution.ts:51-60): mixed = win . quantize_x(RMSNorm
        (x)) ([B | C | z]), the rows' shift and the causal convolution (pllm_conv_step), x += wout . quantize_x(it)."""
        c, B = self.cfg, self.B
        d = c.dim
        self._gemv(B["mixed"].ptr, B["win"].ptr + l * 3 * d * d, B["swin"].ptr + l * 3 * d * (d // 32) * 4, 3 * d, d,
                   B["x"].ptr, B["att_norm"].ptr + l * d * 4, PRO_RMS, EPI_STORE)
        L.pllm_conv_step(B["att"].ptr, 0, B["taps"].ptr + l * c.taps * d * 4, B["rows"].ptr + l * c.taps * d * 4, 0,
                         B["mixed"].ptr, 0, d, c.taps, pos, 1)
        self._gemv(B["x"].ptr, B["wout"].ptr + l * d * d, B["swout"].ptr + l * d * (d // 32) * 4, d, d, B["att"].ptr, 0,
                   PRO_QUANT, EPI_ADD)

    def _enqueue_tp_step(self, need_logits=True):
        """One tensor-parallel step: reduction 2 l after layer l's wo (summed into x1 by its w1/w3 product), 2 l + 1
        after its w2 (summed into x by the next layer's q/k/v product, or the classifier's)."""
        c, B, sh, xg = self.cfg, self.B, self.shard, self.xg.h
        tok, pos = B["tp"].ptr, B["tp"].ptr + 4
        E = 2 if c.half_kv else 4
        pdl = int(self.pdl)
        x0, x1 = B["x"].ptr, B["x1"].ptr
        L.pllm_tp_step(xg)
        L.pllm_embed_q8(x0, B["emb"].ptr, B["emb_s"].ptr, tok, 0, c.dim, 1, c.dim)
        for l in range(c.layers):
            wqkv = B["wqkv"].ptr + l * self.rows_qkv * c.dim
            sqkv = B["sqkv"].ptr + l * self.rows_qkv * (c.dim // 32) * 4
            norm = B["att_norm"].ptr + l * c.dim * 4
            if l == 0:
                L.pllm_gemv_tp(B["qkv"].ptr, x0, 0, norm, c.eps, self.bias, wqkv, sqkv, c.dim, self.rows_qkv,
                               PRO_RMS, EPI_STORE, 0, pdl, xg, 0)
            else:
                L.pllm_gemv_tp(B["qkv"].ptr, x1, x0, norm, c.eps, self.bias, wqkv, sqkv, c.dim, self.rows_qkv,
                               PRO_RMS_SUM, EPI_STORE, 0, pdl, xg, 2 * l - 1)
            kc = B["kc"].ptr + l * c.seq_len * sh.kvdim * E
            vc = B["vc"].ptr + l * c.seq_len * sh.kvdim * E
            qn = B["q_norm"].ptr + l * c.head_size * 4 if c.qk_norm else 0
            kn = B["k_norm"].ptr + l * c.head_size * 4 if c.qk_norm else 0
            L.pllm_attention_step(B["att"].ptr, B["qkv"].ptr, kc, vc, B["scratch"].ptr, pos, c.seq_len, sh.heads,
                                  sh.kv_heads, c.head_size, int(c.half_kv), 0.0, self.SPLIT, qn, kn, B["cos_t"].ptr,
                                  B["sin_t"].ptr, 0, c.eps, B["bad"].ptr, pdl)
            L.pllm_gemv_tp(0, B["att"].ptr, 0, 0, c.eps, self.bias, B["wo"].ptr + l * c.dim * sh.qdim,
                           B["so"].ptr + l * c.dim * (sh.qdim // 32) * 4, sh.qdim, c.dim, PRO_QUANT, EPI_SEND, 0, pdl,
                           xg, 2 * l)
            L.pllm_gemv_tp(B["hb"].ptr, x0, x1, B["ffn_norm"].ptr + l * c.dim * 4, c.eps, self.bias,
                           B["w13"].ptr + l * 2 * sh.hidden * c.dim, B["s13"].ptr + l * 2 * sh.hidden * (c.dim // 32) * 4,
                           c.dim, sh.hidden, PRO_RMS_SUM, EPI_SWIGLU, sh.hidden, pdl, xg, 2 * l)
            L.pllm_gemv_tp(0, B["hb"].ptr, 0, 0, c.eps, self.bias, B["w2"].ptr + l * c.dim * sh.hidden,
                           B["s2"].ptr + l * c.dim * (sh.hidden // 32) * 4, sh.hidden, c.dim, PRO_QUANT, EPI_SEND, 0,
                           pdl, xg, 2 * l + 1)
        # the classifier sums the last reduction whether or not the logits are wanted (every rank takes every step)
        L.pllm_gemv_tp(B["logits"].ptr, x1, x0, B["final_norm"].ptr, c.eps, self.bias, B["cls"].ptr, B["cls_s"].ptr,
                       c.dim, sh.vocab, PRO_RMS_SUM, EPI_STORE, 0, pdl, xg, 2 * c.layers - 1)

    def capture(self):
        """Record one decode step (with logits) as a CUDA graph on the engine's stream."""
        L.pllm_set_stream(self.stream)
        if self.graph:
            L.pllm_graph_destroy(self.graph)
        if L.pllm_graph_begin() != 0:
            check("graph begin")
        self._enqueue_step(True)
        self.graph = L.pllm_graph_end()
        check("graph capture")
        if not self.graph:
            raise RuntimeError("graph capture failed")

    def graph_of(self, enqueue):
        """A CUDA graph of what enqueue() launches (on the engine's stream), for timing kernels without the host's
        launch costs; release it with lib.L.pllm_graph_destroy."""
        L.pllm_set_stream(self.stream)
        if L.pllm_graph_begin() != 0:
            check("graph begin")
        enqueue()
        g = L.pllm_graph_end()
        check("graph capture")
        return g

    def launch_step(self):
        """Enqueue one step for the token and position already in device memory (no copies, no wait)."""
        L.pllm_set_stream(self.stream)
        if self.graphs:
            if not self.graph:
                self.capture()
            L.pllm_graph_launch(self.graph)
        else:
            self._enqueue_step(True)

    # ---- the engine's calls (forward/engine.ts:549-702)
    def forward(self, token, pos, need_logits=True):
        """One token at pos; the logits (a copy) when asked for."""
        c = self.cfg
        if self.batch > 1:
            raise ValueError("a batch engine steps with forward_batch")
        if not (0 <= pos < c.seq_len and 0 <= token < c.vocab):
            raise ValueError(f"token {token} at {pos}: out of range")
        L.pllm_set_stream(self.stream)
        self.tp_host.array[0], self.tp_host.array[1] = token, pos
        L.pllm_h2d(self.B["tp"].ptr, self.tp_host.ptr, 8)
        self.launch_step()
        if need_logits:
            L.pllm_d2h(self.logits_host.ptr, self.B["logits"].ptr, self.shard.vocab * 4)
        L.pllm_sync()
        check("forward")
        return self.logits_host.array.copy() if need_logits else None

    def next_token(self, token, pos, temperature=0.0, topp=0.9, topk=0, minp=0.0, random=None):
        """One decode step: the token at pos in, the next token out, chosen on the device where forward() copies the
        vocabulary's logits back: 8 bytes to the device (and the random number's 8), 4 back.
        temperature 0: the most probable (argmax, sample.ts:6-10); else drawn (sample.ts:248-337) from
        softmax(logits / temperature) by random in [0, 1) (the caller's generator's, as the reference's engine hands
        Python's), of the topk most probable (0: all), then their nucleus (0 < topp < 1), then without those below minp
        times the most probable. -1: the logits' largest is no finite number.
        With tensor parallelism (every rank calls it with the same token and position): greedy only; each rank's
        vocab slice gives its largest as a key (pllm_argmax_key_dev), the ranks' keys meet in an NCCL max, and every
        rank gets the same token, 4 bytes back (the logits stay on the devices)."""
        c = self.cfg
        if self.xg and temperature > 0:
            raise NotImplementedError("with tensor parallelism next_token is greedy: draw from the gathered logits")
        if not (0 <= pos < c.seq_len and 0 <= token < c.vocab):
            raise ValueError(f"token {token} at {pos}: out of range")
        if temperature > 0 and not (random is not None and 0.0 <= random < 1.0):
            raise ValueError("a draw needs a random number in [0, 1)")
        L.pllm_set_stream(self.stream)
        self.tp_host.array[0], self.tp_host.array[1] = token, pos
        L.pllm_h2d(self.B["tp"].ptr, self.tp_host.ptr, 8)
        self.launch_step()
        if temperature > 0:
            if "probs" not in self.B:
                self.B["probs"], self.B["index"] = Buffer(4 * c.vocab), Buffer(4 * c.vocab)
                self.B["random"], self.random_host = Buffer(8), Pinned(1, np.float64)
            self.random_host.array[0] = random
            L.pllm_h2d(self.B["random"].ptr, self.random_host.ptr, 8)
            L.pllm_sample_dev(self.B["next"].ptr, self.B["logits"].ptr, c.vocab, temperature, topp,
                              self.B["random"].ptr, self.B["probs"].ptr, self.B["index"].ptr, topk, minp)
        elif self.xg:
            sh = self.shard
            if "key" not in self.B:
                self.B["key"] = Buffer(8)
                self.xg.collectives(self.device)
            L.pllm_argmax_key_dev(self.B["key"].ptr, self.B["logits"].ptr, sh.vocab, sh.rank * sh.vocab,
                                  self.B["amx"].ptr)
            self.xg.all_reduce(self.B["key"].ptr, 1, "i8", self.stream, op="max")
            L.pllm_key_token_dev(self.B["next"].ptr, self.B["key"].ptr)
        else:
            L.pllm_argmax_dev(self.B["next"].ptr, self.B["logits"].ptr, c.vocab, self.B["amx"].ptr)
        L.pllm_d2h(self.next_host.ptr, self.B["next"].ptr, 4)
        L.pllm_sync()
        check("next_token")
        return int(self.next_host.array[0])

    def _batch_in(self, tokens, positions):
        c, nb = self.cfg, self.batch
        tokens, positions = np.asarray(tokens, np.int64), np.asarray(positions, np.int64)
        if tokens.shape != (nb,) or positions.shape != (nb,):
            raise ValueError(f"a step of the batch takes {nb} tokens and {nb} positions")
        if (positions < 0).any() or (positions >= c.seq_len).any() or (tokens < 0).any() or (tokens >= c.vocab).any():
            raise ValueError("a token or a position out of range")
        L.pllm_set_stream(self.stream)
        self.tp_host.array[:nb] = tokens
        self.tp_host.array[nb:] = positions
        L.pllm_h2d(self.B["tp"].ptr, self.tp_host.ptr, 8 * nb)

    def forward_batch(self, tokens, positions, need_logits=True):
        """One step of the batch: sequence i's token at its position (each sequence its own cache); the logits, a
        row a sequence (a copy), when asked for."""
        if self.batch < 2:
            raise ValueError("forward_batch is the batch engine's step (Engine(batch=B), B > 1)")
        self._batch_in(tokens, positions)
        self.launch_step()
        n = self.batch * self.shard.vocab
        if need_logits:
            L.pllm_d2h(self.logits_host.ptr, self.B["logits"].ptr, n * 4)
        L.pllm_sync()
        check("forward_batch")
        return self.logits_host.array[:n].reshape(self.batch, -1).copy() if need_logits else None

    def next_tokens(self, tokens, positions):
        """The batch's greedy step: the next token of every sequence (argmax on the device, sample.ts:6-10), 8 bytes
        a sequence in and 4 back."""
        if self.batch < 2:
            raise ValueError("next_tokens is the batch engine's step (Engine(batch=B), B > 1)")
        self._batch_in(tokens, positions)
        self.launch_step()
        V = self.shard.vocab
        for i in range(self.batch):
            L.pllm_argmax_dev(self.B["nexts"].ptr + 4 * i, self.B["logits"].ptr + 4 * i * V, V, self.B["amx"].ptr)
        L.pllm_d2h(self.next_host.ptr, self.B["nexts"].ptr, 4 * self.batch)
        L.pllm_sync()
        check("next_tokens")
        return self.next_host.array[:self.batch].copy()

    def forward_many(self, tokens, pos):
        """Tokens at pos, pos + 1, ...: each computed as it would be alone (engine.ts:590); the last one's logits.
        Where the shapes suit the tensor-core prefill (can_prefill) the tokens go through it at once, else one by
        one through the decode step."""
        if len(tokens) > 1 and self.can_prefill():
            return self.prefill(tokens, pos)
        out = None
        for t, token in enumerate(tokens):
            out = self.forward(int(token), pos + t, need_logits=(t == len(tokens) - 1))
        return out

    # ---- prefill: many tokens at once on the tensor cores
    def can_prefill(self):
        """The tensor-core prefill's shapes: products with K and rows in whole 128s, a float16 cache."""
        c, sh = self.cfg, self.shard
        return (not self.exact and not self.hybrid and self.fmt == F_Q8 and c.half_kv and c.head_size <= 128 and all(
            v % 128 == 0 for v in (c.dim, sh.qdim, sh.hidden, self.rows_qkv)))

    def _prefill_buffers(self, M):
        c, sh = self.cfg, self.shard
        P = getattr(self, "P", None)
        if P is None:  # the matrices' scales transposed once (the tensor-core product reads them by column)
            P = {"M": 0}
            B = self.B
            for w, rows, cols in (("sqkv", self.rows_qkv, c.dim), ("so", c.dim, sh.qdim), ("s13", 2 * sh.hidden, c.dim),
                                  ("s2", c.dim, sh.hidden)):
                t = Buffer(B[w].nbytes)
                per = rows * (cols // 32) * 4
                for l in range(c.layers):
                    L.pllm_transpose_scales(t.ptr + l * per, B[w].ptr + l * per, rows, cols // 32)
                P["t" + w] = t
            self.P = P
        if P["M"] < M:
            for k in ("X", "QKV", "ATT", "HB", "XQ", "XS", "TOK", "PART"):
                if k in P:
                    P[k].free()
            wide = max(c.dim, sh.qdim, sh.hidden, self.rows_qkv)
            P["X"], P["QKV"] = Buffer(M * c.dim * 4), Buffer(M * self.rows_qkv * 4)
            P["ATT"], P["HB"] = Buffer(M * sh.qdim * 4), Buffer(M * sh.hidden * 4)
            P["XQ"], P["XS"], P["TOK"] = Buffer(M * wide), Buffer(M * wide // 8), Buffer(M * 4)
            if self.xg:  # the row-parallel products' partials, reduced over the ranks
                P["PART"] = Buffer(M * c.dim * 4)
            P["M"] = M
        return P

    def prefill(self, tokens, pos=0, need_logits=True, seq=0):
        """tokens at positions pos.. through every layer at once (the products on the tensor cores, pllm_gemm_q8; the
        attention of all of them at once, pllm_attention_prefill), the cache filled for them; the last token's logits
        (the decode step's classifier). seq: a batch engine's sequence whose cache they fill.
        With tensor parallelism (every rank calls it with the same tokens): each rank's products over its shares, its
        heads' attention and cache; wo and w2 make partials of every row, summed over the ranks by an NCCL all-reduce
        (pllm.tp.Exchange.all_reduce) and added to the residual; the logits returned are the rank's vocab slice."""
        c, sh, B = self.cfg, self.shard, self.B
        M = len(tokens)
        if not 0 <= seq < self.batch:
            raise ValueError(f"sequence {seq} of {self.batch}")
        if not (M >= 1 and 0 <= pos and pos + M <= c.seq_len):
            raise ValueError(f"{M} tokens at {pos}: out of range")
        if not self.can_prefill():
            raise ValueError("shapes the tensor-core prefill does not take")
        L.pllm_set_stream(self.stream)
        P = self._prefill_buffers(M)
        P["TOK"].upload(np.asarray(tokens, np.int32))
        E = 2
        X, QKV, ATT, HB, XQ, XS = (P[k].ptr for k in ("X", "QKV", "ATT", "HB", "XQ", "XS"))
        PART = P["PART"].ptr if self.xg else 0
        if self.xg:
            self.xg.collectives(self.device)
        L.pllm_embed_q8(X, B["emb"].ptr, B["emb_s"].ptr, P["TOK"].ptr, 0, c.dim, M, c.dim)
        bias = self.bias
        for l in range(c.layers):
            wqkv = B["wqkv"].ptr + l * self.rows_qkv * c.dim
            tqkv = P["tsqkv"].ptr + l * self.rows_qkv * (c.dim // 32) * 4
            L.pllm_norm_quantize_rows(XQ, XS, X, c.dim, B["att_norm"].ptr + l * c.dim * 4, c.eps, c.dim, M, bias)
            L.pllm_gemm_q8(QKV, self.rows_qkv, XQ, XS, wqkv, tqkv, M, self.rows_qkv, c.dim, self.rows_qkv, 0, 0)
            kc = B["kc"].ptr + (l * self.batch + seq) * c.seq_len * sh.kvdim * E
            vc = B["vc"].ptr + (l * self.batch + seq) * c.seq_len * sh.kvdim * E
            qn = B["q_norm"].ptr + l * c.head_size * 4 if c.qk_norm else 0
            kn = B["k_norm"].ptr + l * c.head_size * 4 if c.qk_norm else 0
            L.pllm_qk_rope_cache_rows(QKV, self.rows_qkv, qn, kn, B["cos_t"].ptr, B["sin_t"].ptr, pos, M, kc, vc,
                                      sh.heads, sh.kv_heads, c.head_size, 0, c.eps, 1, B["bad"].ptr)
            L.pllm_attention_prefill(ATT, sh.qdim, QKV, self.rows_qkv, kc, vc, pos, M, sh.heads, sh.kv_heads,
                                     c.head_size)
            L.pllm_norm_quantize_rows(XQ, XS, ATT, sh.qdim, 0, c.eps, sh.qdim, M, bias)
            if self.xg:  # row-parallel: this rank's partial over its heads' groups, summed over the ranks, then added
                L.pllm_gemm_q8(PART, c.dim, XQ, XS, B["wo"].ptr + l * c.dim * sh.qdim,
                               P["tso"].ptr + l * c.dim * (sh.qdim // 32) * 4, M, c.dim, sh.qdim, c.dim, 0, 0)
                self.xg.all_reduce(PART, M * c.dim, "f4", self.stream)
                L.add_inplace(X, PART, M * c.dim)
            else:
                L.pllm_gemm_q8(X, c.dim, XQ, XS, B["wo"].ptr + l * c.dim * sh.qdim,
                               P["tso"].ptr + l * c.dim * (sh.qdim // 32) * 4, M, c.dim, sh.qdim, c.dim, 1, 0)
            L.pllm_norm_quantize_rows(XQ, XS, X, c.dim, B["ffn_norm"].ptr + l * c.dim * 4, c.eps, c.dim, M, bias)
            L.pllm_gemm_q8(HB, sh.hidden, XQ, XS, B["w13"].ptr + l * 2 * sh.hidden * c.dim,
                           P["ts13"].ptr + l * 2 * sh.hidden * (c.dim // 32) * 4, M, sh.hidden, c.dim,
                           2 * sh.hidden, 2, sh.hidden)
            L.pllm_norm_quantize_rows(XQ, XS, HB, sh.hidden, 0, c.eps, sh.hidden, M, bias)
            if self.xg:  # row-parallel over this rank's hidden rows
                L.pllm_gemm_q8(PART, c.dim, XQ, XS, B["w2"].ptr + l * c.dim * sh.hidden,
                               P["ts2"].ptr + l * c.dim * (sh.hidden // 32) * 4, M, c.dim, sh.hidden, c.dim, 0, 0)
                self.xg.all_reduce(PART, M * c.dim, "f4", self.stream)
                L.add_inplace(X, PART, M * c.dim)
            else:
                L.pllm_gemm_q8(X, c.dim, XQ, XS, B["w2"].ptr + l * c.dim * sh.hidden,
                               P["ts2"].ptr + l * c.dim * (sh.hidden // 32) * 4, M, c.dim, sh.hidden, c.dim, 1, 0)
        if not need_logits:
            L.pllm_sync()
            check("prefill")
            return None
        x_row, logits_row = B["x"].ptr + seq * c.dim * 4, B["logits"].ptr + seq * sh.vocab * 4
        L.pllm_d2d(x_row, X + (M - 1) * c.dim * 4, c.dim * 4)
        self._gemv(logits_row, B["cls"].ptr, B["cls_s"].ptr, sh.vocab, c.dim, x_row, B["final_norm"].ptr,
                   PRO_RMS, EPI_STORE, pdl=False)
        L.pllm_d2h(self.logits_host.ptr, logits_row, sh.vocab * 4)
        L.pllm_sync()
        check("prefill")
        return self.logits_host.array[:sh.vocab].copy()

    def close(self):
        if self.graph:
            L.pllm_graph_destroy(self.graph)
            self.graph = 0
        for b in list(self.B.values()) + [v for k, v in getattr(self, "P", {}).items() if k != "M"]:
            if b is not None:
                b.free()
