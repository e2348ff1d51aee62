"""The LFM2-shaped hybrid (short-convolution layers among grouped-query attention layers,
Config(kinds=...)) on the device engine, one sequence and a batch, against a forward made of the oracle's kernels in
the reference engine's order (test infrastructure: forward/engine.ts run(); an attention layer as oracle/or_forward
runs it; a convolution layer as forward/convolution.ts:51-60 does: win . quantize_x(RMSNorm(x)), the rows moved up
one, stateful.ts:70-86's short_conv, x += wout . quantize_x(it); the gated FFN). The line is the int8 engine's
(tests/test_gpu_forward.py: 2e-2 of the largest logit and relative distance, the same greedy token but for one
position in twenty)."""
from dataclasses import replace

import numpy as np
import pytest

import oracle as O
from pllm.forward import LFM2_350M, Config, Engine

from test_gpu_forward import check_logits

pytestmark = pytest.mark.gpu

SMALL_LFM2 = Config(dim=256, hidden=512, layers=6, heads=8, kv_heads=4, head_size=32, vocab=700, seq_len=64,
                    qk_norm=True, rope_theta=1e6, eps=1e-5, kinds="ccacac", taps=3)


class OracleLfm2:
    """One sequence of the hybrid through the oracle's kernels (its own cache and convolution rows)."""

    def __init__(self, cfg, W):
        c, Lr, d, h = cfg, cfg.layers, cfg.dim, cfg.hidden
        shapes = {"wq": (Lr, c.qdim, d), "sq": (Lr, c.qdim, d // 32), "wk": (Lr, c.kvdim, d), "sk": (Lr, c.kvdim, d // 32),
                  "wv": (Lr, c.kvdim, d), "sv": (Lr, c.kvdim, d // 32), "wo": (Lr, d, c.qdim),
                  "so": (Lr, d, c.qdim // 32), "w1": (Lr, h, d), "s1": (Lr, h, d // 32), "w3": (Lr, h, d),
                  "s3": (Lr, h, d // 32), "w2": (Lr, d, h), "s2": (Lr, d, h // 32), "emb": (c.vocab, d),
                  "emb_s": (c.vocab, d // 32), "cls": (c.vocab, d), "cls_s": (c.vocab, d // 32), "att_norm": (Lr, d),
                  "ffn_norm": (Lr, d), "q_norm": (Lr, c.head_size), "k_norm": (Lr, c.head_size),
                  "cos_t": (c.seq_len, c.head_size // 2), "sin_t": (c.seq_len, c.head_size // 2)}
        W = {k: (v.reshape(shapes[k]) if k in shapes and v is not None else v) for k, v in W.items()}
        self.c, self.W = cfg, W
        self.kc = np.zeros((cfg.layers, cfg.seq_len, cfg.kvdim), np.uint16)
        self.vc = np.zeros((cfg.layers, cfg.seq_len, cfg.kvdim), np.uint16)
        self.rows = np.zeros((cfg.layers, cfg.taps, cfg.dim), np.float32)

    def prod(self, x, w, s):
        xq, xs = O.quantize_x(x, 64 if self.c.relaxed else 0)
        return O.matmul_q8r(xq, xs, w, s) if self.c.relaxed else O.matmul_q8(xq, xs, w, s)

    def forward(self, tok, pos):
        c, W = self.c, self.W
        d, hs = c.dim, c.head_size
        x = (W["emb"][tok].astype(np.float32) * np.repeat(W["emb_s"][tok], 32)).astype(np.float32)
        if pos == 0:
            self.rows[:] = 0.0
        for l in range(c.layers):
            xb = O.rmsnorm(x, W["att_norm"][l], c.eps)
            if c.kind(l) == "c":
                mixed = self.prod(xb, W["win"][l], W["swin"][l])
                rows = self.rows[l].copy()
                rows[:-1] = rows[1:]
                out, self.rows[l] = O.short_conv(W["taps"][l], rows, mixed)
                x = O.add_inplace(x, self.prod(out, W["wout"][l], W["swout"][l]))
            else:
                q = self.prod(xb, W["wq"][l], W["sq"][l])
                k = self.prod(xb, W["wk"][l], W["sk"][l])
                v = self.prod(xb, W["wv"][l], W["sv"][l])
                if c.qk_norm:
                    q = np.concatenate([O.rmsnorm(q[h * hs:(h + 1) * hs], W["q_norm"][l], c.eps) for h in range(c.heads)])
                    k = np.concatenate([O.rmsnorm(k[h * hs:(h + 1) * hs], W["k_norm"][l], c.eps)
                                        for h in range(c.kv_heads)])
                q = O.rope(q, W["cos_t"][pos], W["sin_t"][pos], c.heads, hs)
                k = O.rope(k, W["cos_t"][pos], W["sin_t"][pos], c.kv_heads, hs)
                self.kc[l, pos], self.vc[l, pos] = O.to_f16(k)[0], O.to_f16(v)[0]
                att, _ = O.attention(q, self.kc[l, :pos + 1], self.vc[l, :pos + 1], pos, c.heads, c.kv_heads, hs,
                                     half=True)
                x = O.add_inplace(x, self.prod(att, W["wo"][l], W["so"][l]))
            xb = O.rmsnorm(x, W["ffn_norm"][l], c.eps)
            hb = O.swiglu(self.prod(xb, W["w1"][l], W["s1"][l]), self.prod(xb, W["w3"][l], W["s3"][l]))
            x = O.add_inplace(x, self.prod(hb, W["w2"][l], W["s2"][l]))
        return self.prod(O.rmsnorm(x, W["final_norm"], c.eps), W["cls"], W["cls_s"])


def run(cfg, eng, W, steps, nb, seed, flips=None):
    oracles = [OracleLfm2(cfg, W) for _ in range(nb)]
    rng = np.random.default_rng(seed)
    agree = 0
    for step in range(steps):
        toks = rng.integers(0, cfg.vocab, nb)
        poss = np.array([step + 2 * i for i in range(nb)])
        got = eng.forward_batch(toks, poss) if nb > 1 else eng.forward(int(toks[0]), int(poss[0]))[None, :]
        for i in range(nb):
            want = oracles[i].forward(int(toks[i]), int(poss[i]))
            check_logits(got[i], want, (step, i), (0.0, 0.0))
            agree += int(np.argmax(got[i]) == np.argmax(want))
    allowed = max(1, steps * nb // 20) if flips is None else flips
    assert agree >= steps * nb - allowed, agree


@pytest.mark.parametrize("nb", [1, 8])
def test_small_hybrid_matches_oracle(nb):
    eng = Engine(SMALL_LFM2, seed=4, batch=nb)
    W = eng.host_weights()
    run(SMALL_LFM2, eng, W, 16, nb, seed=nb)
    eng.close()


def test_lfm2_350m_widths_match_oracle():
    """configs[2]'s widths (1024 hidden, 16 layers: 10 convolution, 6 attention, 4608 FFN, 65536 vocab)."""
    cfg = replace(LFM2_350M, seq_len=16)
    eng = Engine(cfg, seed=1)
    W = eng.host_weights()
    run(cfg, eng, W, 4, 1, seed=3)
    eng.close()


def test_position_zero_clears_the_rows():
    """A sequence that starts again at position 0 does not see the rows of the one before (clear())."""
    cfg = SMALL_LFM2
    a, b = Engine(cfg, seed=5), Engine(cfg, seed=5)
    for pos, tok in enumerate([3, 9, 27, 81]):
        a.forward(tok, pos)
    for pos, tok in enumerate([5, 6]):
        assert np.array_equal(a.forward(tok, pos), b.forward(tok, pos))
    a.close()
    b.close()
