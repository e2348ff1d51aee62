"""Prefill on the GPU: many tokens through every layer at once (Engine.prefill: the products on the tensor cores,
the attention of all of them at once), against the oracle's forward taken token by token (the reference's engine
runs a prompt as a sequence of decode steps: engine.ts:590) and against the device's own decode step.

  - the prefill attention kernel against the oracle's attention of each token over the positions before it (the
    same float16 cache): float32 rounding only (1e-4 relative);
  - the model's last-token logits after a prompt, and the logits of decode steps that follow it (the cache the
    prefill wrote): the model-level line of the other forward tests (2e-2 of the largest logit, relative distance
    2e-2), the greedy token the oracle's."""
from dataclasses import replace

import numpy as np
import pytest

import oracle as O
from pllm.device import Buffer, init
from pllm.forward import QWEN3_8B, Config, Engine, synthetic_host_weights
from pllm.lib import L, check

from test_gpu_forward import oracle_arrays, oracle_config

pytestmark = pytest.mark.gpu

SMALL = Config(dim=256, hidden=512, layers=2, heads=8, kv_heads=2, head_size=64, vocab=1000, seq_len=300,
               qk_norm=True, rope_theta=1e6, eps=1e-6)


def close(got, want, what):
    rel = float(np.sqrt(((got.astype(np.float64) - want) ** 2).sum() / (want.astype(np.float64) ** 2).sum()))
    peak = float(np.abs(got - want).max() / np.abs(want).max())
    print(f"{what}: relative {rel:.2e}, peak {peak:.2e}, argmax {np.argmax(got)} / {np.argmax(want)}")
    assert rel <= 2e-2 and peak <= 2e-2, (what, rel, peak)


@pytest.mark.parametrize("nh,nkv,hs", [(8, 2, 64), (32, 8, 128), (6, 6, 48), (16, 2, 128)])
@pytest.mark.parametrize("p0,count", [(0, 1), (0, 77), (40, 130), (5, 64)])
def test_attention_prefill_kernel(nh, nkv, hs, p0, count):
    init(0)
    L.pllm_set_stream(0)
    rng = np.random.default_rng(nh + p0 + count)
    npos = p0 + count
    kc = O.to_f16(rng.normal(0, 1, (npos, nkv * hs)).astype(np.float32))[0].reshape(npos, nkv * hs)
    vc = O.to_f16(rng.normal(0, 1, (npos, nkv * hs)).astype(np.float32))[0].reshape(npos, nkv * hs)
    stride = (nh + 2 * nkv) * hs + 16  # rows of a q/k/v product (and some room)
    qkv = rng.normal(0, 1, (count, stride)).astype(np.float32)
    bufs = [Buffer.of(a) for a in (kc, vc, qkv)]
    out = Buffer.of(np.full((count, nh * hs + 4), -7, np.float32))
    L.pllm_attention_prefill(out.ptr, nh * hs + 4, bufs[2].ptr, stride, bufs[0].ptr, bufs[1].ptr, p0, count, nh, nkv,
                             hs)
    assert L.pllm_sync() == 0
    check("pllm_attention_prefill")
    got = out.download(np.float32).reshape(count, nh * hs + 4)
    assert np.all(got[:, nh * hs:] == -7)
    for t in range(count):
        want, _ = O.attention(qkv[t, :nh * hs], kc, vc, p0 + t, nh, nkv, hs, half=True)
        np.testing.assert_allclose(got[t, :nh * hs], want, rtol=1e-4, atol=2e-5)
    for b in bufs + [out]:
        b.free()


def oracle_run(cfg, W, tokens, start=0, A=None):
    A = oracle_arrays(cfg, W) if A is None else A
    oc = oracle_config(cfg)
    out = None
    for i, t in enumerate(tokens):
        out = O.forward(oc, A, int(t), start + i)
    return out, A


@pytest.mark.parametrize("relaxed", [False, True])
def test_prefill_then_decode(relaxed):
    cfg = replace(SMALL, relaxed=relaxed)
    W = synthetic_host_weights(cfg, seed=7)
    eng = Engine(cfg, host=W)
    assert eng.can_prefill()
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, cfg.vocab, 45)
    got = eng.prefill(prompt, 0)
    want, A = oracle_run(cfg, W, prompt)
    close(got, want, "prefill of 45 tokens")
    assert np.argmax(got) == np.argmax(want)
    for i, t in enumerate(rng.integers(0, cfg.vocab, 4)):  # decode steps on the cache the prefill wrote
        got = eng.forward(int(t), 45 + i)
        want, _ = oracle_run(cfg, W, [t], 45 + i, A)
        close(got, want, f"decode at {45 + i}")
    more = rng.integers(0, cfg.vocab, 30)  # a second prefill after the decode steps
    got = eng.prefill(more, 49)
    want, _ = oracle_run(cfg, W, more, 49, A)
    close(got, want, "prefill of 30 more tokens at 49")
    assert L.pllm_device_status() == 0
    eng.close()


def test_prefill_equals_token_by_token_at_8b_width():
    """Qwen3-8B's widths, two layers, a 300-token prompt: the prefill against the decode step taken token by token
    on the same device weights (the same model, another order of the float32 sums), then the caches' contents."""
    cfg = replace(QWEN3_8B, layers=2, seq_len=512)
    a, b = Engine(cfg, seed=2), Engine(cfg, seed=2)
    prompt = np.random.default_rng(5).integers(0, cfg.vocab, 300)
    got = a.prefill(prompt, 0)
    want = None
    for i, t in enumerate(prompt):
        want = b.forward(int(t), i, need_logits=(i == len(prompt) - 1))
    close(got, want, "8B-width prefill of 300 tokens")
    # the keys written for the prompt: layer 0's come from the embedding through one product, so only the order of
    # its float32 sums differs (the float16 rounding of a key flips rarely); layer 1's carry layer 0's flips too
    kvdim = cfg.kv_heads * cfg.head_size
    ka = a.B["kc"].download(np.uint16).reshape(cfg.layers, cfg.seq_len, kvdim)[:, :len(prompt)]
    kb = b.B["kc"].download(np.uint16).reshape(cfg.layers, cfg.seq_len, kvdim)[:, :len(prompt)]
    same0 = float(np.mean(ka[0] == kb[0]))
    fa, fb = (O.from_f16(k.reshape(-1)).reshape(k.shape) for k in (ka, kb))
    rel1 = float(np.linalg.norm(fa[1] - fb[1]) / np.linalg.norm(fb[1]))
    print(f"layer 0 keys equal to the bit: {same0:.5f}; layer 1 keys' relative distance {rel1:.2e}")
    assert same0 > 0.995 and rel1 < 2e-2
    a.close()
    b.close()


def test_8b_width_prefill_matches_oracle():
    """Qwen3-8B's widths, two layers, a 64-token prompt through the tensor-core prefill against the oracle's forward
    of the same tokens (the reference kernels' arithmetic, token after token, on the device's weights), at the int8
    engine's line (2e-2 of the largest logit); then two decode steps on the cache the prefill wrote, at the same line."""
    cfg = replace(QWEN3_8B, layers=2, seq_len=96)
    eng = Engine(cfg, seed=4)
    W = eng.host_weights()
    prompt = np.random.default_rng(6).integers(0, cfg.vocab, 64)
    got = eng.prefill(prompt, 0)
    want, A = oracle_run(cfg, W, prompt)
    close(got, want, "8B-width prefill of 64 tokens against the oracle")
    for i, t in enumerate([17, 40001]):
        got = eng.forward(t, 64 + i)
        want, _ = oracle_run(cfg, W, [t], 64 + i, A)
        close(got, want, f"decode at {64 + i} after the prefill")
    eng.close()
