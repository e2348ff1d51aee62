"""The ternary decode product (the bulk-copy pipeline streaming 2-bit codes and float16 group scales, 0.2656 bytes a
weight; configs[4]'s 27B-class widths) against the oracle's matmul_signs (relaxed/signs.ts:28-55, :117; the codes of
kernels/ternary.ts:25-33): every group's integer exact (checked through the oracle's group sums in the bound), the
float32 rows within 8 x groups x 2^-24 x sum |terms|. The registry's calls (matmul_t2 / matmul_t2r on the
interleave's activations) and the forward driver's form (pllm_gemv from float32 activations: quantize_x, interleave
and minus-sums made in the prologue), its residual and SwiGLU epilogues."""
import numpy as np
import pytest

import oracle as O
from pllm.device import Buffer, init
from pllm.lib import L, check

from test_gpu_kernels import EPS

pytestmark = pytest.mark.gpu

_alive = []


@pytest.fixture(scope="module", autouse=True)
def device():
    init(0)
    L.pllm_set_stream(0)
    yield
    L.pllm_device_sync()


@pytest.fixture(autouse=True)
def keep_buffers():
    yield
    L.pllm_device_sync()
    _alive.clear()


def dev(a):
    b = Buffer.of(np.ascontiguousarray(a))
    _alive.append(b)
    return b


def ternary(rng, rows, k):
    """codes (w + 1) four to a byte (weight j at bits 2 (j & 3) of byte j / 4) and a float16 scale a group of 128."""
    w = rng.integers(-1, 2, (rows, k)).astype(np.int8)
    codes = (w + 1).astype(np.uint8).reshape(rows, k // 4, 4)
    packed = (codes[:, :, 0] | (codes[:, :, 1] << 2) | (codes[:, :, 2] << 4) | (codes[:, :, 3] << 6)).astype(np.uint8)
    scales = rng.normal(0.02, 0.002, (rows, k // 128)).astype(np.float16).view(np.uint16)
    return packed, scales


def bound(il, ext, packed, scales, k):
    G = O.group_sums_signs(il, ext, packed, k).astype(np.float64)  # whole sums a group of 32
    d = np.repeat(scales.view(np.float16).astype(np.float64), 4, axis=1)
    xs = ext[: k // 32].astype(np.float64)
    return 8 * (k // 32) * EPS * (np.abs(G) * xs[None, :] * d).sum(axis=1) + 1e-30


@pytest.mark.parametrize("rows,k", [(512, 5120), (300, 4096), (128, 21504)])
@pytest.mark.parametrize("fn", ["matmul_t2", "matmul_t2r"])
def test_registry_product_is_the_oracles(rows, k, fn):
    rng = np.random.default_rng(rows + k)
    packed, scales = ternary(rng, rows, k)
    xq, xs = O.quantize_x(rng.normal(0, 1, k).astype(np.float32), 0)
    il, ext = O.interleave(xq, xs)
    want = O.matmul_signs(il, ext, packed, scales, k)
    out = dev(np.full(rows + 8, -7, np.float32))
    getattr(L, fn)(out.ptr, dev(il).ptr, dev(ext).ptr, dev(packed).ptr, dev(scales).ptr, k, 0, rows, 3)
    check(fn)
    got = out.download(np.float32)
    assert np.all(np.abs(got[:rows].astype(np.float64) - want) <= bound(il, ext, packed, scales, k))
    assert np.all(got[rows:] == -7)


@pytest.mark.parametrize("epi", [0, 1, 2], ids=["store", "add", "swiglu"])
def test_fused_form_is_the_oracles(epi):
    """pllm_gemv with ternary weights from float32 activations (pro 2: quantize_x; the interleave and minus-sums in
    the prologue) against quantize_x, interleave and matmul_signs on the CPU."""
    rng = np.random.default_rng(epi)
    rows, k = 1024, 5120
    total = 2 * rows if epi == 2 else rows
    packed, scales = ternary(rng, total, k)
    x = rng.normal(0, 1, k).astype(np.float32)
    base = rng.normal(0, 1, rows).astype(np.float32)
    out = dev(base)
    L.pllm_gemv(out.ptr, 0, 0, 0, 0, 0, dev(x).ptr, 0, 0, 1e-6, 0, dev(packed).ptr, dev(scales).ptr, 2, k, 0, rows, 1,
                2, epi, rows if epi == 2 else 0, 0)
    check("pllm_gemv ternary")
    got = out.download(np.float32).astype(np.float64)
    xq, xs = O.quantize_x(x, 0)
    il, ext = O.interleave(xq, xs)
    h = O.matmul_signs(il, ext, packed, scales, k).astype(np.float64)
    b = bound(il, ext, packed, scales, k)
    if epi == 0:
        assert np.all(np.abs(got - h) <= b)
    elif epi == 1:
        assert np.all(np.abs(got - (base + h[:rows])) <= b + 1e-6 * np.abs(base))
    else:
        h1, h3 = h[:rows], h[rows:]
        want = h1 / (1 + np.exp(-h1)) * h3
        assert np.allclose(got, want, rtol=1e-4, atol=1e-4 * np.abs(want).max())


def widened(cfg, W):
    """The ternary engine's host weights as the oracle's int8 arrays (widen_ternary: the same integers)."""
    from pllm.forward import widen_ternary
    from test_gpu_forward import oracle_arrays
    V = dict(W)
    for m in ("q", "k", "v", "o", "1", "2", "3"):
        V["w" + m], V["s" + m] = widen_ternary(W["w" + m], W["s" + m])
    V["cls"], V["cls_s"] = widen_ternary(W["cls"], W["cls_s"])
    return oracle_arrays(cfg, V)


@pytest.mark.parametrize("which", ["small", "27b-widths"])
def test_ternary_engine_matches_oracle(which):
    """The engine on packed ternary matrices (Config(weights="t2"): every product the ternary bulk-copy form, 0.2656
    bytes a weight) against the oracle's forward on the widened weights, at the line of the int8 engine (2e-2 of the
    largest logit, relative distance 2e-2); configs[4]'s widths at two layers."""
    from dataclasses import replace

    from pllm.forward import TERNARY_27B, Config, Engine, synthetic_host_weights
    from test_gpu_forward import check_logits, oracle_config
    if which == "small":
        cfg = Config(dim=1024, hidden=2048, layers=3, heads=8, kv_heads=4, head_size=128, vocab=2048, seq_len=64,
                     weights="t2")
        W = synthetic_host_weights(cfg, seed=4)
        eng = Engine(cfg, host=W)
        A = widened(cfg, W)
        steps = 12
    else:
        cfg = replace(TERNARY_27B, layers=2, seq_len=16)
        eng = Engine(cfg, seed=1)
        A = eng.host_weights()
        from test_gpu_forward import oracle_arrays
        A = oracle_arrays(cfg, A)
        steps = 3
    oc = oracle_config(cfg)
    agree = 0
    for pos, tok in enumerate(np.random.default_rng(2).integers(0, cfg.vocab, steps)):
        want = O.forward(oc, A, int(tok), pos)
        got = eng.forward(int(tok), pos)
        check_logits(got, want, pos, (0.0, 0.0))
        agree += int(np.argmax(got) == np.argmax(want))
    assert agree >= steps - 1
    eng.close()
