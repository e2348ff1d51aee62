"""The reference-order step (pllm_exact_*: every float32 operation in the reference kernels' own order, the
exponential the Cephes expf the reference's table-free exp follows) against the oracle, to the bit: each kernel on
seeded inputs, then whole forward passes, the benchmark's Qwen3-8B-shaped configuration at 2 and 36 layers among
them. Being the oracle's numbers to the bit, the logits meet the north star's line (max |difference| at most 1e-3 of
the largest |logit|) with nothing to spare: the difference is zero."""
from dataclasses import replace

import numpy as np
import pytest

import oracle as O
from pllm.device import Buffer, init
from pllm.forward import QWEN3_8B, Config, Engine, synthetic_host_weights
from pllm.lib import L, check

from test_gpu_forward import STORIES, SMALL_QWEN3, oracle_arrays, oracle_config

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


def empty(nbytes):
    b = Buffer(nbytes)
    _alive.append(b)
    return b


def same_bits(got, want):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    return np.array_equal(got.view(np.int32), want.view(np.int32))


@pytest.mark.parametrize("n", [288, 4096, 12288])
@pytest.mark.parametrize("bias", [0, 64])
@pytest.mark.parametrize("mode", [0, 1, 2])
def test_prepare_is_the_oracles(n, bias, mode):
    rng = np.random.default_rng(n + bias + mode)
    x = (rng.normal(0, 1, 2 * n if mode == 2 else n) * rng.uniform(0.1, 10)).astype(np.float32)
    w = rng.normal(1, 0.1, n).astype(np.float32)
    if mode == 0:
        y = x
    elif mode == 1:
        y = O.rmsnorm(x, w, 1e-6)
    else:
        y = O.swiglu(x[:n], x[n:])
    want_q, want_s = O.quantize_x(y, bias)
    xq, xs, out = empty(n), empty(n // 8), empty(4 * n)
    L.pllm_exact_prepare(xq.ptr, xs.ptr, out.ptr, dev(x).ptr, dev(w).ptr if mode == 1 else 0, n, 1e-6, bias, mode)
    check("pllm_exact_prepare")
    assert same_bits(out.download(np.float32), y)
    assert np.array_equal(xq.download(np.uint8), want_q)
    assert same_bits(xs.download(np.float32), want_s)


@pytest.mark.parametrize("k,rows", [(288, 97), (1024, 1024), (4096, 640), (12288, 256), (800, 33)])
@pytest.mark.parametrize("relaxed", [False, True])
def test_product_is_the_oracles(k, rows, relaxed):
    rng = np.random.default_rng(k * 3 + rows + relaxed)
    w = rng.integers(-127, 128, (rows, k)).astype(np.int8)
    w[0, :64] = -128  # the format's extreme weight
    ws = rng.uniform(0.001, 0.02, (rows, k // 32)).astype(np.float32)
    ws[1, :3] = 0.0
    x = rng.normal(0, 1, k).astype(np.float32)
    bias = 64 if relaxed else 0
    xq, xs = O.quantize_x(x, bias)
    want = O.matmul_q8r(xq, xs, w, ws) if relaxed else O.matmul_q8(xq, xs, w, ws)
    out = empty(4 * rows)
    L.pllm_exact_product(out.ptr, 0, dev(xq).ptr, dev(xs).ptr, dev(w).ptr, dev(ws).ptr, k, rows, int(relaxed))
    check("pllm_exact_product")
    assert same_bits(out.download(np.float32), want)
    # the residual form: x + row, in place
    base = rng.normal(0, 1, rows).astype(np.float32)
    acc = dev(base)
    L.pllm_exact_product(acc.ptr, acc.ptr, dev(xq).ptr, dev(xs).ptr, dev(w).ptr, dev(ws).ptr, k, rows, int(relaxed))
    check("pllm_exact_product add")
    assert same_bits(acc.download(np.float32), base + want)


@pytest.mark.parametrize("nh,nkv,hs", [(32, 8, 128), (6, 6, 48), (16, 2, 64)])
@pytest.mark.parametrize("half", [True, False])
@pytest.mark.parametrize("pos", [0, 1, 2, 3, 4, 130, 511, 512, 700, 1200])
def test_attention_is_the_oracles(nh, nkv, hs, half, pos):
    rng = np.random.default_rng(nh + hs + pos + half)
    cap_pos = 1280
    q = rng.normal(0, 1, nh * hs).astype(np.float32)
    kv = rng.normal(0, 1, (2, cap_pos, nkv * hs)).astype(np.float32)
    if half:
        kc, vc = (O.to_f16(kv[i].reshape(-1))[0].reshape(cap_pos, -1) for i in range(2))
    else:
        kc, vc = kv[0], kv[1]
    want, _ = O.attention(q, kc[:pos + 1], vc[:pos + 1], pos, nh, nkv, hs, half=half)
    out, att = empty(4 * nh * hs), empty(4 * nh * cap_pos)
    L.pllm_exact_attention(out.ptr, dev(q).ptr, dev(kc).ptr, dev(vc).ptr, att.ptr, 0, pos, cap_pos, nh, nkv, hs,
                           int(half), 0.0)
    check("pllm_exact_attention")
    assert same_bits(out.download(np.float32), want)
    # the position read from device memory (a recorded step's form)
    pd = dev(np.array([pos], np.int32))
    out2 = empty(4 * nh * hs)
    L.pllm_exact_attention(out2.ptr, dev(q).ptr, dev(kc).ptr, dev(vc).ptr, att.ptr, pd.ptr, 0, cap_pos, nh, nkv, hs,
                           int(half), 0.0)
    check("pllm_exact_attention pos_dev")
    assert same_bits(out2.download(np.float32), want)


@pytest.mark.parametrize("pos", [5, 67])
def test_capped_attention_is_the_oracles(pos):
    nh, nkv, hs = 8, 2, 64
    rng = np.random.default_rng(pos)
    q = rng.normal(0, 3, nh * hs).astype(np.float32)
    kc = rng.normal(0, 3, (pos + 1, nkv * hs)).astype(np.float32)
    vc = rng.normal(0, 1, (pos + 1, nkv * hs)).astype(np.float32)
    want, _ = O.attention(q, kc, vc, pos, nh, nkv, hs, cap=30.0)
    out, att = empty(4 * nh * hs), empty(4 * nh * (pos + 1))
    L.pllm_exact_attention(out.ptr, dev(q).ptr, dev(kc).ptr, dev(vc).ptr, att.ptr, 0, pos, pos + 1, nh, nkv, hs, 0,
                           30.0)
    check("pllm_exact_attention capped")
    assert same_bits(out.download(np.float32), want)


def test_qk_rope_cache_is_the_oracles():
    nh, nkv, hs, pos, cap_pos = 32, 8, 128, 37, 64
    rng = np.random.default_rng(11)
    qkv = rng.normal(0, 1, (nh + 2 * nkv) * hs).astype(np.float32)
    qn, kn = rng.normal(1, 0.1, hs).astype(np.float32), rng.normal(1, 0.1, hs).astype(np.float32)
    cfg = replace(QWEN3_8B, seq_len=cap_pos)
    from pllm.forward import rope_tables
    cos, sin = rope_tables(cfg)
    q, k, v = qkv[:nh * hs], qkv[nh * hs:(nh + nkv) * hs], qkv[(nh + nkv) * hs:]
    qw = np.concatenate([O.rmsnorm(q[h * hs:(h + 1) * hs], qn, 1e-6) for h in range(nh)])
    kw = np.concatenate([O.rmsnorm(k[h * hs:(h + 1) * hs], kn, 1e-6) for h in range(nkv)])
    qw = O.rope(qw, cos[pos], sin[pos], nh, hs)
    kw = O.rope(kw, cos[pos], sin[pos], nkv, hs)
    d = dev(qkv)
    kc, vc, bad = empty(2 * cap_pos * nkv * hs).zero(), empty(2 * cap_pos * nkv * hs).zero(), empty(4).zero()
    L.pllm_exact_qk_rope_cache(d.ptr, dev(qn).ptr, dev(kn).ptr, dev(cos).ptr, dev(sin).ptr, 0, pos, kc.ptr, vc.ptr, nh,
                               nkv, hs, 1e-6, 1, bad.ptr)
    check("pllm_exact_qk_rope_cache")
    assert same_bits(d.download(np.float32, nh * hs), qw)
    kcache = kc.download(np.uint16).reshape(cap_pos, -1)
    vcache = vc.download(np.uint16).reshape(cap_pos, -1)
    assert np.array_equal(kcache[pos], O.to_f16(kw)[0])
    assert np.array_equal(vcache[pos], O.to_f16(v)[0])


@pytest.mark.parametrize("cfg", [SMALL_QWEN3, STORIES], ids=["qwen3-small", "stories15m"])
@pytest.mark.parametrize("relaxed", [False, True])
def test_exact_forward_is_the_oracles(cfg, relaxed):
    cfg = replace(cfg, relaxed=relaxed)
    W = synthetic_host_weights(cfg, seed=3)
    eng = Engine(cfg, host=W, exact=True)
    A = oracle_arrays(cfg, W)
    oc = oracle_config(cfg)
    for pos, tok in enumerate(np.random.default_rng(1).integers(0, cfg.vocab, 40)):
        want = O.forward(oc, A, int(tok), pos)
        got = eng.forward(int(tok), pos)
        assert same_bits(got, want), (pos, float(np.abs(got - want).max()))
    eng.close()


@pytest.mark.parametrize("layers", [2, 36])
def test_qwen3_8b_shape_exact_logits(layers):
    """BASELINE.json configs[3] (Qwen3-8B-shaped int8, the device-made synthetic weights), the reference-order
    step against the oracle's forward: the same logits to the bit at every position, hence within the north star's
    max-abs 1e-3 of the largest |logit| and with the same greedy token."""
    cfg = replace(QWEN3_8B, seq_len=64, layers=layers)
    eng = Engine(cfg, seed=0, exact=True)
    A = oracle_arrays(cfg, eng.host_weights())
    oc = oracle_config(cfg)
    for pos, tok in enumerate([151, 9000, 42]):
        want = O.forward(oc, A, tok, pos)
        got = eng.forward(tok, pos)
        peak = float(np.abs(got - want).max() / np.abs(want).max())
        print(f"qwen3-8b shape, {layers} layers, position {pos}: max-abs / max|logit| {peak:.2e}, "
              f"argmax {np.argmax(got)} / {np.argmax(want)}")
        assert peak <= 1e-3 and np.argmax(got) == np.argmax(want), (pos, peak)
        assert same_bits(got, want), (pos, peak)
    eng.close()


def test_exact_graph_equals_eager():
    cfg = SMALL_QWEN3
    W = synthetic_host_weights(cfg, seed=5)
    a, b = Engine(cfg, host=W, exact=True, graphs=True), Engine(cfg, host=W, exact=True, graphs=False)
    for pos, tok in enumerate([3, 17, 999, 0, 42]):
        assert same_bits(a.forward(tok, pos), b.forward(tok, pos))
    a.close()
    b.close()
