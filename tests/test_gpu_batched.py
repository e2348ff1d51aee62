"""The batched decode product (3..16 tokens a pass: the bulk-copy pipeline with one tensor-core product a group of 32,
mma m16n8k32 int8 -> int32, 16 tokens x 8 rows) against the oracle's matmul_q8r_tile / matmul_q8 (relaxed/int8.ts:
147-166, matmul.ts:77-104): every group's int32 is the reference's (the group sums are checked to the bit), the float32
rows within the products' bound (8 x groups x 2^-24 x sum |terms|) of the oracle's. The sweep's shapes (BASELINE.json
(K, N) in {(1024, 1024), (1024, 4608), (4096, 4096), (4096, 12288), (12288, 4096)}); K = 12288 reads the
activations from global memory (too long for shared memory beside the stages). The forward driver's fused forms
(RMSNorm / quantize prologues, residual and SwiGLU epilogues) at 16 tokens against the same kernel one token at a
time, within the same bound."""
import numpy as np
import pytest

import oracle as O
from pllm.device import Buffer, init
from pllm.lib import L, check

from test_gpu_kernels import lanes_q8, product_bound

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


def weights(rng, rows, k):
    w = rng.integers(-127, 128, (rows, k)).astype(np.int8)
    w[0, :64] = -128
    ws = rng.uniform(0.001, 0.02, (rows, k // 32)).astype(np.float32)
    return w, ws


@pytest.mark.parametrize("k,rows", [(1024, 1024), (1024, 4608), (4096, 4096), (4096, 12288), (12288, 4096)])
@pytest.mark.parametrize("count", [3, 4, 16, 21])
def test_tile_is_the_oracles(k, rows, count):
    """The registry's matmul_q8r_tile (count tokens a frame apart, outputs os bytes apart) on the batched form."""
    rng = np.random.default_rng(k + rows + count)
    w, ws = weights(rng, rows, k)
    frame = k + k // 8  # the token's bytes, then its scales (16-byte aligned)
    frames = np.zeros((count, frame), np.uint8)
    xq_t, xs_t = [], []
    for t in range(count):
        xq, xs = O.quantize_x(rng.normal(0, 1, k).astype(np.float32), 64)
        frames[t, :k] = xq
        frames[t, k:k + k // 8] = xs.view(np.uint8)
        xq_t.append(xq)
        xs_t.append(xs)
    F, W, WS = dev(frames), dev(w), dev(ws)
    os_ = rows * 4 + 64
    out = dev(np.full(count * os_ // 4, -7, np.float32))
    L.matmul_q8r_tile(out.ptr, F.ptr, F.ptr + k, W.ptr, WS.ptr, 0, k, 0, rows, count, os_, frame)
    check("matmul_q8r_tile")
    got = out.download(np.float32).reshape(count, os_ // 4)
    for t in range(count):
        want = O.matmul_q8r(xq_t[t], xs_t[t], w, ws)
        G = O.group_sums_q8(xq_t[t], w, 64).reshape(rows, k // 32)
        bound = product_bound(G, ws, xs_t[t])
        err = np.abs(got[t, :rows].astype(np.float64) - want)
        assert np.all(err <= bound), (t, float(err.max()), float(bound[np.argmax(err - bound)]))
        assert np.all(got[t, rows:] == -7), t  # nothing past the rows


@pytest.mark.parametrize("k,rows", [(4096, 4096), (12288, 4096)])
def test_plain_product_is_the_oracles(k, rows):
    """matmul_q8's signed activations (bias 0) through pllm_gemv's caller-quantized form, 16 tokens."""
    rng = np.random.default_rng(k)
    w, ws = weights(rng, rows, k)
    count = 16
    xq = np.zeros((count, k), np.uint8)
    xs = np.zeros((count, k // 32), np.float32)
    for t in range(count):
        xq[t], xs[t] = O.quantize_x(rng.normal(0, 1, k).astype(np.float32), 0)
    out = dev(np.zeros(count * rows, np.float32))
    XQ, XS, W, WS = dev(xq), dev(xs), dev(w), dev(ws)
    L.pllm_gemv(out.ptr, rows, XQ.ptr, XS.ptr, k, k // 8, 0, 0, 0, 0.0, 0, W.ptr, WS.ptr, 0, k, 0, rows, count, 0, 0,
                0, 0)
    check("pllm_gemv batched")
    got = out.download(np.float32).reshape(count, rows)
    for t in range(count):
        want = O.matmul_q8(xq[t], xs[t], w, ws)
        bound = product_bound(lanes_q8(xq[t].view(np.int8), w), ws, xs[t])
        assert np.all(np.abs(got[t].astype(np.float64) - want) <= bound), t


@pytest.mark.parametrize("pro,epi", [(1, 0), (2, 1), (1, 2)], ids=["rms-store", "quant-add", "rms-swiglu"])
def test_fused_forms_at_16_tokens(pro, epi):
    """The forward driver's forms (pro 1 RMSNorm + quantize_x, 2 quantize_x; epi 0 store, 1 add, 2 SwiGLU of a row
    pair) at 16 tokens equal the same product one token at a time (the same prologue, so the same int8 activations
    and group sums), within the float32 bound of the sums' other order."""
    rng = np.random.default_rng(pro * 10 + epi)
    k, rows, count = 4096, 2048, 16
    total = 2 * rows if epi == 2 else rows
    w, ws = weights(rng, total, k)
    x = rng.normal(0, 1, (count, k)).astype(np.float32)
    norm = rng.normal(1, 0.1, k).astype(np.float32)
    base = rng.normal(0, 1, (count, rows)).astype(np.float32)
    W, WS, X, N = dev(w), dev(ws), dev(x), dev(norm)
    batched, single = dev(base), dev(base)
    args = lambda out, xp, t, c: (out, rows, 0, 0, 0, 0, xp, k, N.ptr if pro == 1 else 0, 1e-6, 0, W.ptr, WS.ptr, 0,  # noqa: E731
                                  k, 0, rows, c, pro, epi, rows if epi == 2 else 0, 0)
    L.pllm_gemv(*args(batched.ptr, X.ptr, 0, count))
    for t in range(count):
        L.pllm_gemv(*args(single.ptr + t * rows * 4, X.ptr + t * k * 4, t, 1))
    check("pllm_gemv fused forms")
    a = batched.download(np.float32).reshape(count, rows).astype(np.float64)
    b = single.download(np.float32).reshape(count, rows).astype(np.float64)
    # two float32 sums of the same exact terms in other orders: within 2e-5 of the outputs' size (the sums' relative
    # rounding is ~1e-6 at 128 groups; SwiGLU carries each factor's into the other)
    assert np.abs(a - b).max() <= 2e-5 * np.abs(b).max(), float(np.abs(a - b).max())
