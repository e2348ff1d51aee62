"""The prefill product on the tensor cores (pllm_gemm_q8: tcgen05 kind::i8 a group of 32 at a time, the exact int32 of
each group scaled in float32) and its activations (pllm_norm_quantize_rows), against the oracle.

  - every group's integer is exact: with all scales 1 the products are sums of int32s small enough to be exact in
    float32, compared to NumPy's integer product to the bit;
  - with quantize_x's scales the outputs agree with the oracle's matmul_q8 (the reference's lane order) within the
    float32 rounding of the different summation order: 1e-5 of the sum of the groups' |scaled terms|;
  - the epilogues: the residual add and the gated FFN's silu(w1 row) x (w3 row)."""
import numpy as np
import pytest

import oracle as O
from pllm.device import Buffer, init
from pllm.forward import quantize_rows
from pllm.lib import L, check

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _device():
    init(0)
    L.pllm_set_stream(0)
    yield


def dev(a, keep):
    b = Buffer.of(np.ascontiguousarray(a))
    keep.append(b)
    return b.ptr


def gemm(xq, xs, w, ws, epi=0, n=None, pair=0, out=None):
    """pllm_gemm_q8 on host arrays: xq (M x K int8), xs (M x K/32), w (rows x K int8), ws (rows x K/32)."""
    keep = []
    M, K = xq.shape
    rows = w.shape[0]
    n = rows if n is None else n
    o = np.zeros((M, n), np.float32) if out is None else out.astype(np.float32).copy()
    ob = Buffer.of(o)
    keep.append(ob)
    L.pllm_gemm_q8(ob.ptr, n, dev(xq.astype(np.int8), keep), dev(xs.astype(np.float32), keep),
                   dev(w.astype(np.int8), keep), dev(np.ascontiguousarray(ws.T).astype(np.float32), keep), M, n, K,
                   rows, epi, pair)
    assert L.pllm_sync() == 0
    check("pllm_gemm_q8")
    res = ob.download(np.float32).reshape(M, n)
    assert L.pllm_device_status() == 0
    for b in keep:
        b.free()
    return res


@pytest.mark.parametrize("M,N,K,lim", [(128, 128, 128, 127), (200, 256, 1024, 8), (1, 128, 4096, 8),
                                       (300, 384, 512, 127)])
def test_group_integers_exact(M, N, K, lim):
    rng = np.random.default_rng(M + N + K)
    xq = rng.integers(-lim, lim + 1, (M, K)).astype(np.int8)
    w = rng.integers(-lim, lim + 1, (N, K)).astype(np.int8)
    if lim == 127 and K > 128:  # keep the row sums exact in float32: large values in the first group only
        xq[:, 32:] = np.clip(xq[:, 32:], -3, 3)
    got = gemm(xq, np.ones((M, K // 32), np.float32), w, np.ones((N, K // 32), np.float32))
    want = xq.astype(np.int64) @ w.astype(np.int64).T
    assert np.abs(want).max() < 2 ** 24
    assert np.array_equal(got, want.astype(np.float32))


def quantized_problem(M, N, K, seed, bias=0):
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, (M, K)).astype(np.float32)
    q = [O.quantize_x(x[m], bias) for m in range(M)]
    xq = np.stack([a for a, _ in q]).astype(np.int16) - bias  # signed
    xs = np.stack([b for _, b in q])
    w, ws = quantize_rows(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    return xq.astype(np.int8), xs, w, ws, q


def oracle_rows(q, w, ws, bias):
    if bias:
        wc = O.int8_sums(w)
        return np.stack([O.matmul_q8r(a, b, w, ws, wc) for a, b in q])
    return np.stack([O.matmul_q8(a, b, w, ws) for a, b in q])


def magnitude(xq, xs, w, ws):
    """sum over groups of |G_g| * xs * ws per (token, row): the scale of the float32 rounding"""
    M, K = xq.shape
    G = np.einsum("mgk,ngk->mng", xq.reshape(M, K // 32, 32).astype(np.int64),
                  w.reshape(w.shape[0], K // 32, 32).astype(np.int64))
    return (np.abs(G) * xs[:, None, :] * ws[None, :, :]).sum(axis=2)


@pytest.mark.parametrize("M,N,K", [(1, 128, 4096), (77, 256, 512), (128, 128, 1024), (300, 384, 4096)])
@pytest.mark.parametrize("bias", [0, 64])
def test_matches_oracle(M, N, K, bias):
    xq, xs, w, ws, q = quantized_problem(M, N, K, M * 7 + K, bias)
    got = gemm(xq, xs, w, ws)
    want = oracle_rows(q, w, ws, bias)
    tol = 1e-5 * magnitude(xq, xs, w, ws) + 1e-30
    assert np.all(np.abs(got - want) <= tol), np.max(np.abs(got - want) / tol)


def test_residual_add():
    xq, xs, w, ws, q = quantized_problem(130, 256, 512, 3)
    base = np.random.default_rng(4).normal(0, 1, (130, 256)).astype(np.float32)
    got = gemm(xq, xs, w, ws, epi=1, out=base)
    want = base + oracle_rows(q, w, ws, 0)
    tol = 1e-5 * magnitude(xq, xs, w, ws) + 1e-6 * np.abs(base)
    assert np.all(np.abs(got - want) <= tol)


def test_gated_ffn():
    hidden, K = 192, 512
    xq, xs, w, ws, q = quantized_problem(150, 2 * hidden, K, 5)
    got = gemm(xq, xs, w, ws, epi=2, n=hidden, pair=hidden)
    h = oracle_rows(q, w, ws, 0)
    want = np.stack([O.swiglu(r[:hidden], r[hidden:]) for r in h])
    assert np.allclose(got, want, rtol=1e-4, atol=1e-5 * np.abs(want).max())


@pytest.mark.parametrize("bias", [0, 64])
def test_norm_quantize_rows(bias):
    rng = np.random.default_rng(bias)
    rows, n = 37, 4096
    x = rng.normal(0, 1, (rows, n)).astype(np.float32)
    x[3, :32] = 0.0  # an all-zero group (scale 0)
    norm = rng.normal(1, 0.1, n).astype(np.float32)
    keep = []
    xq, xs = Buffer(rows * n), Buffer(rows * n // 8)
    keep += [xq, xs]
    L.pllm_norm_quantize_rows(xq.ptr, xs.ptr, dev(x, keep), n, 0, 1e-6, n, rows, bias)
    assert L.pllm_sync() == 0
    q = xq.download(np.int8).reshape(rows, n)
    s = xs.download(np.float32).reshape(rows, n // 32)
    for r in range(rows):  # quantize_x alone: the oracle's bytes and scales exactly
        wq, ws = O.quantize_x(x[r], bias)
        assert np.array_equal(q[r], (wq.astype(np.int16) - bias).astype(np.int8))
        assert np.array_equal(s[r], ws)
    L.pllm_norm_quantize_rows(xq.ptr, xs.ptr, dev(x, keep), n, dev(norm, keep), 1e-6, n, rows, bias)
    assert L.pllm_sync() == 0
    q = xq.download(np.int8).reshape(rows, n)
    s = xs.download(np.float32).reshape(rows, n // 32)
    flips = 0
    for r in range(rows):  # RMSNorm first: its sum in another order may flip a rounding now and then
        wq, ws = O.quantize_x(O.rmsnorm(x[r], norm, 1e-6), bias)
        want = wq.view(np.int8).astype(np.int16) if bias == 0 else wq.astype(np.int16) - bias
        d = q[r].astype(np.int16) - want
        assert np.abs(d).max() <= 1
        flips += int(np.count_nonzero(d))
        assert np.allclose(s[r], ws, rtol=1e-6, atol=0)
    assert flips <= rows * n * 1e-3
    for b in keep:
        b.free()
