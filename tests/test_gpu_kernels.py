"""Parity of every registry kernel of libpllm.so (called through the C ABI, device memory) with the CPU oracle on the
same inputs: the reference's own kernel-test cases (tests/golden/golden.npz: int8-check.ts and ternary-check.ts
inputs, edge weights and scales) and seeded random ones, plus the registry's contract (row ranges that write no row
outside them, tiles equal to the token kernel, refused arguments).

Bars: integer and byte work (quantize_x, interleave, the corrections, float16, every group's int32 sum, delta_rule)
to the bit; float32 products within float32 rounding of a different summation order, bounded per row by
8 * groups * 2^-24 * sum |group terms|; attention and the glue within 2e-5 relative (1e-4 for a float16 cache)."""
import numpy as np
import pytest

import oracle as O
from pllm.device import Buffer, init
from pllm.lib import L, PllmError, check

pytestmark = pytest.mark.gpu

EPS = 2.0 ** -24


_alive = []  # the buffers of the running test: a temporary's memory must outlive the kernels that read it


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


def get(b, dtype, count=None):
    return b.download(dtype, count)


def bits(a):
    return np.asarray(a, np.float32).view(np.int32)


def product_bound(G, ws, xs):
    """The float32 error bound of sum_g G_g (ws_g xs_g) for each row: (8 groups) 2^-24 sum |terms|. G: the group
    sums (rows, groups), or for matmul_q8 / q6 the four lanes each group is scaled in (rows, groups, 4): the
    reference rounds each lane's product alone, so its error is of the lanes' size, not of their sum's."""
    G = G.astype(np.float64)
    mag = np.abs(G).sum(axis=2) if G.ndim == 3 else np.abs(G)
    terms = mag * ws.astype(np.float64) * xs.astype(np.float64)[None, :]
    return 8 * mag.shape[1] * EPS * terms.sum(axis=1) + 1e-37


def lanes_q8(acts, w):
    """matmul.ts:68-72 (dot32): lane k of a group holds products 2k, 2k+1, 2k+8, 2k+9 of each half: (rows, ng, 4)."""
    rows, n = w.shape
    p = w.reshape(rows, n // 32, 32).astype(np.int64) * acts.reshape(n // 32, 32).astype(np.int64)
    idx = [[h + q for h in (0, 16) for q in (2 * k, 2 * k + 1, 2 * k + 8, 2 * k + 9)] for k in range(4)]
    return np.stack([p[:, :, i].sum(axis=2) for i in idx], axis=2)


# ---------------------------------------------------------------- activations

@pytest.mark.parametrize("bias", [0, 64])
def test_quantize_x_bit_exact(golden, bias):
    for x in (golden["quant_x"], np.random.default_rng(1).normal(0, 3, 4096).astype(np.float32)):
        xq, xs = dev(np.zeros(x.size, np.uint8)), dev(np.zeros(x.size // 32, np.float32))
        L.quantize_x(xq.ptr, xs.ptr, dev(x).ptr, x.size, bias)
        check("quantize_x")
        wq, ws = O.quantize_x(x, bias)
        assert np.array_equal(get(xq, np.uint8), wq)
        assert np.array_equal(bits(get(xs, np.float32)), bits(ws))


@pytest.mark.parametrize("groups", [1, 2, 3, 5, 9])
def test_interleave_bit_exact(golden, groups):
    k = f"tern_g{groups}_"
    n = groups * 128
    a, xs = golden[k + "a"], golden[k + "xs"]
    xq = dev(a.view(np.uint8))
    ext = dev(np.concatenate([xs, np.full(n // 32, -7, np.float32)]))
    L.interleave(xq.ptr, ext.ptr, n)
    check("interleave")
    assert np.array_equal(get(xq, np.int8), golden[k + "il"])
    e = get(ext, np.float32)
    assert np.array_equal(e[n // 32:].view(np.int32), golden[k + "sums"])
    assert np.array_equal(e[: n // 32], xs)


def test_corrections_exact(golden):
    for ng in (1, 9, 13, 81):
        w8, w6 = golden[f"int8_ng{ng}_w8"], golden[f"int8_ng{ng}_w6"]
        groups = w8.size // 32
        out = dev(np.full(groups + 4, -7, np.int32))
        L.int8_sums(out.ptr, dev(w8).ptr, groups)
        got = get(out, np.int32)
        assert np.array_equal(got[:groups], O.int8_sums(w8)) and np.all(got[groups:] == -7)
        L.six_sums(out.ptr, dev(w6).ptr, groups)
        assert np.array_equal(get(out, np.int32)[:groups], O.six_sums(w6))


# ---------------------------------------------------------------- int8 / int6 products

NGS = [1, 2, 3, 4, 5, 6, 7, 8, 9, 12, 13, 81]
RANGES = [(0, 13), (0, 1), (0, 3), (12, 13), (1, 6), (3, 8), (5, 5), (4, 12)]


@pytest.mark.parametrize("ng", NGS)
def test_group_sums_bit_exact(golden, ng):
    """The accumulators: every (row, group) int32 of int8 and int6 rows, plain and relaxed activations."""
    k = f"int8_ng{ng}_"
    n = ng * 32
    w8, w6 = dev(golden[k + "w8"]), dev(golden[k + "w6"])
    out = dev(np.zeros(13 * ng, np.int32))
    for t in range(9):
        for acts, bias in ((golden[k + "qp"][t].view(np.uint8), 0), (golden[k + "qr"][t], 64)):
            xq = dev(acts)
            xs = dev(np.zeros(2 * ng, np.float32))
            L.pllm_group_sums(out.ptr, xq.ptr, xs.ptr, w8.ptr, 0, n, 0, 13, bias)
            check("group sums")
            assert np.array_equal(get(out, np.int32).reshape(13, ng), O.group_sums_q8(acts, golden[k + "w8"], bias))
            L.pllm_group_sums(out.ptr, xq.ptr, xs.ptr, w6.ptr, 1, n, 0, 13, bias)
            assert np.array_equal(get(out, np.int32).reshape(13, ng), O.group_sums_q6(acts, golden[k + "w6"], n, bias))


@pytest.mark.parametrize("ng", NGS)
def test_int8_int6_products(golden, ng):
    """matmul_q8 / q8r / q6 / q6r on int8-check.ts's cases: every row range, nothing written outside it."""
    k = f"int8_ng{ng}_"
    n = ng * 32
    w8h, w6h, wsh = golden[k + "w8"], golden[k + "w6"], golden[k + "ws"]
    w8, w6, ws = dev(w8h), dev(w6h), dev(wsh)
    wc8, wc6 = dev(O.int8_sums(w8h)), dev(O.six_sums(w6h))
    out = dev(np.zeros(14, np.float32))
    for t in range(9):
        for plain in (True, False):
            acts = golden[k + "qp"][t].view(np.uint8) if plain else golden[k + "qr"][t]
            xsh = golden[k + "xp"][t] if plain else golden[k + "xr"][t]
            xq, xs = dev(acts), dev(xsh)
            bias = 0 if plain else 64
            if plain:
                G8 = lanes_q8(acts.view(np.int8), w8h)
                G6 = lanes_q8(acts.view(np.int8), O.widen6(w6h).reshape(13, n))
            else:
                G8 = O.group_sums_q8(acts, w8h, bias)
                G6 = O.group_sums_q6(acts, w6h, n, bias)
            cases = [("q8", G8, lambda r0, r1: L.matmul_q8(out.ptr, xq.ptr, xs.ptr, w8.ptr, ws.ptr, n, r0, r1)
                      if plain else L.matmul_q8r(out.ptr, xq.ptr, xs.ptr, w8.ptr, ws.ptr, wc8.ptr, n, r0, r1),
                      (golden[k + "q8"] if plain else golden[k + "q8r"])[t]),
                     ("q6", G6, lambda r0, r1: L.matmul_q6(out.ptr, xq.ptr, xs.ptr, w6.ptr, ws.ptr, n, r0, r1)
                      if plain else L.matmul_q6r(out.ptr, xq.ptr, xs.ptr, w6.ptr, ws.ptr, wc6.ptr, n, r0, r1),
                      (golden[k + "q6"] if plain else golden[k + "q6r"])[t])]
            for name, G, call, want in cases:
                bound = product_bound(G, wsh.reshape(13, ng), xsh)
                for r0, r1 in RANGES:
                    out.upload(np.full(14, -7, np.float32))
                    call(r0, r1)
                    check(name)
                    got = get(out, np.float32)
                    inside = np.arange(14)
                    inside = (inside >= r0) & (inside < r1)
                    assert np.all(got[~inside] == -7), (name, t, r0, r1)
                    err = np.abs(got[:13][inside[:13]].astype(np.float64) - want[inside[:13]])
                    assert np.all(err <= bound[inside[:13]]), (name, plain, t, r0, r1, err.max())


def test_q8r_tile_equals_token_kernel(golden):
    """relaxed/int8.ts:60-65: each (row, token) of the tile is matmul_q8r's number (here: to the bit on the GPU too),
    for 1..9, 16 and 21 tokens, rows off the fours; nothing written outside the rows and tokens; and every (row,
    token) within the products' bound of the oracle's matmul_q8r_tile."""
    k = "int8_ng13_"
    n, frame, os_ = 13 * 32, 8192, 64
    w8h = golden[k + "w8"]
    w8, ws, wc = dev(w8h), dev(golden[k + "ws"]), dev(O.int8_sums(w8h))
    rng = np.random.default_rng(9)
    tokens = 21
    qr = np.zeros((tokens, frame), np.uint8)
    for t in range(tokens):
        qr[t, :n] = golden[k + "qr"][t] if t < 9 else rng.integers(0, 128, n)
        qr[t, 4096:4096 + 13 * 4] = golden[k + "xr"][t % 9].view(np.uint8)
    frames = dev(qr)
    alone = dev(np.zeros(16, np.float32))
    outs = dev(np.zeros(tokens * os_ // 4, np.float32))
    for count in list(range(1, 10)) + [16, 21]:
        for r0, r1 in ((0, 13), (1, 6), (2, 13), (5, 5)):
            outs.upload(np.full(tokens * os_ // 4, -7, np.float32))
            L.matmul_q8r_tile(outs.ptr, frames.ptr, frames.ptr + 4096, w8.ptr, ws.ptr, wc.ptr, n, r0, r1, count, os_,
                              frame)
            check("matmul_q8r_tile")
            got = get(outs, np.float32).reshape(tokens, os_ // 4)
            for t in range(tokens):
                alone.upload(np.full(16, -7, np.float32))
                if t < count:
                    L.matmul_q8r(alone.ptr, frames.ptr + t * frame, frames.ptr + t * frame + 4096, w8.ptr, ws.ptr,
                                 wc.ptr, n, r0, r1)
                assert np.array_equal(bits(got[t]), bits(get(alone, np.float32))), (count, r0, r1, t)
            if r1 > r0:  # the oracle's tile (relaxed/int8.ts:147-166) on the same frames
                want = O.matmul_q8r_tile(qr, w8h, golden[k + "ws"], n, r0, r1, count, os_, frame)
                for t in range(count):
                    xq_t, xs_t = qr[t, :n], qr[t, 4096:4096 + 13 * 4].view(np.float32)
                    G = O.group_sums_q8(xq_t, w8h, 64).reshape(13, -1)
                    b = product_bound(G, golden[k + "ws"].reshape(13, -1), xs_t)
                    assert np.all(np.abs(got[t, r0:r1].astype(np.float64) - want[t, r0:r1]) <= b[r0:r1]), (count, t)


# ---------------------------------------------------------------- ternary / binary

@pytest.mark.parametrize("groups", [1, 2, 3, 4, 5, 7, 9])
def test_ternary_binary_products(golden, groups):
    k = f"tern_g{groups}_"
    n = groups * 128
    a, xsh = golden[k + "a"], golden[k + "xs"]
    il, ext = O.interleave(a.view(np.uint8), xsh)
    xq, xs = dev(il), dev(ext)
    halves = dev(golden[k + "halves"])
    out = dev(np.zeros(14, np.float32))
    sums = dev(np.zeros(13 * n // 32, np.int32))
    for binary, packed, want, fns in ((False, golden[k + "packed"], golden[k + "t2"], ("matmul_t2", "matmul_t2r")),
                                      (True, golden[k + "bpacked"], golden[k + "b1"], ("matmul_b1", "matmul_b1r"))):
        w = dev(packed)
        G = O.group_sums_signs(il, ext, packed, n, binary)
        L.pllm_group_sums(sums.ptr, xq.ptr, xs.ptr, w.ptr, 3 if binary else 2, n, 0, 13, 0)
        check("group sums signs")
        assert np.array_equal(get(sums, np.int32).reshape(13, -1), G)
        d = O.from_f16(golden[k + "halves"]).reshape(13, groups)
        terms = np.abs(G.astype(np.float64) * ext[: n // 32][None, :] * np.repeat(d, 4, axis=1))
        bound = 8 * (n // 32) * EPS * terms.sum(axis=1) + 1e-37
        for fn in fns:
            for r0, r1 in RANGES:
                out.upload(np.full(14, -7, np.float32))
                getattr(L, fn)(out.ptr, xq.ptr, xs.ptr, w.ptr, halves.ptr, n, r0, r1, 2 if binary else 3)
                check(fn)
                got = get(out, np.float32)
                sel = np.zeros(14, bool)
                sel[r0:r1] = True
                assert np.all(got[~sel] == -7)
                assert np.all(np.abs(got[:13][sel[:13]] - want[sel[:13]]) <= bound[sel[:13]]), (fn, r0, r1)


def test_signs_tiles_equal_token_kernel(golden):
    k = "tern_g5_"
    n, frame, os_ = 5 * 128, 4096, 64
    a, xsh = golden[k + "a"], golden[k + "xs"]
    rng = np.random.default_rng(4)
    tokens = 11
    buf = np.zeros((tokens, frame), np.uint8)
    for t in range(tokens):
        at = a if t == 0 else rng.integers(-128, 128, n).astype(np.int8)
        il, ext = O.interleave(at.view(np.uint8), xsh)
        buf[t, :n] = il
        buf[t, 2048:2048 + ext.nbytes] = ext.view(np.uint8)
    frames = dev(buf)
    halves = dev(golden[k + "halves"])
    for binary, packed, tile, one, code in ((False, golden[k + "packed"], "matmul_t2r_tile", "matmul_t2r", 3),
                                            (True, golden[k + "bpacked"], "matmul_b1r_tile", "matmul_b1r", 2)):
        w = dev(packed)
        outs = dev(np.full(tokens * os_ // 4, -7, np.float32))
        alone = dev(np.zeros(16, np.float32))
        for count in (1, 3, 4, 7, 11):
            outs.upload(np.full(tokens * os_ // 4, -7, np.float32))
            getattr(L, tile)(outs.ptr, frames.ptr, frames.ptr + 2048, w.ptr, halves.ptr, n, 1, 12, count, os_, frame, code)
            check(tile)
            got = get(outs, np.float32).reshape(tokens, -1)
            for t in range(tokens):
                alone.upload(np.full(16, -7, np.float32))
                if t < count:
                    getattr(L, one)(alone.ptr, frames.ptr + t * frame, frames.ptr + t * frame + 2048, w.ptr, halves.ptr,
                                    n, 1, 12, code)
                assert np.array_equal(bits(got[t]), bits(get(alone, np.float32))), (tile, count, t)
                if t < count:  # and against the oracle's signs product (relaxed/signs.ts:77-120) on the token's frame
                    il, ext = buf[t, :n], buf[t, 2048:2048 + n // 4].view(np.float32)
                    want = O.matmul_signs(il, ext, packed, golden[k + "halves"], n, binary, 1, 12)
                    G = O.group_sums_signs(il, ext, packed, n, binary).astype(np.float64)
                    d = np.repeat(O.from_f16(golden[k + "halves"]).reshape(-1, n // 128), 4, axis=1)
                    b = 8 * (n // 32) * EPS * (np.abs(G) * ext[: n // 32][None, :] * d).sum(axis=1) + 1e-37
                    assert np.all(np.abs(got[t, 1:12].astype(np.float64) - want[1:12]) <= b[1:12]), (tile, count, t)


# ---------------------------------------------------------------- model-sized products (size-independent properties)

@pytest.mark.parametrize("mode", [0, 1], ids=["bulk-copy", "register"])
@pytest.mark.parametrize("K,N", [(4096, 12288), (12288, 4096), (1024, 4608)])
def test_large_products_against_oracle(K, N, mode):
    """BASELINE.json's product shapes: every output against the oracle's matmul_q8 within its float32 bound, the
    group sums of 64 sampled rows to the bit, and the relaxed product's sums against the plain ones' integers."""
    rng = np.random.default_rng(K + N)
    from pllm.forward import quantize_rows
    wq, ws = quantize_rows(rng.normal(0, 0.02, (N, K)).astype(np.float32))
    x = rng.normal(0, 1, K).astype(np.float32)
    old = L.pllm_set_gemv_mode(mode)
    W, S = dev(wq), dev(ws)
    out = dev(np.zeros(N, np.float32))
    for bias in (0, 64):
        xqh, xsh = O.quantize_x(x, bias)
        xq, xs = dev(xqh), dev(xsh)
        if bias:
            L.matmul_q8r(out.ptr, xq.ptr, xs.ptr, W.ptr, S.ptr, 0, K, 0, N)
            want = O.matmul_q8r(xqh, xsh, wq, ws)
        else:
            L.matmul_q8(out.ptr, xq.ptr, xs.ptr, W.ptr, S.ptr, K, 0, N)
            want = O.matmul_q8(xqh, xsh, wq, ws)
        check("large product")
        got = get(out, np.float32)
        rows = rng.choice(N, 64, replace=False)
        G = O.group_sums_q8(xqh, wq[rows], bias)
        sums = dev(np.zeros(N * (K // 32), np.int32))
        L.pllm_group_sums(sums.ptr, xq.ptr, xs.ptr, W.ptr, 0, K, 0, N, bias)
        allG = get(sums, np.int32).reshape(N, K // 32)
        assert np.array_equal(allG[rows], G)
        bound = product_bound(allG, ws, xsh)
        assert np.all(np.abs(got.astype(np.float64) - want) <= bound + 1e-7 * np.abs(want))
        assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()
    L.pllm_set_gemv_mode(old)


# ---------------------------------------------------------------- attention, rope, halves

@pytest.mark.parametrize("half", [False, True])
@pytest.mark.parametrize("nh,nkv,hs", [(8, 2, 128), (6, 6, 48), (16, 8, 64), (4, 4, 32)])
@pytest.mark.parametrize("pos", [0, 3, 130, 700])
def test_attention(half, nh, nkv, hs, pos):
    rng = np.random.default_rng(pos * 31 + nh)
    count = pos + 1
    q = rng.normal(0, 1, nh * hs).astype(np.float32)
    kc = rng.normal(0, 1, (count, nkv * hs)).astype(np.float32)
    vc = rng.normal(0, 1, (count, nkv * hs)).astype(np.float32)
    if half:
        kc, _ = O.to_f16(kc)
        vc, _ = O.to_f16(vc)
    want, _ = O.attention(q, kc, vc, pos, nh, nkv, hs, half=half)
    for cap in (0.0, 5.0):
        if cap:
            want, _ = O.attention(q, kc, vc, pos, nh, nkv, hs, half=half, cap=cap)
        out = dev(np.full(nh * hs + 8, -7, np.float32))
        att = dev(np.zeros(nh * count, np.float32))
        K, V, Q = dev(kc), dev(vc), dev(q)
        name = ("attention_f16" if half else "attention") + ("_capped" if cap else "")
        args = [out.ptr, Q.ptr, K.ptr, V.ptr, att.ptr, pos, nh, nkv, hs, 0, nh] + ([cap] if cap else [])
        getattr(L, name)(*args)
        check(name)
        got = get(out, np.float32)
        assert np.all(got[nh * hs:] == -7)
        np.testing.assert_allclose(got[: nh * hs], want, rtol=1e-4, atol=2e-5)
    # a range of heads writes only those heads
    out = dev(np.full(nh * hs, -7, np.float32))
    L.attention_f16(out.ptr, Q.ptr, K.ptr, V.ptr, att.ptr, pos, nh, nkv, hs, 1, nh - 1) if half else \
        L.attention(out.ptr, Q.ptr, K.ptr, V.ptr, att.ptr, pos, nh, nkv, hs, 1, nh - 1)
    got = get(out, np.float32).reshape(nh, hs)
    assert np.all(got[0] == -7) and np.all(got[-1] == -7)


def test_rope_and_halves():
    rng = np.random.default_rng(3)
    nh, hs = 6, 48
    v = rng.normal(0, 1, nh * hs).astype(np.float32)
    c = rng.uniform(-1, 1, hs // 2).astype(np.float32)
    s = rng.uniform(-1, 1, hs // 2).astype(np.float32)
    V = dev(v)
    L.rope(V.ptr, dev(c).ptr, dev(s).ptr, nh, hs, 0)
    np.testing.assert_allclose(get(V, np.float32), O.rope(v, c, s, nh, hs), rtol=1e-6, atol=1e-6)
    x = np.concatenate([rng.normal(0, 1, 3000), rng.normal(0, 1e-6, 500), rng.normal(0, 4e4, 500),
                        [np.inf, -np.inf, np.nan, 65520.0, 2 ** -25, -0.0]]).astype(np.float32)
    H = dev(np.zeros(x.size, np.uint16))
    bad = L.to_f16(H.ptr, dev(x).ptr, x.size)
    want, wbad = O.to_f16(x)
    assert bad == wbad == 3
    assert np.array_equal(get(H, np.uint16), want)
    F = dev(np.zeros(x.size, np.float32))
    L.from_f16(F.ptr, H.ptr, x.size)
    assert np.array_equal(bits(get(F, np.float32)), bits(O.from_f16(want)))
    assert L.finite_f16(H.ptr, x.size) == 0 and L.finite_f16(H.ptr, 3000) == 1


# ---------------------------------------------------------------- glue and the stateful layers

def test_glue():
    rng = np.random.default_rng(11)
    n = 1000
    x, w, y = (rng.normal(0, 1, n).astype(np.float32) for _ in range(3))
    out = dev(np.zeros(n, np.float32))
    L.rmsnorm(out.ptr, dev(x).ptr, dev(w).ptr, n, 1e-5)
    np.testing.assert_allclose(get(out, np.float32), O.rmsnorm(x, w, 1e-5), rtol=2e-6, atol=1e-7)
    L.swiglu(out.ptr, dev(x).ptr, dev(y).ptr, n)
    np.testing.assert_allclose(get(out, np.float32), O.swiglu(x, y), rtol=2e-6, atol=1e-7)
    X = dev(x)
    L.add_inplace(X.ptr, dev(y).ptr, n)
    assert np.array_equal(get(X, np.float32), O.add_inplace(x, y))
    L.gate(out.ptr, dev(x).ptr, dev(y).ptr, n)
    np.testing.assert_allclose(get(out, np.float32), O.gate(x, y), rtol=2e-6, atol=1e-7)
    taps, rows = rng.normal(0, 1, (4, n)).astype(np.float32), rng.normal(0, 1, (4, n)).astype(np.float32)
    L.convolve(out.ptr, dev(taps).ptr, dev(rows).ptr, n, 4)
    np.testing.assert_allclose(get(out, np.float32), O.convolve(taps, rows), rtol=2e-6, atol=1e-7)
    b = rng.normal(0, 1, 3 * n).astype(np.float32)
    R = dev(rows[:3])
    L.short_conv(out.ptr, dev(taps[:3]).ptr, R.ptr, dev(b).ptr, n, 3)
    want, wrows = O.short_conv(taps[:3], rows[:3], b)
    assert np.array_equal(get(out, np.float32), want)
    assert np.array_equal(get(R, np.float32).reshape(3, n), wrows)
    wf = rng.normal(0, 0.1, (37, n)).astype(np.float32)
    o = dev(np.zeros(37, np.float32))
    L.matmul_f32(o.ptr, dev(x).ptr, dev(wf).ptr, n, 0, 37)
    np.testing.assert_allclose(get(o, np.float32), O.matmul_f32(x, wf), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("kh,vh,kd,vd", [(2, 4, 16, 16), (16, 32, 128, 128), (1, 1, 4, 4)])
def test_delta_rule_bit_exact(kh, vh, kd, vd):
    """stateful.ts:96-151: the same float32 operations in the same order, so the same numbers to the bit; the state
    is read, the new one written at next; a head range writes only its heads."""
    rng = np.random.default_rng(kd + vh)
    state = rng.normal(0, 0.5, vh * kd * vd).astype(np.float32)
    c = rng.normal(0, 0.3, 2 * kh * kd + vh * vd).astype(np.float32)
    work = np.concatenate([rng.uniform(0.1, 0.9, vh), rng.uniform(0.5, 1.0, vh), np.zeros(vh * vd)]).astype(np.float32)
    want_out, want_next, want_work = O.delta_rule(state, c, work, kh, kd, vd, vh)
    out, S, N, C, W = dev(np.zeros(vh * vd, np.float32)), dev(state), dev(np.zeros_like(state)), dev(c), dev(work)
    L.delta_rule(out.ptr, S.ptr, N.ptr, C.ptr, W.ptr, kh, kd, vd, vh, 0, vh)
    check("delta_rule")
    assert np.array_equal(bits(get(out, np.float32)), bits(want_out))
    assert np.array_equal(bits(get(N, np.float32)), bits(want_next))
    assert np.array_equal(bits(get(W, np.float32)), bits(want_work))
    assert np.array_equal(get(S, np.float32), state)


@pytest.mark.parametrize("count", [1, 64])
def test_delta_rule_block_is_the_tokens_one_by_one(count):
    """pllm_delta_rule_block: count tokens of the recurrence in one launch (the state on the chip between them) give
    each token's outputs, gates' delta and the last state of delta_rule called a token at a time, to the bit; the
    delta rule's micro-configuration (kh 16, vh 32, kd = vd = 128); a head range writes only its heads."""
    kh, vh, kd, vd = 16, 32, 128, 128
    rng = np.random.default_rng(count)
    state = rng.normal(0, 0.5, vh * kd * vd).astype(np.float32)
    cw = 2 * kh * kd + vh * vd
    c = rng.normal(0, 0.3, (count, cw)).astype(np.float32)
    ww = 2 * vh + vh * vd
    work = np.zeros((count, ww), np.float32)
    work[:, :vh] = rng.uniform(0.1, 0.9, (count, vh))
    work[:, vh:2 * vh] = rng.uniform(0.5, 1.0, (count, vh))
    outs, s = [], state
    for t in range(count):
        o, s, w = O.delta_rule(s, c[t], work[t], kh, kd, vd, vh)
        outs.append(o)
        work_t = w
    for h0, h1 in ((0, vh), (4, 20)):
        out = dev(np.full(count * vh * vd, -7, np.float32))
        S, N, C, W = dev(state), dev(np.zeros_like(state)), dev(c), dev(work)
        L.pllm_delta_rule_block(out.ptr, vh * vd, S.ptr, N.ptr, C.ptr, cw, W.ptr, ww, count, kh, kd, vd, vh, h0, h1)
        check("pllm_delta_rule_block")
        got = get(out, np.float32).reshape(count, vh, vd)
        want = np.stack(outs).reshape(count, vh, vd)
        assert np.array_equal(bits(got[:, h0:h1]), bits(want[:, h0:h1]))
        assert np.all(got[:, :h0] == -7) and np.all(got[:, h1:] == -7)
        nxt = get(N, np.float32).reshape(vh, kd, vd)
        assert np.array_equal(bits(nxt[h0:h1]), bits(s.reshape(vh, kd, vd)[h0:h1]))
        last = get(W, np.float32).reshape(count, ww)[-1]
        delta = last[2 * vh:].reshape(vh, vd)
        assert np.array_equal(bits(delta[h0:h1]), bits(work_t[2 * vh:].reshape(vh, vd)[h0:h1]))


# ---------------------------------------------------------------- the contract's refusals

def test_bad_arguments_launch_nothing():
    out = dev(np.full(4, -7, np.float32))
    z = dev(np.zeros(64, np.uint8))
    for call in (lambda: L.matmul_q8(out.ptr, z.ptr, z.ptr, z.ptr, z.ptr, 33, 0, 1),        # n not whole groups
                 lambda: L.matmul_q8(out.ptr, z.ptr, z.ptr, z.ptr, z.ptr, 32, 2, 1),        # r1 < r0
                 lambda: L.quantize_x(z.ptr, z.ptr, z.ptr, 32, 7),                          # a bias of neither
                 lambda: L.matmul_t2(out.ptr, z.ptr, z.ptr, z.ptr, z.ptr, 128, 0, 1, 2),    # a wrong mask
                 lambda: L.matmul_q8(out.ptr, z.ptr + 4, z.ptr, z.ptr, z.ptr, 32, 0, 1)):   # misaligned
        call()
        with pytest.raises(PllmError):
            check("refused")
    assert np.all(get(out, np.float32) == -7)


# ---------------------------------------------------------------- the forward driver's fused products, both kernels

@pytest.fixture(params=[0, 1], ids=["bulk-copy", "register"])
def gemv_mode(request):
    old = L.pllm_set_gemv_mode(request.param)
    yield request.param
    L.pllm_set_gemv_mode(old)


@pytest.mark.parametrize("K,N", [(4096, 1000), (12288, 520), (384, 77)])
@pytest.mark.parametrize("pro", [1, 2])
@pytest.mark.parametrize("epi", [0, 1, 2])
@pytest.mark.parametrize("relaxed", [False, True])
def test_fused_gemv(gemv_mode, K, N, pro, epi, relaxed):
    """pllm_gemv's prologues (RMSNorm + quantize_x, quantize_x) and epilogues (store, residual add, SwiGLU of a row
    pair) against the oracle's rmsnorm, quantize_x and matmul_q8 / q8r on the same numbers. The input is small
    integers, so that its sum of squares is exact in any order and the quantized activations are the oracle's to the
    byte; every group's integer is then exact and the outputs agree within float32 rounding."""
    rng = np.random.default_rng(K + N + pro + 3 * epi)
    from pllm.forward import quantize_rows
    rows = 2 * N if epi == 2 else N
    wq, ws = quantize_rows(rng.normal(0, 0.02, (rows, K)).astype(np.float32))
    tokens = 2 if (N == 520 and epi != 1) else 1
    x = rng.integers(-8, 9, (tokens, K)).astype(np.float32)
    norm = rng.normal(1, 0.1, K).astype(np.float32)
    eps, bias = 1e-6, (64 if relaxed else 0)
    init = rng.normal(0, 1, (tokens, N)).astype(np.float32)
    W, S, X, NW = dev(wq), dev(ws), dev(x), dev(norm)
    out = dev(init)
    L.pllm_gemv(out.ptr, N, 0, 0, 0, 0, X.ptr, K, NW.ptr if pro == 1 else 0, eps, bias, W.ptr, S.ptr, 0, K, 0, N,
                tokens, pro, epi, N if epi == 2 else 0, 0)
    check("pllm_gemv")
    got = get(out, np.float32).reshape(tokens, N)
    for t in range(tokens):
        xb = O.rmsnorm(x[t], norm, eps) if pro == 1 else x[t]
        xq, xs = O.quantize_x(xb, bias)
        prod = (O.matmul_q8r(xq, xs, wq, ws) if relaxed else O.matmul_q8(xq, xs, wq, ws)).astype(np.float64)
        G = O.group_sums_q8(xq, wq, bias)
        bound = product_bound(G, ws, xs)
        if epi == 0:
            assert np.all(np.abs(got[t] - prod) <= bound), (t, np.abs(got[t] - prod).max())
        elif epi == 1:
            want = init[t].astype(np.float64) + prod
            assert np.all(np.abs(got[t] - want) <= bound + 2 * EPS * np.abs(want))
        else:
            h1, h3 = prod[:N], prod[N:]
            want = h1 / (1 + np.exp(-h1)) * h3
            slack = (np.abs(h3) * bound[:N] + np.abs(h1) * bound[N:]) * 2 + 1e-6 * np.abs(want) + 1e-12
            assert np.all(np.abs(got[t] - want) <= slack), (t, np.abs(got[t] - want).max())
    assert L.pllm_device_status() == 0


@pytest.mark.parametrize("mode", [0, 1])
def test_registry_products_both_kernels(golden, mode):
    """matmul_q8 / q8r through the bulk-copy kernel and the register one give the same numbers as each other within
    float32 rounding, and the same as before on int8-check.ts's cases of 81 groups."""
    old = L.pllm_set_gemv_mode(mode)
    try:
        k = "int8_ng81_"
        n = 81 * 32
        w8h, wsh = golden[k + "w8"], golden[k + "ws"]
        # 81 groups is no multiple of 128 columns: the register kernel serves it in both modes
        w8, ws = dev(w8h), dev(wsh)
        out = dev(np.zeros(13, np.float32))
        for t in range(9):
            xq, xs = dev(golden[k + "qr"][t]), dev(golden[k + "xr"][t])
            L.matmul_q8r(out.ptr, xq.ptr, xs.ptr, w8.ptr, ws.ptr, 0, n, 0, 13)
            check("matmul_q8r")
            G = O.group_sums_q8(golden[k + "qr"][t], w8h, 64)
            bound = product_bound(G, wsh.reshape(13, 81), golden[k + "xr"][t])
            assert np.all(np.abs(get(out, np.float32) - golden[k + "q8r"][t]) <= bound)
    finally:
        L.pllm_set_gemv_mode(old)


@pytest.mark.parametrize("K,N", [(4096, 8192), (12288, 2731), (128, 262144)])
@pytest.mark.parametrize("pro", [0, 1, 2])
@pytest.mark.parametrize("epi", [0, 1, 2])
def test_int6_bulk_copy_is_the_register_kernel(K, N, pro, epi):
    """pllm_gemv on int6 weights (fmt 1) at one token: the bulk-copy form (whole rows a stage, tiles by tickets; it
    serves products of 2^25 weights and more, as these) and the register kernel take every lane's groups of 32 in the
    same order, so their outputs are the same bits, for every prologue (the caller's activations, plain and relaxed;
    RMSNorm + quantize_x; quantize_x) and epilogue (store, residual add, SwiGLU of a row pair). The register kernel's
    numbers are the oracle's within float32 rounding (test_int8_int6_products)."""
    rng = np.random.default_rng(K + N + 5 * pro + epi)
    ng = K // 32
    rows = 2 * N if epi == 2 else N
    w6 = dev(rng.integers(0, 256, (rows, ng * 24), dtype=np.uint8))
    ws = dev(rng.uniform(1e-3, 2e-2, (rows, ng)).astype(np.float32))
    x = dev(rng.normal(0, 1, K).astype(np.float32))
    norm = dev(rng.normal(1, 0.1, K).astype(np.float32))
    init = rng.normal(0, 1, N).astype(np.float32)
    for bias in ((0, 64) if pro == 0 else (0,)):
        lo = 0 if bias else -127
        xq = dev(rng.integers(lo, 128, K).astype(np.int8).view(np.uint8))
        xs = dev(rng.uniform(1e-3, 1e-2, ng).astype(np.float32))
        results = []
        for mode in (0, 1):
            old = L.pllm_set_gemv_mode(mode)
            try:
                out = dev(init)
                L.pllm_gemv(out.ptr, N, xq.ptr if pro == 0 else 0, xs.ptr if pro == 0 else 0, 0, 0,
                            x.ptr if pro else 0, K, norm.ptr if pro == 1 else 0, 1e-6, bias, w6.ptr, ws.ptr, 1, K, 0, N,
                            1, pro, epi, N if epi == 2 else 0, 0)
                check("pllm_gemv int6")
                results.append(get(out, np.float32))
            finally:
                L.pllm_set_gemv_mode(old)
        assert np.isfinite(results[0]).all()
        assert np.array_equal(bits(results[0]), bits(results[1])), (bias, np.abs(results[0] - results[1]).max())
    assert L.pllm_device_status() == 0


@pytest.mark.parametrize("half", [True, False])
@pytest.mark.parametrize("nh,nkv,hs,qk", [(8, 2, 128, True), (6, 6, 48, False), (16, 8, 64, False)])
def test_attention_step(half, nh, nkv, hs, qk):
    """The driver's fused attention step against the oracle's steps on the same numbers: rmsnorm of every q and k
    head (activations.ts:8-20), rope at pos (attention.ts:7-20), the key and value into the cache (halves.ts:35, to
    the bit), attention over 0..pos (attention.ts:87-211); positions inside one slice, at the slices' edges and at
    the cache's end; twice in a row (the slices' counts are left at zero)."""
    rng = np.random.default_rng(nh * hs)
    cap, split, eps = 300, 64, 1e-6
    kvdim = nkv * hs
    E = np.uint16 if half else np.float32
    old = rng.normal(0, 1, (cap, kvdim)).astype(np.float32)
    kc0 = O.to_f16(old)[0].reshape(cap, kvdim) if half else old.copy()
    vc0 = O.to_f16(old[::-1].copy())[0].reshape(cap, kvdim) if half else old[::-1].copy()
    qn = rng.normal(1, 0.1, hs).astype(np.float32) if qk else None
    kn = rng.normal(1, 0.1, hs).astype(np.float32) if qk else None
    ang = np.outer(np.arange(cap), 1.0 / 1e4 ** (np.arange(0, hs, 2) / hs))
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    C, S = dev(cos), dev(sin)
    QN, KN = (dev(qn), dev(kn)) if qk else (None, None)
    scratch = dev(np.zeros(L.pllm_attention_scratch_bytes(nh, hs, cap, split) // 4 + 1, np.float32))
    bad = dev(np.zeros(1, np.int32))
    for pos in (0, 5, 63, 64, 200, cap - 1):
        qkv = rng.normal(0, 1, (nh + 2 * nkv) * hs).astype(np.float32)
        KC, VC = dev(kc0.reshape(-1)), dev(vc0.reshape(-1))
        P = dev(np.array([0, pos], np.int32))
        out = dev(np.zeros(nh * hs, np.float32))
        for _ in range(2):
            L.pllm_attention_step(out.ptr, dev(qkv).ptr, KC.ptr, VC.ptr, scratch.ptr, P.ptr + 4, cap, nh, nkv, hs,
                                  int(half), 0.0, split, QN.ptr if qk else 0, KN.ptr if qk else 0, C.ptr, S.ptr, 0,
                                  eps, bad.ptr, 0)
            check("pllm_attention_step")
            q, k, v = qkv[: nh * hs], qkv[nh * hs: nh * hs + kvdim], qkv[nh * hs + kvdim:]
            if qk:
                q = np.concatenate([O.rmsnorm(q[h * hs:(h + 1) * hs], qn, eps) for h in range(nh)])
                k = np.concatenate([O.rmsnorm(k[h * hs:(h + 1) * hs], kn, eps) for h in range(nkv)])
            q = O.rope(q, cos[pos], sin[pos], nh, hs)
            k = O.rope(k, cos[pos], sin[pos], nkv, hs)
            kc, vc = kc0.copy(), vc0.copy()
            kc[pos] = O.to_f16(k)[0] if half else k
            vc[pos] = O.to_f16(v)[0] if half else v
            got_k = get(KC, E).reshape(cap, kvdim)
            got_v = get(VC, E).reshape(cap, kvdim)
            if half:
                assert np.array_equal(got_k[pos], kc[pos]) and np.array_equal(got_v[pos], vc[pos])
            else:
                np.testing.assert_allclose(got_k[pos], kc[pos], rtol=1e-6, atol=1e-6)
                assert np.array_equal(got_v[pos], vc[pos])
            assert np.array_equal(np.delete(got_k, pos, 0), np.delete(kc0, pos, 0))
            want, _ = O.attention(q, kc[: pos + 1], vc[: pos + 1], pos, nh, nkv, hs, half=half)
            np.testing.assert_allclose(get(out, np.float32), want, rtol=1e-4, atol=2e-5)
    counts = get(scratch, np.int32)[-(nh + 1):]
    assert np.all(counts == 0)


@pytest.mark.parametrize("mode", [1, 0], ids=["clusters", "slices"])
@pytest.mark.parametrize("written", [307, -3])
def test_attention_step_holds_a_device_position_in_the_cache(mode, written):
    """A position in device memory outside the cache (the host's calls check theirs; a graph reads what is there):
    the step takes the cache's last (or first) row instead, reads and writes nothing outside the cache, and reports
    PLLM_ERANGE (5) in the device status word, which reading clears."""
    nh, nkv, hs, cap, split, eps = 8, 2, 128, 300, 64, 1e-6
    held = cap - 1 if written >= cap else 0
    rng = np.random.default_rng(cap)
    kvdim = nkv * hs
    kc0 = O.to_f16(rng.normal(0, 1, (cap, kvdim)).astype(np.float32))[0].reshape(cap, kvdim)
    vc0 = O.to_f16(rng.normal(0, 1, (cap, kvdim)).astype(np.float32))[0].reshape(cap, kvdim)
    ang = np.outer(np.arange(cap), 1.0 / 1e4 ** (np.arange(0, hs, 2) / hs))
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    # guard rows around the cache: a write outside it would show there
    pad = 4 * kvdim
    KC = dev(np.concatenate([np.full(pad, 0x7777, np.uint16), kc0.reshape(-1), np.full(pad, 0x7777, np.uint16)]))
    VC = dev(np.concatenate([np.full(pad, 0x7777, np.uint16), vc0.reshape(-1), np.full(pad, 0x7777, np.uint16)]))
    scratch = dev(np.zeros(L.pllm_attention_scratch_bytes(nh, hs, cap, split) // 4 + 1, np.float32))
    qkv = rng.normal(0, 1, (nh + 2 * nkv) * hs).astype(np.float32)
    out, bad = dev(np.zeros(nh * hs, np.float32)), dev(np.zeros(1, np.int32))
    P = dev(np.array([0, written], np.int32))
    old = L.pllm_set_attention_mode(mode)
    try:
        assert L.pllm_device_status() == 0
        L.pllm_attention_step(out.ptr, dev(qkv).ptr, KC.ptr + 2 * pad, VC.ptr + 2 * pad, scratch.ptr, P.ptr + 4, cap,
                              nh, nkv, hs, 1, 0.0, split, 0, 0, dev(cos).ptr, dev(sin).ptr, 0, eps, bad.ptr, 0)
        check("pllm_attention_step")
        assert L.pllm_device_status() == 5
        assert L.pllm_device_status() == 0
    finally:
        L.pllm_set_attention_mode(old)
    k, v = qkv[nh * hs: nh * hs + kvdim], qkv[nh * hs + kvdim:]
    q = O.rope(qkv[: nh * hs], cos[held], sin[held], nh, hs)
    k = O.rope(k, cos[held], sin[held], nkv, hs)
    kc, vc = kc0.copy(), vc0.copy()
    kc[held], vc[held] = O.to_f16(k)[0], O.to_f16(v)[0]
    got_k, got_v = get(KC, np.uint16), get(VC, np.uint16)
    assert np.all(got_k[:pad] == 0x7777) and np.all(got_k[-pad:] == 0x7777)
    assert np.all(got_v[:pad] == 0x7777) and np.all(got_v[-pad:] == 0x7777)
    assert np.array_equal(got_k[pad:-pad].reshape(cap, kvdim), kc)
    assert np.array_equal(got_v[pad:-pad].reshape(cap, kvdim), vc)
    want, _ = O.attention(q, kc[: held + 1], vc[: held + 1], held, nh, nkv, hs, half=True)
    np.testing.assert_allclose(get(out, np.float32), want, rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("n", [1, 7, 1000, 151936])
def test_argmax_and_penalize(n):
    """sample.ts's argmax (device, both forms) and penalize against the oracle's walks: NaNs, ties, -inf."""
    rng = np.random.default_rng(n)
    cases = [rng.normal(0, 3, n).astype(np.float32)]
    if n > 5:
        t = rng.normal(0, 3, n).astype(np.float32)
        t[[2, n - 1]] = t.max() + 1.0  # a tie: the first wins
        t[1] = np.nan
        cases.append(t)
        z = rng.normal(0, 3, n).astype(np.float32)
        z[0] = np.nan  # the walk starts from a NaN
        cases.append(z)
        cases.append(np.full(n, -np.inf, np.float32))
    scratch = dev(np.zeros(4, np.int32))
    out = dev(np.zeros(1, np.int32))
    for x in cases:
        X = dev(x)
        want = O.argmax(x)
        assert L.argmax(X.ptr, n) == want
        L.pllm_argmax_dev(out.ptr, X.ptr, n, scratch.ptr)
        check("pllm_argmax_dev")
        assert int(get(out, np.int32)[0]) == want
    tokens = rng.integers(0, n, 40).astype(np.int32)
    logits = cases[0]
    X, T = dev(logits), dev(tokens)
    L.penalize(X.ptr, T.ptr, tokens.size, 1.3, 0.4)
    check("penalize")
    np.testing.assert_array_equal(get(X, np.float32)[:n], O.penalize(logits, tokens, 1.3, 0.4))


@pytest.mark.parametrize("n", [50, 1000, 4096, 151936])
def test_sample_draws_the_oracles_tokens(n):
    """sample (sample.ts:248-337) on the device against the oracle's walk (pinned to the reference's NumPy sampler):
    temperature, top-p, top-k and min-p settings, seeded random numbers. The device's probabilities come of CUDA's
    expf (within an ulp or two of the reference's exp) and its double sums of another association, so a draw may
    differ only where the random number falls at a boundary of the walk: wherever the oracle draws the same token
    at random x (1 - 1e-5) and x (1 + 1e-5), the device's token is that token. Both entry points (the waiting one,
    and the one that reads its random number from device memory)."""
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 4.0).astype(np.float32)
    x[n // 3] = x[n // 5]  # a tie
    X, P, I = dev(x), dev(np.zeros(n, np.float32)), dev(np.zeros(n, np.int32))
    R, out = dev(np.zeros(1, np.float64)), dev(np.zeros(1, np.int32))
    checked = 0
    for temperature, topp, topk, minp in [(1.0, 0.9, 0, 0.0), (0.7, 1.0, 0, 0.0), (1.3, 0.0, 40, 0.0),
                                          (1.0, 0.5, 40, 0.05), (1.0, 0.0, 0, 0.05), (0.8, 0.95, 1, 0.0),
                                          (2.0, 0.999, 2000, 0.0)]:
        for r in rng.random(6):
            want = O.sample(x, temperature, topp, r, topk, minp)
            steady = all(O.sample(x, temperature, topp, r * f, topk, minp) == want for f in (1 - 1e-5, 1 + 1e-5))
            got = L.sample(X.ptr, n, temperature, topp, float(r), P.ptr, I.ptr, topk, minp)
            check("sample")
            R.upload(np.array([r], np.float64))
            L.pllm_sample_dev(out.ptr, X.ptr, n, temperature, topp, R.ptr, P.ptr, I.ptr, topk, minp)
            check("pllm_sample_dev")
            got_dev = int(get(out, np.int32)[0])
            if steady:
                assert got == want and got_dev == want, (temperature, topp, topk, minp, r, got, got_dev, want)
                checked += 1
    assert checked >= 30
    bad = x.copy()
    bad[7] = np.nan
    B = dev(bad)
    assert L.sample(B.ptr, n, 1.0, 0.9, 0.5, P.ptr, I.ptr, 0, 0.0) == -1


SB_TYPES = {"Q2_K": (10, 84, (80, 82)), "Q4_K": (12, 144, (0, 2)), "IQ2_XXS": (16, 66, (0,)), "IQ2_XS": (17, 74, (0,)),
            "IQ3_XXS": (18, 98, (0,)), "IQ1_S": (19, 50, (0,)), "IQ3_S": (21, 110, (0,)), "IQ2_S": (22, 82, (0,)),
            "IQ4_XS": (23, 136, (0,)), "IQ1_M": (29, 56, ())}


def sb_blocks(rng, size, halves, count):
    """random blocks (any bytes are blocks) with finite float16 scales of a model's size"""
    raw = rng.integers(0, 256, (count, size), dtype=np.uint8)
    for at in halves:
        d = rng.uniform(0.002, 0.05, count) * np.where(rng.random(count) < 0.2, -1, 1)
        raw[:, at:at + 2] = d.astype("<f2").view(np.uint8).reshape(count, 2)
    if size == 56:  # IQ1_M: d in the top four bits of its four scale words
        d = rng.uniform(0.002, 0.05, count).astype("<f2").view("<u2")
        for k in range(4):
            word = raw[:, 48 + 2 * k:50 + 2 * k].copy().view("<u2").reshape(-1)
            word = (word & 0x0fff) | (((d >> (4 * k)) & 15) << 12)
            raw[:, 48 + 2 * k:50 + 2 * k] = word.astype("<u2").view(np.uint8).reshape(count, 2)
    return raw


@pytest.mark.parametrize("name", list(SB_TYPES))
def test_superblock_products(name):
    """llama.cpp's blocks (blocks/*.ts) on the device against the oracle (pinned to the reference's reader):
    sb_tables' bytes and sb_row's floats to the bit; sums_x to the bit; matmul_sb, matmul_sbr and the tiles (five
    tokens, frame and os strides) within 1e-5 of the sum of |weight x activation| of each row (the blocks' float32
    partial sums in another order; every group's integer is exact); rows r0..r1 only."""
    import os
    t, size, halves = SB_TYPES[name]
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "superblocks.npz"))
    books = g["codebooks"]
    tab_want = O.sb_tables(books)
    tab = dev(np.zeros(O.SB_TABLES, np.uint8))
    assert L.sb_tables(tab.ptr, dev(books).ptr) == O.SB_TABLES
    check("sb_tables")
    assert np.array_equal(get(tab, np.uint8), tab_want)
    rng = np.random.default_rng(t)
    rows, n = 37, 1536
    w = sb_blocks(rng, size, halves, rows * n // 256).reshape(rows, -1)
    W = dev(w)
    out = dev(np.zeros(n, np.float32))
    L.sb_row(out.ptr, W.ptr + 5 * w.shape[1], tab.ptr, n, t)
    check("sb_row")
    assert np.array_equal(get(out, np.float32).view(np.uint32), O.sb_row(w[5], tab_want, n, t).view(np.uint32))
    widened = np.stack([O.sb_row(w[r], tab_want, n, t) for r in range(rows)]).astype(np.float64)
    count, frame = 5, n + n // 2 + 64  # a token's activations then its xs (scales and sums), frame bytes apart
    X = np.zeros((count, frame), np.uint8)
    want = np.zeros((count, rows), np.float64)
    bound = np.zeros((count, rows))
    for k in range(count):
        x = rng.normal(0, 1, n).astype(np.float32)
        xq, xs = O.quantize_x(x, 0)
        X[k, :n] = xq
        X[k, n:n + n // 2] = O.sums_x(xs, xq.view(np.int8)).view(np.uint8)
        a = (xq.view(np.int8).astype(np.float64).reshape(-1, 32) * xs[:, None]).reshape(-1)
        want[k] = O.matmul_sb(xq.view(np.int8), xs, w, tab_want, n, rows, t)
        bound[k] = 1e-5 * (np.abs(widened) * np.abs(a)).sum(axis=1)
    XB = dev(X.reshape(-1))
    for fn in ("matmul_sb", "matmul_sbr"):
        o = dev(np.full(rows, -9.0, np.float32))
        getattr(L, fn)(o.ptr, XB.ptr, XB.ptr + n, W.ptr, tab.ptr, n, 3, rows - 2, t)
        check(fn)
        got = get(o, np.float32)
        assert np.all(got[:3] == -9.0) and np.all(got[rows - 2:] == -9.0)
        assert np.all(np.abs(got[3:rows - 2] - want[0, 3:rows - 2]) <= bound[0, 3:rows - 2]), fn
    os_ = 4 * (rows + 3)
    for fn in ("matmul_sbr_tile", "matmul_sbw_tile"):
        o = dev(np.zeros(count * (rows + 3), np.float32))
        args = [o.ptr, XB.ptr, XB.ptr + n, W.ptr, tab.ptr, n, 0, rows, count, os_, frame, t]
        getattr(L, fn)(*(args + ([0] if fn == "matmul_sbw_tile" else [])))
        check(fn)
        got = get(o, np.float32).reshape(count, rows + 3)[:, :rows]
        assert np.all(np.abs(got - want) <= bound), fn


def test_sums_x_and_signed_dots():
    rng = np.random.default_rng(3)
    n = 4096
    xq = rng.integers(-127, 128, n).astype(np.int8)
    xs = rng.random(n // 32).astype(np.float32)
    buf = np.zeros(n // 2 // 4, np.float32)
    buf[:n // 32] = xs
    B, Q = dev(buf), dev(xq)
    L.sums_x(B.ptr, Q.ptr, n)
    check("sums_x")
    assert np.array_equal(get(B, np.float32).view(np.uint32), O.sums_x(xs, xq).view(np.uint32))
    a = rng.integers(-128, 128, 16).astype(np.int8)
    b = rng.integers(-128, 128, 16).astype(np.int8)
    out = dev(np.zeros(4, np.int32))
    L.signed_dots(out.ptr, dev(a).ptr, dev(b).ptr)
    check("signed_dots")
    assert np.array_equal(get(out, np.int32), (a.astype(np.int32) * b).reshape(4, 4).sum(axis=1))


# ---------------------------------------------------------------- the engine's memory touches as device kernels

def test_memory_touches_are_the_javascripts():
    """pllm_shift_rows (convolution.ts:57's copyWithin), pllm_scale_rows (engine.ts:452-455), pllm_delta_gates
    (linear.ts:151-158: JavaScript's double-precision exp / log1p, stored as float32) and pllm_softcap
    (engine.ts:467-470: each step rounded to float32) against the same arithmetic in NumPy (float64, then float32):
    the moves and products to the bit, the transcendental ones within one float32 step."""
    rng = np.random.default_rng(12)
    n, count = 1000, 3
    rows = rng.normal(0, 1, (count, n)).astype(np.float32)
    R = dev(rows)
    L.pllm_shift_rows(R.ptr, n, count)
    check("pllm_shift_rows")
    want = rows.copy()
    want[:-1] = rows[1:]
    assert np.array_equal(get(R, np.float32).reshape(count, n), want)
    x = rng.normal(0, 1, (4, 640)).astype(np.float32)
    X, S = dev(x), dev(np.array([0.37], np.float32))
    L.pllm_scale_rows(X.ptr, 600, 4, 640, S.ptr)
    check("pllm_scale_rows")
    want = x.copy()
    want[:, :600] = x[:, :600] * np.float32(0.37)
    assert np.array_equal(get(X, np.float32).reshape(4, 640), want)
    vh = 32
    work = np.concatenate([rng.normal(0, 3, vh), rng.normal(0, 12, vh)]).astype(np.float32)
    work[vh + 3] = 30.0  # past softplus's 20
    decays = -np.exp(rng.normal(0, 1, vh)).astype(np.float32)
    dt = rng.normal(0, 1, vh).astype(np.float32)
    W = dev(work)
    L.pllm_delta_gates(W.ptr, dev(decays).ptr, dev(dt).ptr, vh)
    check("pllm_delta_gates")
    b, step = work[:vh].astype(np.float64), work[vh:].astype(np.float64) + dt.astype(np.float64)
    soft = np.where(step > 20, step, np.log1p(np.exp(np.minimum(step, 20))))
    want = np.concatenate([1.0 / (1.0 + np.exp(-b)), np.exp(decays.astype(np.float64) * soft)]).astype(np.float32)
    got = get(W, np.float32)
    assert np.all(np.abs(got.view(np.int32) - want.view(np.int32)) <= 1), (got, want)
    logits = rng.normal(0, 40, 5000).astype(np.float32)
    G = dev(logits)
    L.pllm_softcap(G.ptr, logits.size, 30.0)
    check("pllm_softcap")
    q = (logits.astype(np.float64) / 30.0).astype(np.float32)
    want = (30.0 * np.tanh(q.astype(np.float64)).astype(np.float32).astype(np.float64)).astype(np.float32)
    got = get(G, np.float32)
    assert np.all(np.abs(got.view(np.int32) - want.view(np.int32)) <= 1)
