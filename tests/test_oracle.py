"""The CPU oracle pinned to the reference's known answers (tests/golden/golden.npz) before it is trusted as the
checker of the CUDA kernels. CPU only."""
import os

import numpy as np
import pytest

import oracle as O

RANGES = [(0, 13), (0, 1), (0, 3), (12, 13), (1, 6), (3, 8), (5, 5), (4, 12)]


def bits(a):
    return np.asarray(a, np.float32).view(np.int32)


@pytest.mark.parametrize("bias", [0, 64])
def test_quantize_x_edge_groups(golden, bias):
    """int8-check.ts:232-265: zeros, -0, subnormal groups whose 1/scale overflows, the ends, half steps."""
    xq, xs = O.quantize_x(golden["quant_x"], bias)
    assert np.array_equal(xs.view(np.int32), golden[f"quant_s{bias}"].view(np.int32))
    assert np.array_equal(xq, golden[f"quant_q{bias}"])


def test_quantize_x_is_packing_quantize(golden):
    """engine/packing.py:40-45 (the converter's int8) is quantize_x(bias 0) row by row, to the byte."""
    x = golden["pack_x"]
    for r in range(x.shape[0]):
        xq, xs = O.quantize_x(x[r], 0)
        assert np.array_equal(xq.view(np.int8), golden["pack_q8"].reshape(x.shape)[r])
        assert np.array_equal(xs, golden["pack_s8"].reshape(x.shape[0], -1)[r])


def test_widen6_is_unpack6(golden):
    assert np.array_equal(O.widen6(golden["pack_six"]), golden["pack_six_values"])


@pytest.mark.parametrize("ng", [1, 2, 3, 4, 5, 6, 7, 8, 9, 12, 13, 81])
def test_int8_products_bit_exact(golden, ng):
    """int8-check.ts: matmul_q8r / q6r / q8 / q6 are the written-out models to the bit, on every row range."""
    k = f"int8_ng{ng}_"
    w8, w6, ws = golden[k + "w8"], golden[k + "w6"], golden[k + "ws"]
    n = ng * 32
    wc8 = O.int8_sums(w8)
    wc6 = O.six_sums(w6)
    assert np.array_equal(wc8, -64 * w8.reshape(-1, 32).astype(np.int32).sum(1))
    assert np.array_equal(wc6, -64 * O.widen6(w6).reshape(-1, 32).astype(np.int32).sum(1))
    for t in range(9):
        qr, xr, qp, xp = golden[k + "qr"][t], golden[k + "xr"][t], golden[k + "qp"][t], golden[k + "xp"][t]
        for r0, r1 in RANGES:
            sl = slice(r0, r1)
            got = O.matmul_q8r(qr, xr, w8, ws, wc8, r0, r1)[sl]
            assert np.array_equal(bits(got), bits(golden[k + "q8r"][t][sl])), (t, r0, r1)
            got = O.matmul_q8r(qr, xr, w8, ws, None, r0, r1)[sl]  # without corrections: the same integers
            assert np.array_equal(bits(got), bits(golden[k + "q8r"][t][sl]))
            got = O.matmul_q6r(qr, xr, w6, ws, n, wc6, r0, r1)[sl]
            assert np.array_equal(bits(got), bits(golden[k + "q6r"][t][sl]))
            got = O.matmul_q8(qp.view(np.uint8), xp, w8, ws, r0, r1)[sl]
            assert np.array_equal(bits(got), bits(golden[k + "q8"][t][sl]))
            got = O.matmul_q6(qp.view(np.uint8), xp, w6, ws, n, r0, r1)[sl]
            assert np.array_equal(bits(got), bits(golden[k + "q6"][t][sl]))


@pytest.mark.parametrize("groups", [1, 2, 3, 4, 5, 7, 9])
def test_ternary_binary_bit_exact(golden, groups):
    """ternary-check.ts: interleave's bytes and sums; matmul_t2 / t2r and (binary.ts) matmul_b1 / b1r, to the bit."""
    k = f"tern_g{groups}_"
    n = groups * 128
    a, xs = golden[k + "a"], golden[k + "xs"]
    il, ext = O.interleave(a.view(np.uint8), xs)
    assert np.array_equal(il.view(np.int8), golden[k + "il"])
    assert np.array_equal(ext[n // 32:].view(np.int32), golden[k + "sums"])
    assert np.array_equal(ext[: n // 32], xs)
    t2 = O.matmul_signs(il, ext, golden[k + "packed"], golden[k + "halves"], n, binary=False)
    assert np.array_equal(bits(t2), bits(golden[k + "t2"]))
    b1 = O.matmul_signs(il, ext, golden[k + "bpacked"], golden[k + "halves"], n, binary=True)
    assert np.array_equal(bits(b1), bits(golden[k + "b1"]))


def test_ternary_and_binary_packings_decode(golden):
    """The codes the oracle reads from engine/packing.py's pack_ternary and pack_binary bytes are the weights + 1."""
    n = 256
    for name, binary in (("tern", False), ("bin", True)):
        values = golden[f"pack_{name}_values"].astype(np.int64)
        packed, halves = golden[f"pack_{name}"], golden[f"pack_{name}_s"]
        rng = np.random.default_rng(3)
        a = rng.integers(-127, 128, n).astype(np.int8)
        xs = np.ones(n // 32, np.float32)
        il, ext = O.interleave(a.view(np.uint8), xs)
        sums = O.group_sums_signs(il, ext, packed, n, binary=binary)
        want = (values.reshape(-1, n // 32, 32) * a.reshape(n // 32, 32)).sum(-1)
        assert np.array_equal(sums, want)


def test_group_sums_q8(golden):
    k = "int8_ng9_"
    w8 = golden[k + "w8"]
    for t in range(9):
        qr, qp = golden[k + "qr"][t], golden[k + "qp"][t]
        g = O.group_sums_q8(qr, w8, bias=64)
        want = (w8.reshape(13, 9, 32).astype(np.int64) * (qr.reshape(9, 32).astype(np.int64) - 64)).sum(-1)
        assert np.array_equal(g, want)
        g = O.group_sums_q8(qp.view(np.uint8), w8, bias=0)
        want = (w8.reshape(13, 9, 32).astype(np.int64) * qp.reshape(9, 32).astype(np.int64)).sum(-1)
        assert np.array_equal(g, want)


def test_q8r_tile_is_token_kernel(golden):
    """relaxed/int8.ts:60-65: every (row, token) of the tile is matmul_q8r's number."""
    k = "int8_ng13_"
    w8, ws = golden[k + "w8"], golden[k + "ws"]
    qr, xr = golden[k + "qr"], golden[k + "xr"]
    for t in range(9):
        assert np.array_equal(bits(O.matmul_q8r(qr[t], xr[t], w8, ws)), bits(golden[k + "q8r"][t]))


def test_float_glue_against_numpy(golden):
    """rmsnorm, head norm, rope, swiglu against the reference's NumPy (engine/layers.py) within float32 rounding."""
    out = O.rmsnorm(golden["rms_x"], golden["rms_w"], 1e-5)
    np.testing.assert_allclose(out, golden["rms_out"], rtol=2e-6, atol=1e-7)
    hs = golden["head_w"].size
    x = golden["rms_x"]
    heads = np.concatenate([O.rmsnorm(x[h * hs:(h + 1) * hs], golden["head_w"], 1e-6) for h in range(x.size // hs)])
    np.testing.assert_allclose(heads, golden["head_out"], rtol=2e-6, atol=1e-7)
    r = O.rope(x, golden["rope_cos"], golden["rope_sin"], x.size // hs, hs)
    np.testing.assert_allclose(r, golden["rope_out"], rtol=1e-6, atol=1e-7)
    s = O.swiglu(golden["swiglu_h1"], golden["swiglu_h3"])
    np.testing.assert_allclose(s, golden["swiglu_out"], rtol=2e-6, atol=1e-7)


def test_delta_rule_against_numpy(golden):
    """stateful.ts:96-151 against engine/layers.py:149-156 within delta-check.ts's 2e-5."""
    kh, vh, kd, vd = 2, 4, 16, 16
    c = np.concatenate([golden["delta_qk"].reshape(-1), golden["delta_v"].reshape(-1)])
    work = np.concatenate([golden["delta_beta"], golden["delta_decay"], np.zeros(vh * vd, np.float32)])
    out, nxt, _ = O.delta_rule(golden["delta_state"].reshape(-1), c, work, kh, kd, vd, vh)
    np.testing.assert_allclose(out, golden["delta_out"], rtol=2e-5, atol=2e-5)
    np.testing.assert_allclose(nxt, golden["delta_next"], rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("half", [False, True])
def test_attention_against_numpy(golden, half):
    """attention.ts:87-211 against the NumPy attention of engine/model.py:532-538 (GQA 6 over 2 heads)."""
    nh, nkv, size, count = 6, 2, 16, 21
    keys, values = golden["att_k"], golden["att_v"]
    kc = keys.transpose(1, 0, 2).reshape(count, nkv * size)  # the kernels' [pos][kv heads * size]
    vc = values.transpose(1, 0, 2).reshape(count, nkv * size)
    if half:
        kc, _ = O.to_f16(kc.reshape(-1))
        vc, _ = O.to_f16(vc.reshape(-1))
    out, att = O.attention(golden["att_q"], kc, vc, count - 1, nh, nkv, size, half=half)
    tol = 2e-3 if half else 2e-5
    np.testing.assert_allclose(out, golden["att_out"], rtol=tol, atol=tol)
    np.testing.assert_allclose(att.reshape(nh, count).sum(1), 1.0, rtol=1e-5)


def test_f16_conversions():
    """halves.ts: to_f16 rounds as NumPy's astype(float16) (ties to even, overflow to infinity), counting the inputs
    that were not finite; from_f16 is exact for finite halves and reads an infinity as 65536."""
    rng = np.random.default_rng(5)
    x = np.concatenate([rng.normal(0, 1, 4000), rng.normal(0, 1e-5, 1000), rng.normal(0, 3e4, 1000),
                        [0.0, -0.0, 65504, 65520, 65519.99, 1e5, -1e5, 2 ** -25, 2 ** -24, 3 * 2 ** -26]]).astype(np.float32)
    h, bad = O.to_f16(x)
    with np.errstate(over="ignore"):
        assert np.array_equal(h, x.astype(np.float16).view(np.uint16))
    assert bad == 0
    _, bad = O.to_f16(np.array([np.inf, np.nan, 1.0, -np.inf], np.float32))
    assert bad == 3
    finite = h[(h & 0x7C00) != 0x7C00]
    assert np.array_equal(O.from_f16(finite), finite.view(np.float16).astype(np.float32))
    assert O.from_f16(np.array([0x7C00], np.uint16))[0] == 65536.0
    assert O.finite_f16(finite) == 1 and O.finite_f16(np.array([1, 0x7C00], np.uint16)) == 0


def test_exp_close_to_libm():
    xs = np.linspace(-86, 88, 2001, dtype=np.float32)
    got = np.array([O.lib().or_fexp(float(v)) for v in xs], np.float32)
    np.testing.assert_allclose(got, np.exp(xs.astype(np.float64)), rtol=3e-7)
    assert O.lib().or_fexp(-90.0) == 0.0 and O.lib().or_vexp(-90.0) > 0


def test_argmax_and_penalize_walks():
    """sample.ts's argmax (the first of equal largest; a NaN never greater, one at index 0 the answer) and penalize
    (each distinct token once), against NumPy written the same way."""
    x = np.array([1.0, 3.0, -2.0, 3.0, np.nan, 2.5], np.float32)
    assert O.argmax(x) == 1
    assert O.argmax(np.array([np.nan, 5.0, 7.0], np.float32)) == 0
    assert O.argmax(np.array([-np.inf, -np.inf], np.float32)) == 0
    logits = np.array([2.0, -1.0, 0.5, 4.0, -3.0], np.float32)
    got = O.penalize(logits, np.array([3, 1, 3, 4, 1], np.int32), 1.3, 0.25)
    want = logits.copy()
    for t in (3, 1, 4):
        v = want[t]
        want[t] = (v / np.float32(1.3) if v > 0 else v * np.float32(1.3)) - np.float32(0.25)
    np.testing.assert_array_equal(got, want)


def test_sample_draws_the_reference_samplers_tokens():
    """or_sample (sample.ts:248-337) against the reference's NumPy sampler (engine/sampler.py NumpySampler.drawing,
    which the kernel restates) on the draws of tests/golden/sampling.npz: three vocabularies, temperature, top-p,
    top-k and min-p settings, random numbers handed in; every token the same."""
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "sampling.npz"))
    logits = [g["logits0"], g["logits1"], g["logits2"]]
    for v, t, p, k, m, r, tok in g["draws"]:
        assert O.sample(logits[int(v)], float(t), float(p), r, int(k), float(m)) == int(tok), (v, t, p, k, m, r)
    bad = logits[1].copy()
    bad[7] = np.nan
    assert O.sample(bad, 1.0, 0.9, 0.5) == -1
    bad[7] = np.inf
    assert O.sample(bad, 1.0, 0.9, 0.5) == -1


SB_TYPES = ["Q2_K", "Q4_K", "IQ2_XXS", "IQ2_XS", "IQ3_XXS", "IQ1_S", "IQ3_S", "IQ2_S", "IQ4_XS", "IQ1_M"]


def test_superblock_rows_are_the_reference_readers():
    """or_sb_row (blocks/row.ts: each weight as the reference's reader makes it) on the ten block types of
    tests/golden/superblocks.npz equals the reference's NumPy reader (convert/superblocks.py) to the bit: the bytes'
    layouts, the scales' order of float32 products, IQ1's shifts, the K types' minima. And or_matmul_sb (the token's
    arithmetic, blocks/types.ts:66-83) agrees with the widened rows times the dequantized activations."""
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "superblocks.npz"))
    tab = O.sb_tables(g["codebooks"])
    rng = np.random.default_rng(0)
    for name in SB_TYPES:
        t, blocks = int(g[f"{name}/ggml"]), g[f"{name}/blocks"]
        got = np.stack([O.sb_row(b, tab, 256, t) for b in blocks])
        assert np.array_equal(got.view(np.uint32), g[f"{name}/weights"].view(np.uint32)), name
        w = blocks.reshape(3, -1)  # 3 rows of 4 blocks
        x = rng.normal(0, 1, 1024).astype(np.float32)
        xq, xs = O.quantize_x(x, 0)
        out = O.matmul_sb(xq.view(np.int8), xs, w, tab, 1024, 3, t)
        a = (xq.view(np.int8).astype(np.float64).reshape(-1, 32) * xs[:, None]).reshape(-1)
        rows = np.stack([O.sb_row(w[r], tab, 1024, t) for r in range(3)]).astype(np.float64)
        bound = 1e-5 * (np.abs(rows) * np.abs(a)).sum(axis=1)
        assert np.all(np.abs(out - rows @ a) <= bound), name


def test_sums_x_is_the_sums():
    rng = np.random.default_rng(1)
    xq = rng.integers(-127, 128, 512).astype(np.int8)
    xs = rng.random(16).astype(np.float32)
    out = O.sums_x(xs, xq)
    assert np.array_equal(out[:16], xs)
    s16 = out[16:16 + 16].view(np.int16)
    s8 = out[32:32 + 32].view(np.int16)
    assert np.array_equal(s16, xq.reshape(-1, 16).astype(np.int32).sum(axis=1))
    assert np.array_equal(s8, xq.reshape(-1, 8).astype(np.int32).sum(axis=1))
