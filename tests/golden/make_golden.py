"""Generates tests/golden/golden.npz: the known answers the CPU oracle is pinned to before it is trusted.

Run in a container that holds the reference read-only (its path in the environment variable PLLM_REFERENCE, which must be set):
    python tests/golden/make_golden.py
The output is committed; no test reads the reference at run time.

Two kinds of answers:
  1. Bytes and floats of the reference's own NumPy code, imported from the reference tree and run here:
     src/python/engine/packing.py (quantize :40-45, six :83-86 with pack6 :56-63 / unpack6 :66-71, ternary
     :117-127, binary :167-177) and src/python/engine/layers.py (rmsnorm :44-45, head_norm :48-51, rope :362-369,
     silu :127-128, delta_rule :149-156), plus the attention of src/python/engine/model.py:532-538 written with the
     same NumPy expressions on the same arrays.
  2. Bit-exact answers of the reference's kernel tests' written-out models (the TypeScript tests cannot run here: no
     Node/Bun): tests/int8-check.ts:65-91 (matmul_q8r and matmul_q8, float32 in the kernels' order), :232-265
     (quantize_x at both biases), tests/ternary-check.ts:84-101 (interleave) and :118-129 (matmul_t2 / t2r). Those
     models are ported below to NumPy float32 scalars (each JavaScript Math.fround of a double sum or product is the
     float32 operation: double holds the exact result of one float32 add or multiply before its single rounding).
     Inputs come from the tests' LCG (tests/int8-check.ts:117) and follow their edge cases: weights at both ends and
     alternating, activations at both ends, zero and subnormal scales, rows of 1..9, 12, 13 and 81 groups.
"""
import os
import sys

import numpy as np

REF = os.environ.get("PLLM_REFERENCE")
if not REF:
    sys.exit("set PLLM_REFERENCE to the reference's source tree (read-only)")
sys.path.insert(0, os.path.join(REF, "src", "python"))
from engine import layers, packing  # noqa: E402  (the reference's own NumPy)

f32 = np.float32
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")


class Lcg:
    """tests/int8-check.ts:116-117: seed = seed * 1103515245 + 12345 (mod 2^32), each draw the seed >> 8."""

    def __init__(self, seed):
        self.seed = seed

    def next(self):
        self.seed = (self.seed * 1103515245 + 12345) & 0xFFFFFFFF
        return self.seed >> 8


def scale_of(rng, i):
    """int8-check.ts:83: a subnormal one in eleven, a zero one in thirteen, else 1e-3 .. 1."""
    if i % 11 == 7:
        return f32(2.0 ** -130 * (1 + rng.next() % 1000))
    if i % 13 == 5:
        return f32(0.0)
    return f32(1e-3 * (1 + rng.next() % 1000))


def nearest(v):
    return np.rint(v)  # round half to even, as f32x4.nearest


def quantize_model(x, bias):
    """int8-check.ts:244-257: the scalar steps of quantize_x, group by group."""
    qmax = f32(127.0 if bias == 0 else 63.0)
    n = x.size
    xq = np.zeros(n, np.uint8)
    xs = np.zeros(n // 32, np.float32)
    for g in range(n // 32):
        grp = x[g * 32:(g + 1) * 32]
        largest = f32(np.max(np.abs(grp)))
        s = f32(largest / qmax)
        inv = f32(f32(1.0) / s) if s > 0 else f32(0.0)
        xs[g] = s
        for j in range(32):
            with np.errstate(over="ignore", invalid="ignore"):
                v = nearest(f32(grp[j] * inv))
            t = 0 if np.isnan(v) else int(max(-(2 ** 31), min(2 ** 31 - 1, float(v))))
            w = ((t + bias + 2 ** 31) % 2 ** 32) - 2 ** 31  # the bias added in int32, wrapping
            xq[j + 32 * g] = max(-128, min(127, w)) & 0xFF
    return xq, xs


def q8r_model(w, q, ws, xs, ng):
    """int8-check.ts:65-77."""
    ng4 = ng & ~3
    lanes = [f32(0)] * 4
    exact = (w.reshape(ng, 32).astype(np.int64) * (q.reshape(ng, 32).astype(np.int64) - 64)).sum(axis=1)
    g = 0
    while g < ng4:
        lanes[g & 3] = f32(lanes[g & 3] + f32(f32(exact[g]) * f32(ws[g] * xs[g])))
        g += 1
    s = f32(f32(f32(lanes[0] + lanes[1]) + lanes[2]) + lanes[3])
    while g < ng:
        s = f32(s + f32(f32(exact[g]) * f32(ws[g] * xs[g])))
        g += 1
    return s


def q8_model(w, q, ws, xs, ng):
    """int8-check.ts:79-91: lane k holds products 2k, 2k+1, 2k+8, 2k+9 of each half of a group."""
    lanes = [f32(0)] * 4
    prod = w.reshape(ng, 32).astype(np.int64) * q.reshape(ng, 32).astype(np.int64)
    for g in range(ng):
        s = f32(ws[g] * xs[g])
        for k in range(4):
            idx = [h + p for h in (0, 16) for p in (2 * k, 2 * k + 1, 2 * k + 8, 2 * k + 9)]
            lanes[k] = f32(lanes[k] + f32(f32(prod[g, idx].sum()) * s))
    return f32(f32(f32(lanes[0] + lanes[1]) + lanes[2]) + lanes[3])


def pack6_bytes(values):
    """int8-check.ts:55-62 (the bytes of llama2_numpy.pack6)."""
    return packing.pack6(values).reshape(-1)


def int8_cases(G):
    rng = Lcg(644)
    rows, tokens = 13, 9
    for ng in (1, 2, 3, 4, 5, 6, 7, 8, 9, 12, 13, 81):
        n = ng * 32
        w8 = np.array([(rng.next() & 255) - 128 for _ in range(rows * n)], np.int8)
        v6 = np.array([4 * ((rng.next() & 63) - 32) for _ in range(rows * n)], np.int8)
        w8[:n] = 127
        w8[n:2 * n] = -128
        v6[:n] = 124
        v6[n:2 * n] = -128
        w8[2 * n:3 * n] = np.where(np.arange(n) & 1, 127, -128)
        v6[2 * n:3 * n] = np.where(np.arange(n) & 1, 124, -128)
        ws = np.array([scale_of(rng, i) for i in range(rows * ng)], np.float32)
        # relaxed activations 0..127: all 127, all 0, alternating, quantize_x(bias 64) of random floats, random
        qr = np.zeros((tokens, n), np.uint8)
        xr = np.zeros((tokens, ng), np.float32)
        xf = np.array([f32(((rng.next() % 2001) - 1000) * 1e-3 * (1 + (j % 5))) for j in range(n)], np.float32)
        for t in range(tokens):
            if t == 3:
                qr[t], xr[t] = quantize_model(xf, 64)
                continue
            if t == 0:
                qr[t] = 127
            elif t == 1:
                qr[t] = 0
            elif t == 2:
                qr[t] = np.where(np.arange(n) & 1, 127, 0)
            else:
                qr[t] = [rng.next() & 127 for _ in range(n)]
            xr[t] = [scale_of(rng, g + t) for g in range(ng)]
        # plain activations -127..127
        qp = np.zeros((tokens, n), np.int8)
        xp = xr.copy()
        for t in range(tokens):
            if t == 3:
                b, xp[t] = quantize_model(xf, 0)
                qp[t] = b.view(np.int8)
            elif t == 0:
                qp[t] = 127
            elif t == 1:
                qp[t] = -127
            elif t == 2:
                qp[t] = np.where(np.arange(n) & 1, 127, -127)
            else:
                qp[t] = [(rng.next() % 255) - 127 for _ in range(n)]
        want = {}
        for name, weights, model, acts, scales in (("q8r", w8, q8r_model, qr, xr), ("q6r", v6, q8r_model, qr, xr),
                                                     ("q8", w8, q8_model, qp, xp), ("q6", v6, q8_model, qp, xp)):
            want[name] = np.array([[model(weights[i * n:(i + 1) * n], acts[t], ws[i * ng:(i + 1) * ng], scales[t], ng)
                                    for i in range(rows)] for t in range(tokens)], np.float32)
        key = f"int8_ng{ng}_"
        G[key + "w8"] = w8.reshape(rows, n)
        G[key + "w6"] = pack6_bytes(v6.reshape(-1, 32))
        G[key + "ws"] = ws
        G[key + "qr"], G[key + "xr"], G[key + "qp"], G[key + "xp"] = qr, xr, qp, xp
        for name, v in want.items():
            G[key + name] = v


def quantize_cases(G):
    """int8-check.ts:232-265: groups of every size, zeros, -0, the ends at both places, half steps."""
    rng = Lcg(232)
    groups = 12
    x = np.zeros(groups * 32, np.float32)
    sizes = [1, 3.0000002, 1e-30, 65504, 1.5e-5, 2 ** -140]
    for g in range(groups):
        size = sizes[g % 6]
        for j in range(32):
            x[g * 32 + j] = 0.0 if g == 4 else (-0.0 if g == 5 else f32(((rng.next() % 2001) - 1000) * 1e-3 * size))
    x[6 * 32], x[6 * 32 + 31] = -3.0, 3.0
    for j in range(1, 31):
        x[7 * 32 + j] = (j - 15) * 0.5
    x[7 * 32], x[7 * 32 + 31] = 63.0, -63.0
    G["quant_x"] = x
    for bias in (0, 64):
        G[f"quant_q{bias}"], G[f"quant_s{bias}"] = quantize_model(x, bias)


def ternary_cases(G):
    """ternary-check.ts:84-129: interleave, then matmul_t2 / t2r against its written-out model; binary (binary.ts)
    takes the same integers for weights of -1 and +1 (codes 0 and 2)."""
    rng = Lcg(231)
    rows = 13
    for groups in (1, 2, 3, 4, 5, 7, 9):
        n = groups * 128
        ng = n // 32
        codes = np.array([rng.next() & 3 for _ in range(rows * n)], np.uint8)
        codes[:128] = 2
        if groups > 1:
            codes[n + 128:n + 256] = 0
        halves = np.zeros(rows * groups, np.float16)
        for g in range(rows * groups):
            v = 2.0 ** -20 * (1 + rng.next() % 1000) if g % 11 == 7 else (0.0 if g % 13 == 5 else 1e-3 * (1 + rng.next() % 1000))
            halves[g] = np.float16(v)
        a = np.array([(rng.next() & 255) - 128 for _ in range(n)], np.int8)
        a[:64] = 127
        a[64:128] = -128
        if groups > 1:
            a[128:256] = -128
        xs = np.array([f32(1e-2 * (1 + rng.next() % 1000)) for _ in range(ng)], np.float32)
        packed = np.zeros(rows * n // 4, np.uint8)
        for j in range(rows * n):
            packed[j >> 2] |= codes[j] << (2 * (j & 3))
        bcodes = np.where(codes >= 2, 2, 0).astype(np.uint8)  # binary: weights +1 (code 2) and -1 (code 0)
        signs = (bcodes.astype(np.int8) - 1).reshape(-1, 128)
        bpacked = packing.pack_binary(signs).reshape(-1)
        # interleave (ternary-check.ts:98-107): the bytes and the minus-sums
        il = np.zeros(n, np.int8)
        for at in range(n):
            il[at] = a[(at & ~63) + 4 * (at & 15) + ((at >> 4) & 3)]
        sums = np.array([-int(a[g * 32:(g + 1) * 32].astype(np.int64).sum()) for g in range(ng)], np.int32)

        def model(cd):
            out = np.zeros(rows, np.float32)
            for i in range(rows):
                lanes = [f32(0)] * 4
                for g in range(groups):
                    d = f32(halves[i * groups + g])
                    for lane in range(4):
                        j0 = g * 128 + lane * 32
                        s = int(((cd[i * n + j0:i * n + j0 + 32].astype(np.int64) - 1) * a[j0:j0 + 32]).sum())
                        lanes[lane] = f32(lanes[lane] + f32(f32(f32(s) * xs[g * 4 + lane]) * d))
                out[i] = f32(f32(f32(lanes[0] + lanes[1]) + lanes[2]) + lanes[3])
            return out

        key = f"tern_g{groups}_"
        G[key + "packed"], G[key + "bpacked"], G[key + "halves"] = packed, bpacked, halves.view(np.uint16)
        G[key + "a"], G[key + "xs"], G[key + "il"], G[key + "sums"] = a, xs, il, sums
        G[key + "t2"], G[key + "b1"] = model(codes), model(bcodes)


def packing_cases(G):
    rng = np.random.default_rng(0)
    x = (rng.normal(0, 0.02, (8, 256))).astype(np.float32)
    G["pack_x"] = x
    G["pack_q8"], G["pack_s8"] = packing.quantize(x)
    six_bytes, six_scales = packing.six(x)
    G["pack_six"], G["pack_six_s"] = six_bytes.reshape(-1), six_scales
    G["pack_six_values"] = packing.unpack6(six_bytes).reshape(-1)
    t = rng.integers(-1, 2, (8, 256)).astype(np.float32)
    tscale = np.float16(rng.normal(0.02, 0.002, (16, 1))).astype(np.float32)
    tv = (t.reshape(16, 128) * tscale).reshape(8, 256)
    tb, th = packing.ternary(tv)
    G["pack_tern_values"], G["pack_tern"], G["pack_tern_s"] = t.astype(np.int8), tb.reshape(-1), th.view(np.uint16)
    bsign = np.where(rng.integers(0, 2, (8, 256)) > 0, 1, -1).astype(np.float32)
    bv = (bsign.reshape(16, 128) * tscale).reshape(8, 256)
    bb, bh = packing.binary(bv)
    G["pack_bin_values"], G["pack_bin"], G["pack_bin_s"] = bsign.astype(np.int8), bb.reshape(-1), bh.view(np.uint16)


def float_cases(G):
    rng = np.random.default_rng(7)
    dim, hs = 288, 48
    x = rng.normal(0, 1, dim).astype(np.float32)
    w = rng.normal(1, 0.1, dim).astype(np.float32)
    G["rms_x"], G["rms_w"] = x, w
    G["rms_out"] = layers.rmsnorm(x, w, 1e-5).astype(np.float32)
    qn = rng.normal(1, 0.1, hs).astype(np.float32)
    G["head_w"] = qn
    G["head_out"] = layers.head_norm(x, qn, 1e-6).astype(np.float32)
    pos = 5
    freqs = layers.rope_frequencies(hs, 10000.0)
    cos, sin = np.cos(pos * freqs).astype(np.float32), np.sin(pos * freqs).astype(np.float32)
    G["rope_cos"], G["rope_sin"] = cos, sin
    G["rope_out"] = layers.rope(x.reshape(-1, hs), cos, sin).reshape(-1).astype(np.float32)
    h1 = rng.normal(0, 2, 768).astype(np.float32)
    h3 = rng.normal(0, 1, 768).astype(np.float32)
    G["swiglu_h1"], G["swiglu_h3"] = h1, h3
    G["swiglu_out"] = (layers.silu(h1) * h3).astype(np.float32)
    # the delta rule (layers.py:149-156), Qwen3.5-like heads: kh 2, vh 4, kd vd 16
    kh, vh, kd, vd = 2, 4, 16, 16
    state = rng.normal(0, 0.5, (vh, kd, vd)).astype(np.float32)
    qk = rng.normal(0, 0.3, (2 * kh, kd)).astype(np.float32)
    v = rng.normal(0, 1, (vh, vd)).astype(np.float32)
    beta = rng.uniform(0.1, 0.9, vh).astype(np.float32)
    decay = rng.uniform(0.5, 1.0, vh).astype(np.float32)
    G["delta_state"], G["delta_qk"], G["delta_v"], G["delta_beta"], G["delta_decay"] = state, qk, v, beta, decay
    each = vh // kh
    qh = np.repeat(qk[:kh], each, axis=0)
    kk = np.repeat(qk[kh:], each, axis=0)
    s2 = state.copy()
    G["delta_out"] = layers.delta_rule(s2, qh, kk, v, beta, decay).astype(np.float32).reshape(-1)
    G["delta_next"] = s2.reshape(-1)
    # attention (model.py:532-538): GQA 6 q heads over 2 kv heads of 16, 21 positions
    nh, nkv, size, count = 6, 2, 16, 21
    q = rng.normal(0, 1, nh * size).astype(np.float32)
    keys = rng.normal(0, 1, (nkv, count, size)).astype(np.float32)
    values = rng.normal(0, 1, (nkv, count, size)).astype(np.float32)
    qq = q.reshape(nkv, nh // nkv, size)
    att = (qq @ keys.transpose(0, 2, 1)) * np.float32(1.0 / np.sqrt(size))
    att = np.exp(att - att.max(axis=-1, keepdims=True))
    att /= att.sum(axis=-1, keepdims=True)
    G["att_q"], G["att_k"], G["att_v"] = q, keys, values
    G["att_out"] = (att @ values).reshape(-1).astype(np.float32)


def main():
    G = {}
    packing_cases(G)
    quantize_cases(G)
    int8_cases(G)
    ternary_cases(G)
    float_cases(G)
    np.savez_compressed(OUT, **G)
    print(f"wrote {OUT}: {len(G)} arrays, {os.path.getsize(OUT)} bytes")


if __name__ == "__main__":
    main()
