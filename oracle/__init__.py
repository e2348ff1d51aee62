"""TEST INFRASTRUCTURE ONLY: the CPU oracle, a C restatement of the reference's kernels (pllm_oracle.c), via ctypes.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and reference legs may import this module. The
product (the CUDA library and its host driver) never does: it fails loudly when its own extension is missing.

Every function takes NumPy arrays and returns new arrays; the argument names and meanings are the reference kernels'
(kernels/kernel/*.ts, kernels/relaxed/*.ts), with the addresses replaced by arrays.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_lib = None


def build():
    """Compile liboracle.so with the committed Makefile (gcc; no GPU needed)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = ctypes.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P, I32, F32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_float


def _declare(L):
    sig = {
        "or_fexp": ([F32], F32), "or_vexp": ([F32], F32), "or_half": ([ctypes.c_uint16], F32),
        "or_quantize_x": ([P, P, P, I32, I32], None), "or_int8_sums": ([P, P, I32], None),
        "or_six_sums": ([P, P, I32], None), "or_interleave": ([P, P, I32], None), "or_widen6": ([P, P], None),
        "or_matmul_q8": ([P, P, P, P, P, I32, I32, I32], None),
        "or_matmul_q8r": ([P, P, P, P, P, P, I32, I32, I32], None),
        "or_matmul_q8r_tile": ([P, P, P, P, P, P, I32, I32, I32, I32, I32, I32], None),
        "or_matmul_q6": ([P, P, P, P, P, I32, I32, I32], None),
        "or_matmul_q6r": ([P, P, P, P, P, P, I32, I32, I32], None),
        "or_matmul_signs": ([P, P, P, P, P, I32, I32, I32, I32, I32], None),
        "or_matmul_signs_tile": ([P, P, P, P, P, I32, I32, I32, I32, I32, I32, I32, I32], None),
        "or_matmul_f32": ([P, P, P, I32, I32, I32], None),
        "or_group_sums_q8": ([P, P, P, I32, I32, I32, I32], None),
        "or_group_sums_q6": ([P, P, P, I32, I32, I32, I32], None),
        "or_group_sums_signs": ([P, P, P, P, I32, I32, I32, I32, I32], None),
        "or_rope": ([P, P, P, I32, I32, I32], None),
        "or_attention": ([P, P, P, P, P, I32, I32, I32, I32, I32, I32, I32, F32], None),
        "or_to_f16": ([P, P, I32], I32), "or_from_f16": ([P, P, I32], None), "or_finite_f16": ([P, I32], I32),
        "or_rmsnorm": ([P, P, P, I32, F32], None), "or_swiglu": ([P, P, P, I32], None),
        "or_add_inplace": ([P, P, I32], None), "or_gate": ([P, P, P, I32], None),
        "or_convolve": ([P, P, P, I32, I32], None), "or_short_conv": ([P, P, P, P, I32, I32], None),
        "or_delta_rule": ([P, P, P, P, P, I32, I32, I32, I32, I32, I32], None),
        "or_forward": ([P, P, I32, I32, P, I32], I32), "or_threads": ([], I32),
        "or_argmax": ([P, I32], I32), "or_penalize": ([P, P, I32, F32, F32], None),
        "or_sample": ([P, I32, F32, F32, ctypes.c_double, I32, F32], I32),
        "or_sb_size": ([I32], I32), "or_sb_tables": ([P, P], I32), "or_sums_x": ([P, P, I32], None),
        "or_matmul_sb": ([P, P, P, P, P, I32, I32, I32, I32], None), "or_sb_row": ([P, P, P, I32, I32], None),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes, fn.restype = args, res


def _p(a):
    # a pointer that holds the array (a temporary made by _c lives until the call returns)
    return a.ctypes.data_as(ctypes.c_void_p) if a is not None else None


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ---- activations
def quantize_x(x, bias=0):
    """quantize.ts:124-151 -> (xq uint8 bytes, xs float32 scales). Bytes are int8 for bias 0, 1..127 for bias 64."""
    x = _c(x, np.float32)
    n = x.shape[-1]
    xq = np.zeros(n, np.uint8)
    xs = np.zeros(n // 32, np.float32)
    lib().or_quantize_x(_p(xq), _p(xs), _p(x), n, bias)
    return xq, xs


def int8_sums(w):
    w = _c(w, np.int8).reshape(-1)
    out = np.zeros(w.size // 32, np.int32)
    lib().or_int8_sums(_p(out), _p(w), out.size)
    return out


def six_sums(w6):
    w6 = _c(w6, np.uint8).reshape(-1)
    out = np.zeros(w6.size // 24, np.int32)
    lib().or_six_sums(_p(out), _p(w6), out.size)
    return out


def interleave(xq, xs):
    """matmul.ts:129-146 -> (interleaved bytes, xs extended by the int32 minus-sums as float32 bit patterns)."""
    xq = _c(xq, np.uint8).copy()
    n = xq.size
    ext = np.zeros(2 * (n // 32), np.float32)
    ext[: n // 32] = xs
    lib().or_interleave(_p(xq), _p(ext), n)
    return xq, ext


def widen6(packed):
    packed = _c(packed, np.uint8).reshape(-1, 24)
    out = np.zeros((packed.shape[0], 32), np.int8)
    for g in range(packed.shape[0]):
        lib().or_widen6(out[g].ctypes.data, packed[g].ctypes.data)
    return out.reshape(-1)


# ---- products
def matmul_q8(xq, xs, wq, ws, r0=0, r1=None):
    wq = _c(wq, np.int8)
    rows, n = wq.shape
    r1 = rows if r1 is None else r1
    out = np.zeros(rows, np.float32)
    lib().or_matmul_q8(_p(out), _p(_c(xq, np.uint8)), _p(_c(xs, np.float32)), _p(wq), _p(_c(ws, np.float32)), n, r0, r1)
    return out


def matmul_q8r(xq, xs, wq, ws, wc=None, r0=0, r1=None):
    wq = _c(wq, np.int8)
    rows, n = wq.shape
    r1 = rows if r1 is None else r1
    out = np.zeros(rows, np.float32)
    wc = None if wc is None else _c(wc, np.int32)
    lib().or_matmul_q8r(_p(out), _p(_c(xq, np.uint8)), _p(_c(xs, np.float32)), _p(wq), _p(_c(ws, np.float32)), _p(wc),
                        n, r0, r1)
    return out


def matmul_q8r_tile(frames, wq, ws, n, r0, r1, count, os_, frame, xs_at=4096):
    """relaxed/int8.ts:147-166: count tokens, token t's activations at byte t frame of frames (its scales xs_at bytes
    further), its outputs os bytes apart -> (count, rows) outputs (rows r0..r1 written, the rest zero)."""
    wq = _c(wq, np.int8).reshape(-1, n)
    rows = wq.shape[0]
    frames = _c(frames, np.uint8)
    out = np.zeros(count * os_ // 4, np.float32)
    base = frames.ctypes.data
    lib().or_matmul_q8r_tile(_p(out), ctypes.c_void_p(base), ctypes.c_void_p(base + xs_at), _p(wq),
                             _p(_c(ws, np.float32)), None, n, r0, r1, count, os_, frame)
    return out.reshape(count, os_ // 4)[:, :rows]


def matmul_q6(xq, xs, w6, ws, n, r0=0, r1=None):
    w6 = _c(w6, np.uint8)
    rows = w6.size // (n // 32 * 24)
    r1 = rows if r1 is None else r1
    out = np.zeros(rows, np.float32)
    lib().or_matmul_q6(_p(out), _p(_c(xq, np.uint8)), _p(_c(xs, np.float32)), _p(w6), _p(_c(ws, np.float32)), n, r0, r1)
    return out


def matmul_q6r(xq, xs, w6, ws, n, wc=None, r0=0, r1=None):
    w6 = _c(w6, np.uint8)
    rows = w6.size // (n // 32 * 24)
    r1 = rows if r1 is None else r1
    out = np.zeros(rows, np.float32)
    wc = None if wc is None else _c(wc, np.int32)
    lib().or_matmul_q6r(_p(out), _p(_c(xq, np.uint8)), _p(_c(xs, np.float32)), _p(w6), _p(_c(ws, np.float32)), _p(wc),
                        n, r0, r1)
    return out


def matmul_signs(xq_il, xs_ext, wq, ws16, n, binary=False, r0=0, r1=None):
    """matmul_t2 / t2r (binary=False, code 3) or matmul_b1 / b1r (binary=True, code 2) on interleaved activations."""
    wq = _c(wq, np.uint8)
    rows = wq.size // (n // (8 if binary else 4))
    r1 = rows if r1 is None else r1
    out = np.zeros(rows, np.float32)
    lib().or_matmul_signs(_p(out), _p(_c(xq_il, np.uint8)), _p(_c(xs_ext, np.float32)), _p(wq),
                          _p(_c(ws16, np.uint16)), n, r0, r1, 2 if binary else 3, int(binary))
    return out


def matmul_f32(x, w, r0=0, r1=None):
    w = _c(w, np.float32)
    rows, n = w.shape
    r1 = rows if r1 is None else r1
    out = np.zeros(rows, np.float32)
    lib().or_matmul_f32(_p(out), _p(_c(x, np.float32)), _p(w), n, r0, r1)
    return out


def group_sums_q8(xq, wq, bias=0):
    wq = _c(wq, np.int8)
    rows, n = wq.shape
    out = np.zeros((rows, n // 32), np.int32)
    lib().or_group_sums_q8(_p(out), _p(_c(xq, np.uint8)), _p(wq), n, 0, rows, bias)
    return out


def group_sums_q6(xq, w6, n, bias=0):
    w6 = _c(w6, np.uint8)
    rows = w6.size // (n // 32 * 24)
    out = np.zeros((rows, n // 32), np.int32)
    lib().or_group_sums_q6(_p(out), _p(_c(xq, np.uint8)), _p(w6), n, 0, rows, bias)
    return out


def group_sums_signs(xq_il, xs_ext, wq, n, binary=False):
    wq = _c(wq, np.uint8)
    rows = wq.size // (n // (8 if binary else 4))
    out = np.zeros((rows, n // 32), np.int32)
    lib().or_group_sums_signs(_p(out), _p(_c(xq_il, np.uint8)), _p(_c(xs_ext, np.float32)), _p(wq), n, 0, rows,
                              2 if binary else 3, int(binary))
    return out


# ---- attention, rope, halves
def rope(v, fcr, fci, nh, hs, rot=0):
    v = _c(v, np.float32).copy()
    lib().or_rope(_p(v), _p(_c(fcr, np.float32)), _p(_c(fci, np.float32)), nh, hs, rot)
    return v


def attention(q, kc, vc, pos, nh, nkv, hs, half=False, cap=0.0, h0=0, h1=None):
    """attention.ts:87-211. kc, vc: [positions][nkv * hs] float32, or uint16 float16 bits when half."""
    h1 = nh if h1 is None else h1
    kc = _c(kc, np.uint16 if half else np.float32)
    vc = _c(vc, np.uint16 if half else np.float32)
    out = np.zeros(nh * hs, np.float32)
    att = np.zeros(nh * (pos + 1), np.float32)
    lib().or_attention(_p(out), _p(_c(q, np.float32)), _p(kc), _p(vc), _p(att), pos, nh, nkv, hs, h0, h1, int(half),
                       float(cap))
    return out, att


def to_f16(x):
    x = _c(x, np.float32)
    out = np.zeros(x.size, np.uint16)
    bad = lib().or_to_f16(_p(out), _p(x), x.size)
    return out, bad


def from_f16(h):
    h = _c(h, np.uint16)
    out = np.zeros(h.size, np.float32)
    lib().or_from_f16(_p(out), _p(h), h.size)
    return out


def finite_f16(h):
    h = _c(h, np.uint16)
    return lib().or_finite_f16(_p(h), h.size)


# ---- glue and stateful layers
def rmsnorm(x, w, eps):
    x = _c(x, np.float32)
    out = np.zeros_like(x)
    lib().or_rmsnorm(_p(out), _p(x), _p(_c(w, np.float32)), x.size, eps)
    return out


def swiglu(h1, h3):
    h1 = _c(h1, np.float32)
    out = np.zeros_like(h1)
    lib().or_swiglu(_p(out), _p(h1), _p(_c(h3, np.float32)), h1.size)
    return out


def add_inplace(x, y):
    x = _c(x, np.float32).copy()
    lib().or_add_inplace(_p(x), _p(_c(y, np.float32)), x.size)
    return x


def argmax(x):
    """sample.ts:6-10"""
    x = _c(x, np.float32)
    return int(lib().or_argmax(_p(x), x.size))


def penalize(logits, tokens, penalty, presence):
    """sample.ts:16-30 (a copy of the logits, penalized)"""
    out = _c(logits, np.float32).copy()
    t = _c(tokens, np.int32)
    lib().or_penalize(_p(out), _p(t), t.size, penalty, presence)
    return out


def sample(logits, temperature, topp, random, topk=0, minp=0.0):
    """sample.ts:248-337: the token drawn with this random number in [0, 1) (-1: the largest logit is not finite)"""
    x = _c(logits, np.float32)
    return int(lib().or_sample(_p(x), x.size, temperature, topp, float(random), topk, minp))


SB_TABLES = 34992  # sb_tables' bytes (blocks/types.ts:94)


def sb_tables(codebooks):
    """blocks/types.ts:294-322: the kernels' tables from the checkpoint's codebooks row (uint8)"""
    area = np.zeros(SB_TABLES, np.uint8)
    lib().or_sb_tables(_p(area), _p(_c(codebooks, np.uint8)))
    return area


def sums_x(xs, xq):
    """blocks/token.ts:158-172: the scales followed by the int16 sums of each 16 and each 8 activations"""
    n = xq.size
    out = np.zeros(n // 32 + n // 16 // 2 + n // 8 // 2, np.float32)
    out[:n // 32] = xs
    lib().or_sums_x(_p(out), _p(_c(xq, np.int8)), n)
    return out


def matmul_sb(xq, xs, w, tab, n, rows, btype):
    """blocks/token.ts:130-141: one token against rows of n weights in llama.cpp's blocks of btype"""
    out = np.zeros(rows, np.float32)
    lib().or_matmul_sb(_p(out), _p(_c(xq, np.int8)), _p(_c(xs, np.float32)), _p(_c(w, np.uint8)),
                       _p(_c(tab, np.uint8)), n, 0, rows, btype)
    return out


def sb_row(w, tab, n, btype):
    """blocks/row.ts: a row of n weights in blocks of btype as float32"""
    out = np.zeros(n, np.float32)
    lib().or_sb_row(_p(out), _p(_c(w, np.uint8)), _p(_c(tab, np.uint8)), n, btype)
    return out


def gate(x, g):
    x = _c(x, np.float32)
    out = np.zeros_like(x)
    lib().or_gate(_p(out), _p(x), _p(_c(g, np.float32)), x.size)
    return out


def convolve(taps, rows):
    taps, rows = _c(taps, np.float32), _c(rows, np.float32)
    count, n = rows.shape
    out = np.zeros(n, np.float32)
    lib().or_convolve(_p(out), _p(taps), _p(rows), n, count)
    return out


def short_conv(taps, rows, b):
    """-> (out, rows with the newest row written)"""
    taps, rows, b = _c(taps, np.float32), _c(rows, np.float32).copy(), _c(b, np.float32)
    count, n = rows.shape
    out = np.zeros(n, np.float32)
    lib().or_short_conv(_p(out), _p(taps), _p(rows), _p(b), n, count)
    return out, rows


def delta_rule(state, c, work, kh, kd, vd, vh, h0=0, h1=None):
    """stateful.ts:96-151 -> (out, next, work after the call)."""
    h1 = vh if h1 is None else h1
    state, c, work = _c(state, np.float32), _c(c, np.float32), _c(work, np.float32).copy()
    nxt = np.zeros_like(state)
    out = np.zeros(vh * vd, np.float32)
    lib().or_delta_rule(_p(out), _p(state), _p(nxt), _p(c), _p(work), kh, kd, vd, vh, h0, h1)
    return out, nxt, work


# ---- the decoder forward (the CPU baseline and the model-level check)
class Config(ctypes.Structure):
    _fields_ = [(k, I32) for k in ("dim", "hidden", "layers", "heads", "kv_heads", "head_size", "vocab", "seq_len",
                                   "qk_norm", "relaxed", "half_kv")] + [("eps", F32)]


class Weights(ctypes.Structure):
    _fields_ = [(k, P) for k in ("wq", "wk", "wv", "wo", "w1", "w2", "w3", "sq", "sk", "sv", "so", "s1", "s2", "s3",
                                 "cq", "ck", "cv", "co", "c1", "c2", "c3", "emb", "emb_s", "cls", "cls_s", "cls_c",
                                 "att_norm", "ffn_norm", "final_norm", "q_norm", "k_norm", "cos_t", "sin_t", "kc", "vc")]


def threads():
    return lib().or_threads()


def forward(config, arrays, token, pos, nthreads=0):
    """One decode step. config: Config; arrays: dict of NumPy arrays by the Weights field names (kept alive by the
    caller; kc/vc are written at pos). Returns the logits."""
    w = Weights(**{k: (v.ctypes.data if v is not None else None) for k, v in arrays.items()})
    logits = np.zeros(config.vocab, np.float32)
    rc = lib().or_forward(ctypes.byref(config), ctypes.byref(w), token, pos, _p(logits), nthreads)
    if rc != 0:
        raise ValueError("oracle forward: bad arguments")
    return logits
