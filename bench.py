#!/usr/bin/env python
"""bench.py: batch-1 int8 decode of the Qwen3-8B-shaped configuration on B200s.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one decode token of the 36-layer model (8.51 GB of int8 weights and scales, a float16 KV cache) at positions
2048 onward, after a 2048-token prompt has filled the cache. Weights are seeded synthetic N(0, 0.02) int8 (the
reference's group-of-32 format); the prompt is seeded random ids. Prints one JSON line (rank 0):
  value       decode tok/s of the whole job, device-timed (CUDA events on the engine's stream), each step's token and
              position already in device memory; the 8.5 GB of weights (> the 126 MB L2) stream from HBM every step
  e2e         the same through the engine's public call: at N = 1 Engine.next_token(token, pos), the greedy step (the
              token and position copied from pinned host memory, 8 bytes, and the next token back, 4 bytes, every
              step: the argmax runs on the device); at N > 1 the same call on every rank (each rank's vocab slice
              gives its largest as a key; the keys' max is an NCCL all-reduce on the devices; 4 bytes back a rank)
  roofline    the dominant kernel (the fused w1/w3 product: 2 x 12288 x 4096 int8 + scales, SwiGLU epilogue), its
              algorithmic bytes a launch over its CUDA-event duration, against MEASURED_PEAKS.json's HBM copy GB/s
  cpu_baseline  the CPU oracle (the reference kernels' arithmetic in C, OpenMP over rows) decoding the same model
              on the host cores, a bounded sample of tokens (rank 0, N = 1)
Under torchrun (N > 1) the ranks decode one stream together, tensor-parallel (pllm.tp: each GPU holds 1/N of every
matrix and its heads' cache; the two reductions a layer go over NVLink in the products' epilogues and prologues;
the prompt's prefill on the tensor cores, its row-parallel partials summed by NCCL all-reduces): scaling "strong" (the
work of a token is fixed), value = tokens / the slowest rank's time.

--impl reference: the reference's CPU implementation of the path, timed on the host cores: its kernels are
AssemblyScript compiled to WASM and cannot run on this image (no Node, Bun or AssemblyScript), so the oracle's C
restatement of them runs instead, on all host threads, on the same config and metric (rank 0 alone under torchrun).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (ROOT, os.path.join(ROOT, "pyodide-llm_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402

METRIC = "int8 decode tok/s (batch 1) + prefill tok/s; GEMV HBM GB/s vs 8 TB/s peak"
PROMPT = 2048


def kernel_case(which):
    """A kernel's small case for profiling, three launches: the prefill product at M 512, N 4096, K 4096 (a wo-sized
    product; 21 MB of weights, > L2 after the first pass is not needed: one launch is captured), or the forward step's
    attention at position 2559 of the Qwen3-8B shape (32 / 8 heads of 128, a float16 cache of 2560 positions)."""
    from pllm.device import Buffer, init
    from pllm.lib import L, check
    init(0)
    L.pllm_set_stream(0)
    bufs = []
    if which == "gemv":  # the decode step's w1/w3 product (rows 2 x 12288, K 4096: 113 MB > L2), RMSNorm and SwiGLU
        from pllm.forward import F_Q8
        hidden, K = 12288, 4096
        w, ws = Buffer(2 * hidden * K), Buffer(2 * hidden * K // 8)
        x, norm, out = Buffer(K * 4), Buffer(K * 4), Buffer(hidden * 4)
        bufs += [w, ws, x, norm, out]
        L.pllm_synth_q8(w.ptr, ws.ptr, 2 * hidden, K, 1, 0.02)
        L.pllm_synth_f32(x.ptr, K, 2, 0.0, 1.0)
        L.pllm_synth_f32(norm.ptr, K, 3, 1.0, 0.1)
        for _ in range(3):
            L.pllm_gemv(out.ptr, 0, 0, 0, 0, 0, x.ptr, 0, norm.ptr, 1e-6, 0, w.ptr, ws.ptr, F_Q8, K, 0, hidden, 1, 1, 2,
                        hidden, 0)
    elif which in ("qkv", "wo", "w2"):  # the step's other int8 products at the Qwen3-8B shape, one token
        # qkv: rows 6144, K 4096, RMSNorm prologue; wo: rows 4096, K 4096 and w2: rows 4096, K 12288, quantize_x
        # prologue and the residual add
        rows, K, pro, epi = {"qkv": (6144, 4096, 1, 0), "wo": (4096, 4096, 2, 1), "w2": (4096, 12288, 2, 1)}[which]
        w, ws = Buffer(rows * K), Buffer(rows * K // 8)
        x, norm, out = Buffer(K * 4), Buffer(K * 4), Buffer(rows * 4)
        bufs += [w, ws, x, norm, out]
        L.pllm_synth_q8(w.ptr, ws.ptr, rows, K, 1, 0.02)
        L.pllm_synth_f32(x.ptr, K, 2, 0.0, 1.0)
        L.pllm_synth_f32(norm.ptr, K, 3, 1.0, 0.1)
        L.pllm_synth_f32(out.ptr, rows, 4, 0.0, 1.0)
        for _ in range(3):
            L.pllm_gemv(out.ptr, 0, 0, 0, 0, 0, x.ptr, 0, norm.ptr if pro == 1 else 0, 1e-6, 0, w.ptr, ws.ptr, 0, K, 0,
                        rows, 1, pro, epi, 0, 0)
    elif which == "attention_prefill":  # the prefill's attention: 2,048 tokens at positions 0.., 32 / 8 heads of 128
        M, nh, nkv, hs = 2048, 32, 8, 128
        rows = (nh + 2 * nkv) * hs
        rng = np.random.default_rng(0)
        qkv = Buffer.of(rng.normal(0, 1, M * rows).astype(np.float32))
        kc = Buffer.of(rng.normal(0, 1, M * nkv * hs).astype(np.float16).view(np.uint16))
        vc = Buffer.of(rng.normal(0, 1, M * nkv * hs).astype(np.float16).view(np.uint16))
        out = Buffer(M * nh * hs * 4)
        bufs += [qkv, kc, vc, out]
        for _ in range(3):
            L.pllm_attention_prefill(out.ptr, nh * hs, qkv.ptr, rows, kc.ptr, vc.ptr, 0, M, nh, nkv, hs)
    elif which == "prefill":  # the whole prefill of configs[3]: 2,048 tokens through 36 layers, twice (the launch list)
        from pllm.forward import QWEN3_8B, Engine
        eng = Engine(QWEN3_8B, seed=0)
        ids = np.random.default_rng(1).integers(0, QWEN3_8B.vocab, 2048).astype(np.int32)
        for _ in range(2):
            eng.prefill(ids, 0, need_logits=False)
        L.pllm_sync()
        eng.close()
    elif which == "decode16":  # configs[3] at batch 16: two steps of the batch engine, eager (its launch list)
        from pllm.forward import QWEN3_8B, Engine
        eng = Engine(QWEN3_8B, seed=0, batch=16, graphs=False, pdl=False)
        for s in range(2):
            eng.forward_batch(np.arange(16) + 5 + s, np.full(16, 2048 + s), need_logits=False)
        eng.close()
    elif which == "cls":  # the classifier product: 151,936 rows, K 4096, RMSNorm prologue (171 MB: > L2)
        rows, K = 151936, 4096
        w, ws = Buffer(rows * K), Buffer(rows * K // 8)
        x, norm, out = Buffer(K * 4), Buffer(K * 4), Buffer(rows * 4)
        bufs += [w, ws, x, norm, out]
        L.pllm_synth_q8(w.ptr, ws.ptr, rows, K, 1, 0.02)
        L.pllm_synth_f32(x.ptr, K, 2, 0.0, 1.0)
        L.pllm_synth_f32(norm.ptr, K, 3, 1.0, 0.1)
        for _ in range(3):
            L.pllm_gemv(out.ptr, 0, 0, 0, 0, 0, x.ptr, 0, norm.ptr, 1e-6, 0, w.ptr, ws.ptr, 0, K, 0, rows, 1, 1, 0, 0, 0)
    elif which in ("q6r", "b1r"):  # the registry's int6 (bulk-copy) and binary (register) products, 16,384 x 4096
        rows, K = 16384, 4096
        rng = np.random.default_rng(7)
        wbytes = rows * K * 6 // 8 if which == "q6r" else rows * K // 8
        w = Buffer.of(rng.integers(0, 256, wbytes, dtype=np.uint8))
        out = Buffer(rows * 4)
        xq = Buffer.of(rng.integers(0, 128, K, dtype=np.uint8))
        bufs += [w, out, xq]
        if which == "q6r":
            ws = Buffer.of(rng.normal(0.02, 0.002, rows * K // 32).astype(np.float32))
            wc = Buffer.of(rng.integers(-2000, 2000, rows * K // 32).astype(np.int32))
            xs = Buffer.of(rng.normal(0.02, 0.002, K // 32).astype(np.float32))
            bufs += [ws, wc, xs]
            for _ in range(3):
                L.matmul_q6r(out.ptr, xq.ptr, xs.ptr, w.ptr, ws.ptr, wc.ptr, K, 0, rows)
        else:
            halves = Buffer.of(rng.normal(0.02, 0.002, rows * K // 128).astype(np.float16).view(np.uint16))
            ext = Buffer.of(np.concatenate([rng.normal(0.02, 0.002, K // 32).astype(np.float32).view(np.int32),
                                            rng.integers(-2000, 2000, K // 32).astype(np.int32)]))
            bufs += [halves, ext]
            for _ in range(3):
                L.matmul_b1r(out.ptr, xq.ptr, ext.ptr, w.ptr, halves.ptr, K, 0, rows, 2)
    elif which in ("delta1", "delta64"):  # the delta rule's micro-configuration: kh 16, vh 32, kd = vd = 128
        kh, vh, kd, vd = 16, 32, 128, 128
        count = 1 if which == "delta1" else 64
        sbytes = vh * kd * vd * 4
        states = Buffer(2 * 3 * sbytes)  # three state pairs (12 MB), one a launch
        cw, ww = 2 * kh * kd + vh * vd, 2 * vh + vh * vd
        c, work, out = Buffer(64 * cw * 4), Buffer(64 * ww * 4), Buffer(64 * vh * vd * 4)
        bufs += [states, c, work, out]
        L.pllm_synth_f32(states.ptr, 2 * 3 * sbytes // 4, 31, 0.0, 0.5)
        L.pllm_synth_f32(c.ptr, 64 * cw, 32, 0.0, 0.3)
        L.pllm_synth_f32(work.ptr, 64 * ww, 33, 0.5, 0.1)
        for i in range(3):
            s0 = states.ptr + 2 * i * sbytes
            if count == 1:
                L.delta_rule(out.ptr, s0, s0 + sbytes, c.ptr, work.ptr, kh, kd, vd, vh, 0, vh)
            else:
                L.pllm_delta_rule_block(out.ptr, vh * vd, s0, s0 + sbytes, c.ptr, cw, work.ptr, ww, count, kh, kd, vd,
                                        vh, 0, vh)
    elif which == "sample":  # the greedy step's argmax and a draw (temperature 0.8, top-p 0.9) over 151,936 logits
        n = 151936
        logits = Buffer(n * 4)
        L.pllm_synth_f32(logits.ptr, n, 5, 0.0, 3.0)
        nxt, amx, probs, index, rnd = Buffer(4), Buffer(16).zero(), Buffer(4 * n), Buffer(4 * n), Buffer.of(
            np.array([0.37], np.float64))
        bufs += [logits, nxt, amx, probs, index, rnd]
        for _ in range(3):
            L.pllm_argmax_dev(nxt.ptr, logits.ptr, n, amx.ptr)
        for _ in range(3):
            L.pllm_sample_dev(nxt.ptr, logits.ptr, n, 0.8, 0.9, rnd.ptr, probs.ptr, index.ptr, 0, 0.0)
    elif which in ("sbq4k", "sbiq2xs"):  # super-block products (matmul_sbr) over 16,384 x 4096: Q4_K, IQ2_XS
        t, size, halves = {"sbq4k": (12, 144, (0, 2)), "sbiq2xs": (17, 74, (0,))}[which]
        rows, n = 16384, 4096
        rng = np.random.default_rng(t)
        raw = rng.integers(0, 256, (rows * n // 256, size), dtype=np.uint8)  # any bytes are blocks
        for at in halves:  # finite float16 scales of a model's size
            raw[:, at:at + 2] = rng.uniform(0.002, 0.05, raw.shape[0]).astype("<f2").view(np.uint8).reshape(-1, 2)
        books = np.load(os.path.join(ROOT, "tests", "golden", "superblocks.npz"))["codebooks"]
        W, tab, bk = Buffer.of(raw.reshape(-1)), Buffer(34992), Buffer.of(books)
        X = Buffer.of(np.concatenate([rng.integers(0, 128, n, dtype=np.uint8),
                                      rng.normal(0, 0.02, n // 8).astype(np.float32).view(np.uint8)]))
        out = Buffer(rows * 4)
        bufs += [W, tab, bk, X, out]
        L.sb_tables(tab.ptr, bk.ptr)
        for _ in range(3):
            L.matmul_sbr(out.ptr, X.ptr, X.ptr + n, W.ptr, tab.ptr, n, 0, rows, t)
    elif which == "gemv16":  # the batch-16 step's w1/w3 product (the batched tensor-core form), 16 tokens
        hidden, K, M = 12288, 4096, 16
        w, ws = Buffer(2 * hidden * K), Buffer(2 * hidden * K // 8)
        x, norm, out = Buffer(M * K * 4), Buffer(K * 4), Buffer(M * hidden * 4)
        bufs += [w, ws, x, norm, out]
        L.pllm_synth_q8(w.ptr, ws.ptr, 2 * hidden, K, 1, 0.02)
        L.pllm_synth_f32(x.ptr, M * K, 2, 0.0, 1.0)
        L.pllm_synth_f32(norm.ptr, K, 3, 1.0, 0.1)
        for _ in range(3):
            L.pllm_gemv(out.ptr, hidden, 0, 0, 0, 0, x.ptr, K, norm.ptr, 1e-6, 0, w.ptr, ws.ptr, 0, K, 0, hidden, M, 1, 2,
                        hidden, 0)
    elif which == "t2":  # configs[4]'s w1/w3 product (ternary, 2 x 21504 rows, K 5120), three copies: none in L2
        hidden, K = 21504, 5120
        ws_ = [(Buffer(2 * hidden * K // 4), Buffer(2 * hidden * K // 64)) for _ in range(3)]
        x, norm, out = Buffer(K * 4), Buffer(K * 4), Buffer(hidden * 4)
        bufs += [b for pair in ws_ for b in pair] + [x, norm, out]
        for i, (w, ws) in enumerate(ws_):
            L.pllm_synth_t2(w.ptr, ws.ptr, 2 * hidden, K, 1 + i, 0.02, 0.002)
        L.pllm_synth_f32(x.ptr, K, 2, 0.0, 1.0)
        L.pllm_synth_f32(norm.ptr, K, 3, 1.0, 0.1)
        for i in range(3):
            w, ws = ws_[i]
            L.pllm_gemv(out.ptr, 0, 0, 0, 0, 0, x.ptr, 0, norm.ptr, 1e-6, 0, w.ptr, ws.ptr, 2, K, 0, hidden, 1, 1, 2,
                        hidden, 0)
    elif which == "gemm":
        M, N, K = 512, 4096, 4096
        xq, xs, w, ws, wt, out = (Buffer(n) for n in (M * K, M * K // 8, N * K, N * K // 8, N * K // 8, M * N * 4))
        bufs += [xq, xs, w, ws, wt, out]
        L.pllm_synth_q8(w.ptr, ws.ptr, N, K, 1, 0.02)
        L.pllm_synth_q8(xq.ptr, xs.ptr, M, K, 2, 1.0)
        L.pllm_transpose_scales(wt.ptr, ws.ptr, N, K // 32)
        for _ in range(3):
            L.pllm_gemm_q8(out.ptr, N, xq.ptr, xs.ptr, w.ptr, wt.ptr, M, N, K, N, 0, 0)
    else:
        nh, nkv, hs, cap, split = 32, 8, 128, 2560, 128
        rng = np.random.default_rng(0)
        kc = Buffer.of(rng.normal(0, 1, cap * nkv * hs).astype(np.float16).view(np.uint16))
        vc = Buffer.of(rng.normal(0, 1, cap * nkv * hs).astype(np.float16).view(np.uint16))
        qkv = Buffer.of(rng.normal(0, 1, (nh + 2 * nkv) * hs).astype(np.float32))
        ones = Buffer.of(np.ones(hs, np.float32))
        ang = np.outer(np.arange(cap), 1.0 / 1e6 ** (np.arange(0, hs, 2) / hs))
        cos, sin = Buffer.of(np.cos(ang).astype(np.float32)), Buffer.of(np.sin(ang).astype(np.float32))
        out, bad = Buffer(nh * hs * 4), Buffer(4).zero()
        sc = Buffer(L.pllm_attention_scratch_bytes(nh, hs, cap, split)).zero()
        pos = Buffer.of(np.array([2559], np.int32))
        bufs += [kc, vc, qkv, ones, cos, sin, out, bad, sc, pos]
        for _ in range(3):
            L.pllm_attention_step(out.ptr, qkv.ptr, kc.ptr, vc.ptr, sc.ptr, pos.ptr, cap, nh, nkv, hs, 1, 0.0, split,
                                  ones.ptr, ones.ptr, cos.ptr, sin.ptr, 0, 1e-6, bad.ptr, 0)
    L.pllm_sync()
    check(which)
    status = L.pllm_device_status()
    for b in bufs:
        b.free()
    print(json.dumps({"kernel_case": which, "status": status}))
    return 0 if status == 0 else 1


def gemm_tops(eng, cfg, M, timed):
    """The prefill's dominant product alone: layer 0's w1/w3 (M x 2 hidden x dim, gated epilogue) on the prefill's own
    buffers, 5 launches; int8 tera-ops a second against twice the measured bf16 dense rate (B200's int8 rate is twice
    its bf16 rate; no int8 figure is measured)."""
    from pllm.lib import L
    c, sh, B, P = cfg, eng.shard, eng.B, eng.P
    run = lambda: L.pllm_gemm_q8(P["HB"].ptr, sh.hidden, P["XQ"].ptr, P["XS"].ptr, B["w13"].ptr,  # noqa: E731
                                 P["ts13"].ptr, M, sh.hidden, c.dim, 2 * sh.hidden, 2, sh.hidden)
    run()
    ms = timed(lambda: [run() for _ in range(5)]) / 5
    tops = 2.0 * M * 2 * sh.hidden * c.dim / (ms / 1000) / 1e12
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, kind = 2 * float(json.load(f)["bf16_tflops"]), "2 x measured bf16 dense"
    except Exception:
        peak, kind = 2 * 1590.0, "2 x fallback bf16 dense"
    return {"kernel": "gemm_q8_kernel<gated FFN> (w1/w3, layer 0)", "M": M, "N": 2 * sh.hidden, "K": c.dim,
            "us": round(ms * 1000, 1), "tops": round(tops, 1), "bound": "tensor", "peak_tops": peak,
            "peak_kind": kind, "frac": round(tops / peak, 4)}


SWEEP_SHAPES = [(1024, 1024), (1024, 4608), (4096, 4096), (4096, 12288), (12288, 4096)]  # (K, N): configs[1]


def product_sweep(timed, Ms=(1, 4, 16, 128, 512, 2048)):
    """the isolated products at (K, N) x M, every launch of a measurement on another window of
    a 512 MB weight arena (so that no launch finds its weights in the 126 MB L2). M <= 16: the decode products
    (pllm_gemv: int8 on the bulk-copy pipeline -- 1..2 tokens dp4a, 3..16 the tensor-core form; int6 and ternary at one
    token on their bulk-copy forms (int6 from 2^25 weights up), past one token on the register kernel), their
    algorithmic bytes (weights N K (1 + 1/8) int8, (3/4 + 1/8) int6, (1/4 + 2/128) ternary, plus the activations and
    outputs) over the CUDA-event time, against the measured HBM copy rate. M >= 128:
    the int8 tensor-core product (pllm_gemm_q8, tcgen05 kind::i8), 2 M N K operations against twice the measured bf16
    dense rate (int6 and ternary checkpoints are widened to int8 for it, so their prefill is this product)."""
    from pllm.device import Buffer
    from pllm.lib import L, check
    hbm, _ = peaks()
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tpeak = 2 * float(json.load(f)["bf16_tflops"])
    except Exception:
        tpeak = 2 * 1590.0
    ARENA = 512 << 20
    wq, ws = Buffer(ARENA), Buffer(ARENA // 8)
    L.pllm_synth_q8(wq.ptr, ws.ptr, ARENA // 4096, 4096, 7, 0.02)
    t2, t2s = Buffer(ARENA // 4), Buffer(ARENA // 64)  # ternary: codes of ARENA weights and their float16 scales
    L.pllm_synth_t2(t2.ptr, t2s.ptr, ARENA // 4096, 4096, 8, 0.02, 0.002)
    kmax, mmax = 12288, 2048
    xq, xs = Buffer(mmax * kmax), Buffer(mmax * kmax // 8 * 2)
    L.pllm_synth_q8(xq.ptr, xs.ptr, mmax, kmax, 9, 1.0)
    out = Buffer(mmax * 12288 * 4)
    wt = Buffer(12288 * 4096 // 8 * 4)
    ev = {}
    fmts = {"q8": (0, 1.0, 32), "q6": (1, 0.75, 32), "t2": (2, 0.25, 128)}
    for name, (fmt, vb, gk) in fmts.items():
        ev[name] = {}
        for K, N in SWEEP_SHAPES:
            row = {}
            wbytes = int(N * K * vb)
            sbytes = N * (K // gk) * (2 if fmt == 2 else 4)
            arena, sarena = (t2, t2s) if fmt == 2 else (wq, ws)
            windows = max(4, min(40, (256 << 20) // max(wbytes, 1)))
            span = arena.nbytes - wbytes
            for M in Ms:
                if M > 16 and fmt != 0:
                    continue
                offs = [((i * 7919 * 4096) % max(span, 1)) & ~4095 for i in range(windows)]
                if M <= 16:
                    def run():
                        for i, o in enumerate(offs):
                            so = (i * sbytes) % max(sarena.nbytes - sbytes, 1) & ~255
                            L.pllm_gemv(out.ptr, N, xq.ptr, xs.ptr, K, K // 8 * (2 if fmt == 2 else 1), 0, 0, 0, 0.0,
                                        0, arena.ptr + o, sarena.ptr + so, fmt, K, 0, N, M, 0, 0, 0, 0)
                    launches = windows
                else:
                    L.pllm_transpose_scales(wt.ptr, ws.ptr, N, K // 32)

                    def run():
                        for o in offs[:4]:
                            L.pllm_gemm_q8(out.ptr, N, xq.ptr, xs.ptr, wq.ptr + o, wt.ptr, M, N, K, N, 0, 0)
                    launches = 4
                run()
                ms = timed(lambda: [run() for _ in range(3)]) / (3 * launches)
                check(f"sweep {name} {K}x{N} M {M}")
                if M <= 16:
                    byts = wbytes + sbytes + M * K * (1 + 4 / 32) + 4 * M * N
                    gbs = byts / (ms / 1000) / 1e9
                    row[str(M)] = {"us": round(ms * 1000, 2), "gbs": round(gbs, 1), "frac": round(gbs / hbm, 3)}
                else:
                    tops = 2.0 * M * N * K / (ms / 1000) / 1e12
                    row[str(M)] = {"us": round(ms * 1000, 2), "tops": round(tops, 1), "frac": round(tops / tpeak, 4)}
            ev[name][f"K{K}_N{N}"] = row
    for b in (wq, ws, t2, t2s, xq, xs, out, wt):
        b.free()
    return {"shapes": "K x N (configs[1]); M tokens", "l2": "every launch on another window of a 512 MB arena",
            "gbs_peak": hbm, "tops_peak": tpeak, "products": ev}


def batch_decode(cfg, nb, prompt, warmup, steps, timed, hbm):
    """configs[3] at batch nb: nb sequences, each its own 2048-token prompt (the tensor-core prefill, a sequence at a
    time) and cache, then decode steps of all of them at once (one CUDA graph a step: the products over the nb tokens on
    the batched tensor-core form, the attention of all sequences in one launch). tok/s of the whole batch; the step's
    algorithmic bytes are the weights (8.51 GB) plus every sequence's cache read (2 x layers x (pos + 1) x kvdim x 2
    bytes). e2e: Engine.next_tokens (8 bytes a sequence in, 4 back)."""
    from pllm.device import Buffer
    from pllm.forward import Engine
    from pllm.lib import L
    eng = Engine(cfg, seed=0, batch=nb)
    L.pllm_set_stream(eng.stream)
    rng = np.random.default_rng(3)
    ids = rng.integers(0, cfg.vocab, (nb, prompt + warmup + 2 * steps)).astype(np.int32)
    for i in range(nb):
        eng.prefill(ids[i, :prompt], 0, need_logits=False, seq=i)
    eng.capture()
    total = warmup + 2 * steps
    tp = np.zeros((total, 2 * nb), np.int32)
    for s in range(total):
        tp[s, :nb] = ids[:, prompt + s]
        tp[s, nb:] = prompt + s
    staged = Buffer.of(tp)

    def device_steps(first, count):
        for s in range(first, first + count):
            L.pllm_d2d(eng.B["tp"].ptr, staged.ptr + 8 * nb * s, 8 * nb)
            L.pllm_graph_launch(eng.graph)

    device_steps(0, warmup)
    ms = timed(lambda: device_steps(warmup, steps))
    kv = 2 * cfg.layers * cfg.kvdim * 2 * nb * sum(prompt + warmup + s + 1 for s in range(steps)) / steps
    byts = cfg.weight_bytes() + kv
    e2e_ms = timed(lambda: [eng.next_tokens(ids[:, prompt + warmup + steps + s], tp[warmup + steps + s, nb:])
                            for s in range(steps)])
    eng.close()
    staged.free()
    tps = nb * steps / (ms / 1000)
    return {"batch": nb, "value": tps, "unit": "tok/s", "ms_per_step": ms / steps, "steps": steps,
            "positions": f"{prompt}..{prompt + warmup + steps}", "bytes_per_step": byts,
            "hbm_frac": byts / (ms / steps / 1000) / 1e9 / hbm,
            "e2e": {"value": nb * steps / (e2e_ms / 1000), "unit": "tok/s", "h2d_bytes_per_step": 8 * nb,
                    "d2h_bytes_per_step": 4 * nb, "call": "Engine.next_tokens (greedy: argmax on the device)"},
            "method": "Engine(batch=16): batched tensor-core products (mma m16n8k32 int8 groups in the bulk-copy "
                      "pipeline), the batch's attention in one launch"}


def ternary_decode(prompt, warmup, steps, timed, hbm):
    """the 27B-class ternary decoder (5120 hidden, 62 layers, 32 / 16 heads of 128, 21504
    FFN, 262144 vocab; every matrix packed ternary, 0.2656 bytes a weight: 6.83 GB a token), seeded synthetic codes
    and float16 row scales; its prompt through the decode step (the tensor-core prefill takes int8 matrices), then
    batch-1 decode steps (one CUDA graph a step). tok/s; the step's algorithmic bytes are the matrices' plus the cache
    read."""
    from pllm.device import Buffer
    from pllm.forward import TERNARY_27B, Engine
    from pllm.lib import L
    cfg = TERNARY_27B
    eng = Engine(cfg, seed=0)
    L.pllm_set_stream(eng.stream)
    eng.capture()
    ids = np.random.default_rng(5).integers(0, cfg.vocab, prompt + warmup + steps).astype(np.int32)
    staged = Buffer.of(np.stack([ids, np.arange(ids.size, dtype=np.int32)], axis=1).reshape(-1))

    def device_steps(first, count):
        for i in range(first, first + count):
            L.pllm_d2d(eng.B["tp"].ptr, staged.ptr + 8 * i, 8)
            L.pllm_graph_launch(eng.graph)

    prompt_ms = timed(lambda: device_steps(0, prompt))
    device_steps(prompt, warmup)
    ms = timed(lambda: device_steps(prompt + warmup, steps))
    kv = 2 * cfg.layers * cfg.kvdim * 2 * sum(prompt + warmup + s + 1 for s in range(steps)) / steps
    byts = cfg.weight_bytes() + kv
    eng.close()
    staged.free()
    return {"config": "configs[4]: 27B-class ternary (5120 hidden, 62 layers, 32/16 heads x 128, 21504 FFN, "
                      "262144 vocab), packed ternary matrices", "value": steps / (ms / 1000), "unit": "tok/s",
            "ms_per_step": ms / steps, "positions": f"{prompt}..{prompt + warmup + steps}",
            "weight_bytes": cfg.weight_bytes(), "bytes_per_step": byts, "hbm_frac": byts / (ms / steps / 1000) / 1e9 / hbm,
            "prompt": {"tokens": prompt, "tok_s": prompt / (prompt_ms / 1000), "method": "the decode step a token"},
            "method": "gemv_tma_t2_kernel: bulk-copy stages of 2-bit codes and float16 scales, unpacked in registers"}


def lfm2_decode(nb, prompt, warmup, steps, timed, hbm):
    """the LFM2-350M-shaped hybrid (1024 hidden, 16 layers: 10 short-convolution layers of 3
    taps among 6 grouped-query attention layers of 16 / 8 heads of 64, 4608 FFN, 65536 vocab), seeded synthetic int8
    weights, at batch nb: every sequence's 512-token prompt through the decode step (all the batch's at once), then
    decode steps (one CUDA graph a step). tok/s of the batch; the step's bytes are the matrices' (0.40 GB) plus the
    caches read."""
    from pllm.device import Buffer
    from pllm.forward import LFM2_350M, Engine
    from pllm.lib import L
    cfg = LFM2_350M
    eng = Engine(cfg, seed=0, batch=nb)
    L.pllm_set_stream(eng.stream)
    eng.capture()
    total = prompt + warmup + steps
    ids = np.random.default_rng(11).integers(0, cfg.vocab, (total, nb)).astype(np.int32)
    tp = np.concatenate([ids, np.repeat(np.arange(total, dtype=np.int32)[:, None], nb, axis=1)], axis=1)
    staged = Buffer.of(tp)

    def device_steps(first, count):
        for s in range(first, first + count):
            L.pllm_d2d(eng.B["tp"].ptr, staged.ptr + 8 * nb * s, 8 * nb)
            L.pllm_graph_launch(eng.graph)

    prompt_ms = timed(lambda: device_steps(0, prompt))
    device_steps(prompt, warmup)
    ms = timed(lambda: device_steps(prompt + warmup, steps))
    attn = sum(1 for k in cfg.kinds if k == "a")
    kv = 2 * attn * cfg.kvdim * 2 * nb * sum(prompt + warmup + s + 1 for s in range(steps)) / steps
    byts = cfg.weight_bytes() + kv
    eng.close()
    staged.free()
    return {"batch": nb, "value": nb * steps / (ms / 1000), "unit": "tok/s", "ms_per_step": ms / steps,
            "positions": f"{prompt}..{prompt + warmup + steps}", "bytes_per_step": byts,
            "hbm_frac": byts / (ms / steps / 1000) / 1e9 / hbm,
            "prompt": {"tokens": prompt, "tok_s": nb * prompt / (prompt_ms / 1000), "method": "the decode step"}}


def delta_rule_micro(timed, hbm):
    """The delta rule's micro-configuration (no BASELINE config has the layer): kh 16, vh 32, kd = vd = 128, one token
    (delta_rule: the state read and the next written, 2 x 2 MB) and a block of 64 tokens (pllm_delta_rule_block: the
    state read once and written once for all 64); its HBM bytes over the CUDA-event time. Each launch on another of 40
    state pairs (160 MB: none in L2)."""
    from pllm.device import Buffer
    from pllm.lib import L
    kh, vh, kd, vd, n = 16, 32, 128, 128, 40
    sbytes = vh * kd * vd * 4
    states = Buffer(2 * n * sbytes)
    L.pllm_synth_f32(states.ptr, 2 * n * sbytes // 4, 31, 0.0, 0.5)
    cw, ww = 2 * kh * kd + vh * vd, 2 * vh + vh * vd
    c, work, out = Buffer(64 * cw * 4), Buffer(64 * ww * 4), Buffer(64 * vh * vd * 4)
    L.pllm_synth_f32(c.ptr, 64 * cw, 32, 0.0, 0.3)
    L.pllm_synth_f32(work.ptr, 64 * ww, 33, 0.5, 0.1)
    res = {}
    for name, count in (("token", 1), ("block64", 64)):
        def run():
            for i in range(n):
                s0 = states.ptr + 2 * i * sbytes
                if count == 1:
                    L.delta_rule(out.ptr, s0, s0 + sbytes, c.ptr, work.ptr, kh, kd, vd, vh, 0, vh)
                else:
                    L.pllm_delta_rule_block(out.ptr, vh * vd, s0, s0 + sbytes, c.ptr, cw, work.ptr, ww, count, kh,
                                            kd, vd, vh, 0, vh)
        run()
        ms = timed(lambda: [run() for _ in range(3)]) / (3 * n)
        byts = 2 * sbytes + count * (cw + ww + vh * vd) * 4
        res[name] = {"tokens": count, "us": round(ms * 1000, 2), "gbs": round(byts / (ms / 1000) / 1e9, 1),
                     "frac": round(byts / (ms / 1000) / 1e9 / hbm, 3), "us_per_token": round(ms * 1000 / count, 3)}
    for b in (states, c, work, out):
        b.free()
    res["config"] = "kh 16, vh 32, kd = vd = 128 (the state 2 MB a layer)"
    return res


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic(name):
    """dram bytes a launch from the committed ncu summary of that kernel (profiles/<name>.md: 'traffic_bytes: N')."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    try:
        for line in open(path):
            if line.strip().startswith("traffic_bytes:"):
                return int(float(line.split(":")[1]))
    except Exception:
        pass
    return None


class Clocks:
    """nvidia-smi sampled every 200 ms during the timed region."""

    FIELDS = ("index,pci.bus_id,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, bus=None):
        self.bus_id = f":{bus:02x}:" if isinstance(bus, int) else ""
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if not self.proc:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait()
        self.file.flush()
        rows = [r.split(", ") for r in open(self.file.name).read().strip().splitlines() if r.count(",") >= 9]
        os.unlink(self.file.name)
        if self.bus_id:
            mine = [r for r in rows if self.bus_id in r[1].lower()]
            rows = mine or rows
        if not rows:
            return None
        sm = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[6 + i].strip() == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][3]) if rows[0][3].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------------------------------------------ the CPU oracle leg

def oracle_decode(cfg, W, kc, vc, pos0, budget_s, most):
    """The oracle's decode (all host threads) from pos0: tokens decoded and seconds taken (at least one token)."""
    import oracle as O
    oc = O.Config(dim=cfg.dim, hidden=cfg.hidden, layers=cfg.layers, heads=cfg.heads, kv_heads=cfg.kv_heads,
                  head_size=cfg.head_size, vocab=cfg.vocab, seq_len=cfg.seq_len, qk_norm=int(cfg.qk_norm),
                  relaxed=int(cfg.relaxed), half_kv=int(cfg.half_kv), eps=cfg.eps)
    A = dict(W)
    A.update(cq=None, ck=None, cv=None, co=None, c1=None, c2=None, c3=None, cls_c=None, kc=kc, vc=vc)
    rng = np.random.default_rng(7)
    done, t0 = 0, time.perf_counter()
    while done < most and (done == 0 or time.perf_counter() - t0 < budget_s):
        O.forward(oc, A, int(rng.integers(0, cfg.vocab)), pos0 + done)
        done += 1
    return done, time.perf_counter() - t0, O.threads()


def reference_weights(cfg):
    """Host weights for the reference arm, made without the GPU library: random int8 values and float32 scales of the
    converter's layout (the CPU kernels' speed does not depend on the values), the cache's first PROMPT positions
    random float16."""
    rng = np.random.default_rng(0)
    c = cfg

    def q8(rows, cols):
        return (np.frombuffer(rng.bytes(rows * cols), np.int8).reshape(rows, cols) // 8,
                np.full((rows, cols // 32), 0.02 * 3 / 127, np.float32))

    W = {}
    for name, rows, cols in (("q", c.qdim, c.dim), ("k", c.kvdim, c.dim), ("v", c.kvdim, c.dim), ("o", c.dim, c.qdim),
                             ("1", c.hidden, c.dim), ("2", c.dim, c.hidden), ("3", c.hidden, c.dim)):
        w, s = q8(c.layers * rows, cols)
        W["w" + name], W["s" + name] = w, s
    W["emb"], W["emb_s"] = q8(c.vocab, c.dim)
    W["cls"], W["cls_s"] = q8(c.vocab, c.dim)
    for k, shape in (("att_norm", (c.layers, c.dim)), ("ffn_norm", (c.layers, c.dim)), ("final_norm", (c.dim,)),
                     ("q_norm", (c.layers, c.head_size)), ("k_norm", (c.layers, c.head_size))):
        W[k] = np.ones(shape, np.float32)
    freqs = 1.0 / c.rope_theta ** (np.arange(0, c.head_size, 2, dtype=np.float64) / c.head_size)
    angles = np.outer(np.arange(c.seq_len, dtype=np.float64), freqs)
    W["cos_t"], W["sin_t"] = np.cos(angles).astype(np.float32), np.sin(angles).astype(np.float32)
    n = c.layers * c.seq_len * c.kvdim
    kc = np.zeros(n, np.uint16)
    vc = np.zeros(n, np.uint16)
    filled = (rng.normal(0, 1, c.kvdim * 4096).astype(np.float16)).view(np.uint16)
    for l in range(c.layers):
        at = l * c.seq_len * c.kvdim
        for p in range(0, PROMPT, 4096 // 1):
            m = min(4096, PROMPT - p) * c.kvdim
            kc[at + p * c.kvdim: at + p * c.kvdim + m] = filled[:m]
            vc[at + p * c.kvdim: at + p * c.kvdim + m] = filled[:m]
    return W, kc, vc


class ReferenceShape:
    """configs[3]'s shape for the reference arm (kept apart from the GPU package, which that arm does not load)"""
    dim, hidden, layers, heads, kv_heads, head_size, vocab, seq_len = 4096, 12288, 36, 32, 8, 128, 151936, 2560
    qk_norm, rope_theta, eps, relaxed, half_kv = True, 1e6, 1e-6, False, True
    qdim, kvdim = 32 * 128, 8 * 128


def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", 0))
    if rank != 0:
        return
    W, kc, vc = reference_weights(cfg)
    import oracle as O
    # warm-up steps, then the timed ones: each a decode token at PROMPT + i; the number of timed tokens is bounded so
    # the run ends within minutes (the count run is reported)
    warmup = max(3, args.warmup)
    oracle_decode(cfg, W, kc, vc, PROMPT, 0.0, warmup)
    n, secs, threads = oracle_decode(cfg, W, kc, vc, PROMPT + warmup, 60.0, args.steps)
    value = n / secs
    line = {"metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus, "steps": n, "warmup": warmup,
            "ms_per_step": 1000 * secs / n, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic", "impl": "reference",
            "config": {"workload": "qwen3-8b-int8 batch-1 decode at positions 2048+ (BASELINE.json configs[3])",
                       "model": "Qwen3-8B-shaped int8 (36 layers, 4096 hidden, 32/8 heads, 12288 FFN, 151936 vocab)",
                       "global_batch": 1, "seq_len": PROMPT, "layers": cfg.layers,
                       "parallelism": f"host threads (OpenMP, {threads}), rank 0 alone"},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": f"{n} decode tokens at positions {PROMPT + warmup}.. of the full 36-layer model "
                                       "(the reference's WASM kernels cannot run here: the C restatement of them)"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    del O


# ------------------------------------------------------------------------------------------------ our arm

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--prompt", type=int, default=PROMPT)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--eager", action="store_true", help="profiling only: launch each kernel (no CUDA graph, no PDL)")
    ap.add_argument("--no-micro", action="store_true", help="profiling only: skip the per-kernel timings")
    ap.add_argument("--no-sweep", action="store_true", help="skip configs[1]'s product sweep (N = 1 only)")
    ap.add_argument("--batch", type=int, default=16, help="configs[3]'s batched decode (N = 1 only; 0: skip)")
    ap.add_argument("--no-ternary", action="store_true", help="skip configs[4]'s ternary decode (N = 1 only)")
    ap.add_argument("--no-lfm2", action="store_true", help="skip configs[2]'s hybrid decode (N = 1 only)")
    ap.add_argument("--layers", type=int, default=0,
                    help="profiling only: the same shapes with fewer layers (a small case for ncu captures)")
    ap.add_argument("--kernel", choices=["gemm", "attention", "attention_prefill", "prefill", "decode16", "gemv", "qkv",
                                         "wo", "w2", "cls", "q6r", "b1r", "delta1", "delta64", "sample", "sbq4k",
                                         "sbiq2xs", "gemv16", "t2"],
                    help="profiling only: three launches of one kernel's small case (for ncu), then exit")
    args = ap.parse_args()

    if args.kernel:
        return kernel_case(args.kernel)
    if args.impl == "reference":
        return run_reference(args, ReferenceShape())
    from dataclasses import replace

    from pllm.forward import QWEN3_8B
    cfg = replace(QWEN3_8B, layers=args.layers) if args.layers else QWEN3_8B

    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    dist = None
    from pllm.device import Buffer, init
    from pllm.forward import Engine
    from pllm.lib import L, check
    from pllm.tp import Exchange
    init(local)
    xg = None
    if world > 1:  # host plumbing only (handles, barriers, the max of the ranks' times): the data path is NVLink
        import datetime

        import torch.distributed as dist
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
        xg = Exchange(cfg, rank, world)

    steps, warmup = args.steps, max(3, args.warmup)
    prompt = args.prompt
    assert prompt + warmup + steps <= cfg.seq_len, "positions past the cache"
    eng = Engine(cfg, seed=0, device=local, graphs=not args.eager, pdl=not args.eager, exchange=xg)
    sh = eng.shard
    L.pllm_set_stream(eng.stream)
    rng = np.random.default_rng(1)  # one stream: the same ids on every rank
    ids = rng.integers(0, cfg.vocab, prompt + warmup + steps).astype(np.int32)
    tp = np.stack([ids, np.arange(ids.size, dtype=np.int32)], axis=1).reshape(-1)
    staged = Buffer.of(tp)  # every step's (token, position) in device memory before the timed region
    ev = [L.pllm_event_create() for _ in range(2)]

    def device_steps(first, count):
        for i in range(first, first + count):
            L.pllm_d2d(eng.B["tp"].ptr, staged.ptr + 8 * i, 8)
            eng.launch_step()

    def timed(fn):
        L.pllm_sync()
        if dist:
            dist.barrier()
        L.pllm_event_record(ev[0])
        fn()
        L.pllm_event_record(ev[1])
        ms = L.pllm_event_ms(ev[0], ev[1])
        check("timed region")
        if dist:
            import torch
            t = torch.tensor([ms], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    if not args.eager:
        eng.capture()
    # the prompt: the tensor-core prefill (every layer's products for all its tokens at once), filling the cache; with
    # tensor parallelism (or shapes it does not take) a decode step a token
    gemm = None
    if eng.can_prefill():
        eng.prefill(ids[:prompt], 0)  # warm: the scales' transposed copies, the buffers, the tensor maps' encoder
        prefill_ms = timed(lambda: [eng.prefill(ids[:prompt], 0) for _ in range(3)]) / 3
        prefill_tps = prompt / (prefill_ms / 1000)
        prefill_method = "tensor-core prefill (pllm_gemm_q8 tcgen05 kind::i8 products, pllm_attention_prefill)"
        gemm = gemm_tops(eng, cfg, prompt, timed)
    else:
        device_steps(0, 8)
        prefill_ms = timed(lambda: device_steps(8, prompt - 8))
        prefill_tps = (prompt - 8) / (prefill_ms / 1000)
        prefill_method = "token by token through the decode graph"
    device_steps(prompt, warmup)

    try:
        import torch
        bus = torch.cuda.get_device_properties(local).pci_bus_id if hasattr(torch.cuda.get_device_properties(local), "pci_bus_id") else None
    except Exception:
        bus = None
    clocks = Clocks(bus)
    decode_ms = timed(lambda: device_steps(prompt + warmup, steps))
    clock = clocks.stop()
    value = steps / (decode_ms / 1000)

    # end to end through the public call: token and position in from pinned memory, the next token (N = 1) or the
    # rank's logits (N > 1) out, every step
    e2e_steps = min(steps, cfg.seq_len - prompt - warmup - steps) or 0
    e2e_first = prompt + warmup + steps
    if e2e_steps < 8:  # rewind into the decode range (the cache's later positions are rewritten, as a new request)
        e2e_first, e2e_steps = prompt + warmup, steps
    # the greedy step's public call: the token and position in, the next token out (N > 1: every rank's vocab slice
    # gives its largest as a key, the keys meet in an NCCL max on the devices, each rank gets the token back)
    e2e_ms = timed(lambda: [eng.next_token(int(ids[i % ids.size]), i) for i in range(e2e_first, e2e_first + e2e_steps)])
    d2h_step = 4 * world
    e2e = e2e_steps / (e2e_ms / 1000)

    gemv, gemv_us, attention, achieved, w13_bytes = {}, {}, {}, None, None
    peak, peak_kind = peaks()
    c, B = cfg, eng.B
    if not args.no_micro:
        # the kernels alone, each family's 36 launches (every layer's weights: no L2 reuse) recorded as one CUDA graph
        # and replayed, so that the host's launch costs are not in the times
        c = cfg
        B = eng.B
        reps = 5
        E = 2 if c.half_kv else 4

        def graph_ms(enqueue, launches):
            g = eng.graph_of(enqueue)
            L.pllm_graph_launch(g)
            ms = timed(lambda: [L.pllm_graph_launch(g) for _ in range(reps)]) / (reps * launches)
            L.pllm_graph_destroy(g)
            return ms

        def w13_all():  # this rank's rows (all of them on one GPU)
            for l in range(c.layers):
                eng._gemv(B["hb"].ptr, B["w13"].ptr + l * 2 * sh.hidden * c.dim,
                          B["s13"].ptr + l * 2 * sh.hidden * (c.dim // 32) * 4, sh.hidden, c.dim, B["x"].ptr,
                          B["ffn_norm"].ptr + l * c.dim * 4, 1, 2, pair=sh.hidden, pdl=False)

        w13_ms = graph_ms(w13_all, c.layers)
        w13_bytes = 2 * sh.hidden * c.dim * 1.125 + c.dim * 4 * 2 + sh.hidden * 4
        peak, peak_kind = peaks()
        achieved = w13_bytes / (w13_ms / 1000) / 1e9
        gemv = {"w13_swiglu": round(achieved, 1)}
        gemv_us = {"w13_swiglu": round(w13_ms * 1000, 2)}

        def each(name, wq, ws, rows, cols, xin, norm, pro, epi):
            def run():
                for l in range(c.layers):
                    eng._gemv(B["qkv"].ptr if epi == 0 else B["x"].ptr, wq + l * rows * cols, ws + l * rows * (cols // 32) * 4,
                              rows, cols, xin, norm, pro, epi, pdl=False)
            ms = graph_ms(run, c.layers)
            gemv[name] = round(rows * cols * 1.125 / (ms / 1000) / 1e9, 1)
            gemv_us[name] = round(ms * 1000, 2)

        each("wqkv", B["wqkv"].ptr, B["sqkv"].ptr, eng.rows_qkv, c.dim, B["x"].ptr, B["att_norm"].ptr, 1, 0)
        each("wo", B["wo"].ptr, B["so"].ptr, c.dim, sh.qdim, B["att"].ptr, 0, 2, 1)
        each("w2", B["w2"].ptr, B["s2"].ptr, c.dim, sh.hidden, B["hb"].ptr, 0, 2, 1)
        L.pllm_set_stream(eng.stream)

        def cls_run():
            eng._gemv(B["logits"].ptr, B["cls"].ptr, B["cls_s"].ptr, sh.vocab, c.dim, B["x"].ptr, B["final_norm"].ptr, 1,
                      0, pdl=False)
        cls_ms = graph_ms(cls_run, 1)
        gemv["cls"] = round(sh.vocab * c.dim * 1.125 / (cls_ms / 1000) / 1e9, 1)
        gemv_us["cls"] = round(cls_ms * 1000, 2)

        # the attention alone at the last decode position (36 layers' caches, 2 kernels a layer)
        def attention_all():
            for l in range(c.layers):
                L.pllm_attention_step(B["att"].ptr, B["qkv"].ptr, B["kc"].ptr + l * c.seq_len * sh.kvdim * E,
                                      B["vc"].ptr + l * c.seq_len * sh.kvdim * E, B["scratch"].ptr, B["tp"].ptr + 4,
                                      c.seq_len, sh.heads, sh.kv_heads, c.head_size, int(c.half_kv), 0.0, eng.SPLIT,
                                      B["q_norm"].ptr + l * c.head_size * 4, B["k_norm"].ptr + l * c.head_size * 4,
                                      B["cos_t"].ptr, B["sin_t"].ptr, 0, c.eps, B["bad"].ptr, 0)

        att_ms = graph_ms(attention_all, c.layers)
        last_pos = int(B["tp"].download(np.int32)[1])
        att_bytes = 2 * (last_pos + 1) * sh.kvdim * E
        attention = {"us_per_layer": round(att_ms * 1000, 2), "position": last_pos,
                     "gbs": round(att_bytes / (att_ms / 1000) / 1e9, 1)}

    sweep = None
    if world == 1 and not args.no_sweep and not args.no_micro:
        sweep = product_sweep(timed)
        sweep["delta_rule"] = delta_rule_micro(timed, peaks()[0])
        L.pllm_set_stream(eng.stream)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        W = eng.host_weights()
        E = np.uint16
        kc = B["kc"].download(E)
        vc = B["vc"].download(E)
        n, secs, threads = oracle_decode(cfg, W, kc, vc, prompt, 20.0, 8)
        cpu = {"value": n / secs, "unit": "tok/s", "cores": threads, "kind": "port",
               "sample": f"{n} decode tokens at positions {prompt}.. of the same 36-layer model and cache (the C "
                         "restatement of the reference kernels, OpenMP over rows and heads)"}

    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warmup,
        "ms_per_step": decode_ms / steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic",
        "config": {"workload": "qwen3-8b-int8 batch-1 decode at positions 2048+ (BASELINE.json configs[3])",
                   "model": "Qwen3-8B-shaped int8 (36 layers, 4096 hidden, 32/8 heads x 128, QK-norm, 12288 FFN, "
                            "151936 vocab), float16 KV cache", "global_batch": 1, "seq_len": prompt,
                   "parallelism": f"tp{world} (NVLink exchange in the products)" if world > 1 else "1 GPU",
                   "layers": cfg.layers,
                   "l2": "no flush: every step streams 8.51 GB of weights (> 126 MB L2)"},
        "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8 * world,  # every rank's copies
                "d2h_bytes_per_step": d2h_step,
                "call": "Engine.next_token (greedy: argmax on the device)" if world == 1 else
                        "Engine.next_token (greedy: the ranks' argmax keys' NCCL max on the devices)"},
        "prefill": {"value": prefill_tps, "unit": "tok/s", "tokens": prompt, "ms": prefill_ms, "method": prefill_method,
                    "gemm": gemm},
        "gemv_gbs": gemv,
        "gemv_us": gemv_us,
        "attention": attention,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak if achieved else None,
                     "peak_kind": peak_kind, "kernel": "gemv_tma_kernel<1, 1, 2> (w1/w3: int8, 1 token, RMSNorm, SwiGLU)",
                     "bytes_per_launch": w13_bytes,  # a rank's launch: its 1/N of the rows
                     "traffic": (profile_traffic("gemv_q8_w13_qwen3-8b") or 0) / world or None},
        "decode_roofline_frac": (c.weight_bytes() / (decode_ms / steps / 1000) / 1e9) / (peak * world),
        "gpu_launches": eng.launches_per_step * steps * world,
        "clocks": clock,
    }
    if sweep:
        line["sweep"] = sweep
    if world == 1 and args.batch > 1:
        eng.close()
        bsteps = min(64, (cfg.seq_len - prompt - warmup) // 2)
        line["decode_batch"] = batch_decode(cfg, args.batch, prompt, warmup, bsteps, timed, peak)
    if world == 1 and not args.no_ternary:
        if not (args.batch > 1):
            eng.close()
        line["decode_ternary_27b"] = ternary_decode(1024, warmup, 128, timed, peak)
    if world == 1 and not args.no_lfm2:
        if args.batch <= 1 and args.no_ternary:
            eng.close()
        line["decode_lfm2_350m"] = [lfm2_decode(nb, 512, warmup, 256, timed, peak) for nb in (1, 8)]
    if cpu:
        line["cpu_baseline"] = cpu
    if rank == 0:
        print(json.dumps(line), flush=True)
    if not (world == 1 and (args.batch > 1 or not args.no_ternary or not args.no_lfm2)):
        eng.close()
    if xg:
        xg.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
