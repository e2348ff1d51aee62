"""The registry's job table over the C ABI: src/runtime/jobs.ts's WORK (:207-333), PACKED (:396-444) and runner()
(:456-478), kept line for line in meaning so that a job built by the reference's engine runs here unchanged.

A job is [kind, out, a, b, a4, a5, a6, a7, a8, rows, count, os, as, bs] (jobs.ts:36-45); its kind is the number of
a line of WORK (KIND). runner(k)(job, r0, r1) runs the rows [r0, r1) of the job on the device: one kernel launch a
call where the reference loops over rows and chunks in a software thread. `k` is pllm.lib.L (the library), whose
kernels take device addresses; there is one module (the reference's plain and relaxed modules are one library here).
"""
from .lib import L

THREE, TWO = 3, 2  # jobs.ts:49-51: the codes' masks the ternary and binary kernels take
BATCH = 16         # jobs.ts:23: the most tokens that go through the layers together
CHUNK_BYTES = 16384

# kind: (from, one(k), tile(k) or None, rowBytes(n) or None). The argument mapping of each is jobs.ts's.
WORK = {
    "matmul_q8r": ("relaxed",
                   lambda k: lambda out, a, b, a4, a5, a6, a7, a8, rows, r0, r1, a9=0: k.matmul_q8r(out, a, b, a4, a5, a6, a7, r0, r1),
                   lambda k: lambda out, a, b, a4, a5, a6, a7, r0, r1, count, os, as_, a8=0: k.matmul_q8r_tile(out, a, b, a4, a5, a6, a7, r0, r1, count, os, as_),
                   lambda n: n),
    "matmul_q8": ("plain",
                  lambda k: lambda out, a, b, a4, a5, a6, a7, a8, rows, r0, r1, a9=0: k.matmul_q8(out, a, b, a4, a5, a7, r0, r1),
                  None, lambda n: n),
    "matmul_f32": ("plain",
                   lambda k: lambda out, a, b, a4, a5, a6, a7, a8, rows, r0, r1, a9=0: k.matmul_f32(out, a, a4, a7, r0, r1),
                   None, lambda n: 4 * n),
    "attention": ("plain",
                  lambda k: lambda out, a, b, a4, a5, a6, a7, a8, rows, r0, r1, a9=0: k.attention(out, a, b, a4, a5, a6, rows, a7, a8, r0, r1),
                  None, None),
    "attention_f16": ("plain",
                      lambda k: lambda out, a, b, a4, a5, a6, a7, a8, rows, r0, r1, a9=0: k.attention_f16(out, a, b, a4, a5, a6, rows, a7, a8, r0, r1),
                      None, None),
    "matmul_q6r": ("relaxed",
                   lambda k: lambda out, a, b, a4, a5, a6, a7, a8, rows, r0, r1, a9=0: k.matmul_q6r(out, a, b, a4, a5, a6, a7, r0, r1),
                   None, lambda n: n * 3 // 4),
    "matmul_q6": ("plain",
                  lambda k: lambda out, a, b, a4, a5, a6, a7, a8, rows, r0, r1, a9=0: k.matmul_q6(out, a, b, a4, a5, a7, r0, r1),
                  None, lambda n: n * 3 // 4),
    "delta_rule": ("plain",
                   lambda k: lambda out, a, b, a4, a5, a6, a7, a8, rows, r0, r1, a9=0: k.delta_rule(out, a, b, a4, a5, a6, a7, a8, rows, r0, r1),
                   None, None),
    "matmul_t2r": ("relaxed",
                   lambda k: lambda out, a, b, a4, a5, a6, a7, a8, rows, r0, r1, a9=0: k.matmul_t2r(out, a, b, a4, a5, a7, r0, r1, THREE),
                   lambda k: lambda out, a, b, a4, a5, a6, a7, r0, r1, count, os, as_, a8=0: k.matmul_t2r_tile(out, a, b, a4, a5, a7, r0, r1, count, os, as_, THREE),
                   lambda n: n // 4),
    "matmul_t2": ("plain",
                  lambda k: lambda out, a, b, a4, a5, a6, a7, a8, rows, r0, r1, a9=0: k.matmul_t2(out, a, b, a4, a5, a7, r0, r1, THREE),
                  None, lambda n: n // 4),
    "matmul_b1r": ("relaxed",
                   lambda k: lambda out, a, b, a4, a5, a6, a7, a8, rows, r0, r1, a9=0: k.matmul_b1r(out, a, b, a4, a5, a7, r0, r1, TWO),
                   lambda k: lambda out, a, b, a4, a5, a6, a7, r0, r1, count, os, as_, a8=0: k.matmul_b1r_tile(out, a, b, a4, a5, a7, r0, r1, count, os, as_, TWO),
                   lambda n: n // 8),
    "matmul_b1": ("plain",
                  lambda k: lambda out, a, b, a4, a5, a6, a7, a8, rows, r0, r1, a9=0: k.matmul_b1(out, a, b, a4, a5, a7, r0, r1, TWO),
                  None, lambda n: n // 8),
    "attention_capped": ("plain",
                         lambda k: lambda out, a, b, a4, a5, a6, a7, a8, rows, r0, r1, a9=0: k.attention_capped(out, a, b, a4, a5, a6, rows, a7, a8, r0, r1, a9),
                         None, None),
    "attention_f16_capped": ("plain",
                             lambda k: lambda out, a, b, a4, a5, a6, a7, a8, rows, r0, r1, a9=0: k.attention_f16_capped(out, a, b, a4, a5, a6, rows, a7, a8, r0, r1, a9),
                             None, None),
}
KIND = {name: i for i, name in enumerate(WORK)}


def _biased(k, relaxed):
    bias = 64 if relaxed else 0
    return lambda xq, xs, x, n: k.quantize_x(xq, xs, x, n, bias)


def _interleaved(k, relaxed):
    def ready(xq, xs, x, n):
        k.quantize_x(xq, xs, x, n, 0)
        k.interleave(xq, xs, n)
    return ready


# jobs.ts:396-444 (the packings of this path): rowBytes, the scale's bytes, the jobs' kinds, the corrections'
# kernel, how the activations are made ready, the bytes of xs a group of 32, the weights a scale is of
PACKED = {
    "int8": dict(rowBytes=lambda n: n, scale=4, jobs=dict(relaxed=KIND["matmul_q8r"], plain=KIND["matmul_q8"]),
                 sums="int8_sums", ready=_biased, xs=4, group=32),
    "int6": dict(rowBytes=lambda n: n // 32 * 24, scale=4, jobs=dict(relaxed=KIND["matmul_q6r"], plain=KIND["matmul_q6"]),
                 sums="six_sums", ready=_biased, xs=4, group=32),
    "ternary": dict(rowBytes=lambda n: n // 4, scale=2, jobs=dict(relaxed=KIND["matmul_t2r"], plain=KIND["matmul_t2"]),
                    sums=None, ready=_interleaved, xs=8, group=128),
    "binary": dict(rowBytes=lambda n: n // 8, scale=2, jobs=dict(relaxed=KIND["matmul_b1r"], plain=KIND["matmul_b1"]),
                   sums=None, ready=_interleaved, xs=8, group=128),
}


def weight_bytes(packing):
    """jobs.ts:451: the bytes a weight takes (int8 1.125, int6 0.875, ternary 0.265625)."""
    p = PACKED[packing]
    return (p["rowBytes"](p["group"]) + p["scale"]) / p["group"]


def runner(k=L):
    """jobs.ts:456-478: runRows(job, r0, r1). A job of one token calls its kind's kernel for the rows; count > 1 goes
    to the kind's tile when it has one, else to the kernel token by token (on the device the reference's chunking
    of rows for its caches is not needed: a launch takes all the rows)."""
    names = list(WORK)
    ones = [WORK[n][1](k) for n in names]
    tiles = [WORK[n][2](k) if WORK[n][2] else None for n in names]

    def run(job, r0, r1):
        kind, out, a, b, a4, a5, a6, a7, a8, rows, count, os, as_, bs = job
        one = ones[kind]
        if count == 1:
            return one(out, a, b, a4, a5, a6, a7, a8, rows, r0, r1, os)
        tile = tiles[kind]
        if tile:
            return tile(out, a, b, a4, a5, a6, a7, r0, r1, count, os, as_, a8)
        for t in range(count):
            one(out + t * os, a + t * as_, b + t * bs, a4, a5, a6, a7, a8, rows, r0, r1, 0)
    return run
