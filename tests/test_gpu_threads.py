"""The registry's threading contract (src/runtime/forward/threads.ts:90-133: many host threads call one kernel at
once on disjoint row ranges [r0, r1), or head ranges [h0, h1)): four Python threads (ctypes lets go of the GIL in a
call) each on its own stream, each calling the kernel on its quarter of the rows, many times over; the outputs are
the one full-range call's to the bit. The current stream is a thread's own, and each bulk-copy product launch takes
its own ticket counter, so the threads do not meet."""
import threading

import numpy as np
import pytest

import oracle as O
from pllm.device import Buffer, init
from pllm.lib import L, check

pytestmark = pytest.mark.gpu

THREADS, ROUNDS = 4, 25


@pytest.fixture(scope="module", autouse=True)
def device():
    init(0)
    L.pllm_set_stream(0)
    yield
    L.pllm_device_sync()


def run_threads(work):
    """work(i) in THREADS threads at once, each on a stream of its own; every exception is raised here."""
    errors, start = [], threading.Barrier(THREADS)

    def body(i):
        try:
            s = L.pllm_stream_create()
            L.pllm_set_stream(s)
            start.wait()
            for _ in range(ROUNDS):
                work(i)
            L.pllm_sync()
            check(f"thread {i}")
            L.pllm_stream_destroy(s)
        except Exception as e:  # noqa: BLE001
            errors.append(e)

    ts = [threading.Thread(target=body, args=(i,)) for i in range(THREADS)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    if errors:
        raise errors[0]


@pytest.mark.parametrize("kernel", ["matmul_q8", "matmul_q8r", "matmul_t2r"])
def test_row_ranges_from_four_threads_are_one_call(kernel):
    rng = np.random.default_rng(3)
    rows, k = 4096, 4096
    x = rng.normal(0, 1, k).astype(np.float32)
    if kernel == "matmul_t2r":
        codes = rng.integers(0, 3, (rows, k)).astype(np.int8) - 1
        wq = np.zeros((rows, k // 4), np.uint8)  # ternary.ts's layout: weight j at byte j >> 2, bits 2 (j & 3)
        for j in range(4):
            wq |= ((codes[:, j::4] + 1).astype(np.uint8) << (2 * j))
        ws = np.full((rows, k // 128), 0x2148, np.uint16)  # float16 0.0102
        xq, xs = O.quantize_x(x, 64)
        xq, xs = O.interleave(xq, xs)
    else:
        wq = rng.integers(-127, 128, (rows, k)).astype(np.int8)
        ws = rng.uniform(0.001, 0.02, (rows, k // 32)).astype(np.float32)
        xq, xs = O.quantize_x(x, 64 if kernel == "matmul_q8r" else 0)
    XQ, XS, WQ, WS = (Buffer.of(np.ascontiguousarray(a)) for a in (xq, xs, wq, ws))
    whole, parts = Buffer(rows * 4).zero(), Buffer(rows * 4).zero()
    fn = getattr(L, kernel)

    def call(out, r0, r1):
        if kernel == "matmul_q8":
            fn(out.ptr, XQ.ptr, XS.ptr, WQ.ptr, WS.ptr, k, r0, r1)
        elif kernel == "matmul_q8r":
            fn(out.ptr, XQ.ptr, XS.ptr, WQ.ptr, WS.ptr, 0, k, r0, r1)
        else:
            fn(out.ptr, XQ.ptr, XS.ptr, WQ.ptr, WS.ptr, k, r0, r1, 3)

    call(whole, 0, rows)
    L.pllm_sync()
    check(kernel)
    want = whole.download(np.float32)
    share = rows // THREADS
    run_threads(lambda i: call(parts, i * share, (i + 1) * share))
    got = parts.download(np.float32)
    assert np.array_equal(got.view(np.int32), want.view(np.int32))


def test_head_ranges_from_four_threads_are_one_call():
    nh, nkv, hs, pos = 32, 8, 128, 900
    rng = np.random.default_rng(5)
    q = rng.normal(0, 1, nh * hs).astype(np.float32)
    kc, _ = O.to_f16(rng.normal(0, 1, (pos + 1) * nkv * hs).astype(np.float32))
    vc, _ = O.to_f16(rng.normal(0, 1, (pos + 1) * nkv * hs).astype(np.float32))
    Q, K, V = Buffer.of(q), Buffer.of(kc), Buffer.of(vc)
    whole, parts = Buffer(nh * hs * 4).zero(), Buffer(nh * hs * 4).zero()
    atts = [Buffer(nh * (pos + 1) * 4) for _ in range(THREADS + 1)]
    L.attention_f16(whole.ptr, Q.ptr, K.ptr, V.ptr, atts[THREADS].ptr, pos, nh, nkv, hs, 0, nh)
    L.pllm_sync()
    check("attention_f16")
    share = nh // THREADS
    run_threads(lambda i: L.attention_f16(parts.ptr, Q.ptr, K.ptr, V.ptr, atts[i].ptr, pos, nh, nkv, hs, i * share,
                                          (i + 1) * share))
    assert np.array_equal(parts.download(np.float32), whole.download(np.float32))


def test_waiting_calls_from_four_threads():
    """argmax and to_f16 wait for a result in the library's own scratch: concurrent callers take turns, each gets
    its own answer."""
    rng = np.random.default_rng(8)
    xs = [rng.normal(0, 1, 100_000).astype(np.float32) for _ in range(THREADS)]
    for i, x in enumerate(xs):
        x[1000 * (i + 1)] = 50.0 + i
        x[7] = np.inf if i == 2 else x[7]
    bufs = [Buffer.of(x) for x in xs]
    halves = [Buffer(x.size * 2) for x in xs]
    got_max, got_bad = [None] * THREADS, [None] * THREADS

    def work(i):
        got_max[i] = L.argmax(bufs[i].ptr, xs[i].size)
        got_bad[i] = L.to_f16(halves[i].ptr, bufs[i].ptr, xs[i].size)
        assert got_max[i] == O.argmax(xs[i]), (i, got_max[i])
        assert got_bad[i] == O.to_f16(xs[i])[1], (i, got_bad[i])

    run_threads(work)
