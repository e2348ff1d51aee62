"""Tensor-parallel decode on the GPU: the exchange's sends and summing prologue (pllm_gemv_tp), its bounded wait, and
ranks on several GPUs against the whole model on one.

With one rank the exchange path makes the plain engine's numbers to the bit: the plain product adds its rows to x
(x + v), the exchanged one sends v and the next product's prologue makes x + v. With several ranks the wo and w2
partials are summed in rank order, so the logits move within float32 rounding, carried (now and then) through a
quantize_x rounding flip: held to the model-level line of the other forward tests (2e-2 of the largest logit)."""
import json
import os
import subprocess
import sys
import time
from dataclasses import replace

import numpy as np
import pytest

from pllm.forward import Config, Engine, PRO_RMS_SUM, EPI_STORE
from pllm.lib import L
from pllm.tp import Exchange

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SMALL = Config(dim=256, hidden=512, layers=3, heads=8, kv_heads=2, head_size=64, vocab=1000, seq_len=64,
               qk_norm=True, rope_theta=1e6, eps=1e-6)


@pytest.mark.parametrize("graphs", [False, True])
@pytest.mark.parametrize("relaxed", [False, True])
def test_one_rank_exchange_is_the_engine(graphs, relaxed):
    cfg = replace(SMALL, relaxed=relaxed)
    plain = Engine(cfg, seed=4, graphs=graphs)
    xg = Exchange(cfg)
    eng = Engine(cfg, seed=4, graphs=graphs, exchange=xg)
    try:
        assert np.array_equal(eng.host_weights()["wo"], plain.host_weights()["wo"])  # block synthesis: same bytes
        for pos, tok in enumerate(np.random.default_rng(2).integers(0, cfg.vocab, 5)):
            want = plain.forward(int(tok), pos)
            got = eng.forward(int(tok), pos)
            assert np.array_equal(got, want), (pos, np.abs(got - want).max())
        assert L.pllm_device_status() == 0
    finally:
        eng.close()
        plain.close()
        xg.close()


def test_exchange_wait_gives_up():
    """A summing prologue whose partials never come (no rank sends): the wait gives up after about 2 s, records
    PLLM_ETIMEOUT, and the library goes on working."""
    cfg = replace(SMALL, layers=1)
    eng = Engine(cfg, seed=1)
    xg = Exchange(cfg)
    try:
        B = eng.B
        L.pllm_device_status()
        L.pllm_set_stream(0)
        L.pllm_tp_step(xg.h)
        t0 = time.time()
        L.pllm_gemv_tp(B["qkv"].ptr, B["x"].ptr, B["hb"].ptr, B["att_norm"].ptr, cfg.eps, 0, B["wqkv"].ptr,
                       B["sqkv"].ptr, cfg.dim, eng.rows_qkv, PRO_RMS_SUM, EPI_STORE, 0, 0, xg.h, 1)
        assert L.pllm_sync() == 0
        elapsed = time.time() - t0
        assert L.pllm_device_status() == 3
        assert 1.5 < elapsed < 30, elapsed
        logits = eng.forward(3, 0)  # the device is still usable
        assert np.isfinite(logits).all()
        assert L.pllm_device_status() == 0
    finally:
        eng.close()
        xg.close()


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ranks_against_one_gpu(world, tmp_path):
    if _gpus() < world:
        pytest.skip(f"{world} GPUs needed")
    out = tmp_path / "tp.json"
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", "--master-port=29533",
           os.path.join(ROOT, "tests", "tp_worker.py"), "--layers", "4", "--out", str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["statuses"] == [0] * world
    for row in res["rows"]:
        print(f"{world} ranks, position {row['pos']}: relative {row['rel']:.2e}, peak {row['peak']:.2e}, "
              f"argmax {row['argmax']}")
        assert row["rel"] <= 2e-2 and row["peak"] <= 2e-2, row
    for row in res["prefill_rows"]:  # the tensor-core prefill across the ranks, then decode steps after it
        print(f"{world} ranks, {row['pos']}: relative {row['rel']:.2e}, peak {row['peak']:.2e}, argmax {row['argmax']}")
        assert row["rel"] <= 2e-2 and row["peak"] <= 2e-2, row
    # every rank's greedy token (the keys' max across the ranks) is the gathered logits' argmax
    assert all(t == res["gathered_argmax"] for t in res["greedy"]), res
