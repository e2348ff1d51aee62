"""Checkpoints the reference wrote (tests/golden/checkpoints.npz), read by pllm/checkpoint.py into the forward driver on
the GPU: the logits of a short sequence against the oracle's forward on the same weights (the model-level line of the
other forward tests: 2e-2 of the largest logit, relative distance 2e-2, the same greedy token) and against the
reference's own NumPy forward on the file (its line for the int8 kernels: the greedy token at 85 % of the positions
or more, relative distance 5e-2 on average)."""
import numpy as np
import pytest

import oracle as O
from pllm.checkpoint import load

from test_checkpoint import GOLDEN, NAMES, files, form_of  # noqa: F401  (files: the fixture)
from test_gpu_forward import oracle_arrays, oracle_config

pytestmark = pytest.mark.gpu


def test_engine_runs_the_reference_files(files):  # noqa: F811
    agree, total, rels = 0, 0, []
    for name in NAMES:
        eng, cfg = load(files[name], form_of(name))
        from pllm.checkpoint import Checkpoint
        ck = Checkpoint(files[name], form_of(name))
        A, oc = oracle_arrays(cfg, ck.host_weights(cfg)), oracle_config(cfg)
        for pos, t in enumerate(GOLDEN["tokens"]):
            got = eng.forward(int(t), pos)
            want = O.forward(oc, A, int(t), pos)
            rel = float(np.linalg.norm(got - want) / np.linalg.norm(want))
            peak = float(np.abs(got - want).max() / np.abs(want).max())
            assert rel <= 2e-2 and peak <= 2e-2 and np.argmax(got) == np.argmax(want), (name, pos, rel, peak)
            ref = GOLDEN[f"{name}/logits"][pos]
            rels.append(float(np.linalg.norm(got - ref) / np.linalg.norm(ref)))
            agree += int(np.argmax(got) == np.argmax(ref))
            total += 1
        eng.close()
    print(f"against the reference's NumPy forward: greedy token {agree}/{total}, relative distance mean "
          f"{np.mean(rels):.2e} max {max(rels):.2e}")
    assert agree >= 0.85 * total and np.mean(rels) <= 5e-2
