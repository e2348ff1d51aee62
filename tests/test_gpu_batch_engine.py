"""The batch engine (Engine(batch=B): B sequences a step, each with its own cache and position; the products over all
of them at once on the batched tensor-core form, the attention in one launch) against the oracle's forward of each
sequence alone (its own cache), at the line the single-sequence engine meets (tests/test_gpu_forward.py: 2e-2 of the
largest logit and relative distance, the same greedy token at all but one step in twenty); and the greedy step
(next_tokens) against the argmax of the logits."""
from dataclasses import replace

import numpy as np
import pytest

import oracle as O
from pllm.forward import QWEN3_8B, Engine, synthetic_host_weights

from test_gpu_forward import SMALL_QWEN3, check_logits, oracle_arrays, oracle_config

pytestmark = pytest.mark.gpu


def run_against_oracle(cfg, eng, W, steps, offsets, seed, flips=None):
    nb = eng.batch
    A = [oracle_arrays(cfg, W) for _ in range(nb)]  # each sequence its own cache
    oc = oracle_config(cfg)
    rng = np.random.default_rng(seed)
    agree = 0
    for step in range(steps):
        toks = rng.integers(0, cfg.vocab, nb)
        poss = np.array([step + o for o in offsets])
        got = eng.forward_batch(toks, poss)
        for i in range(nb):
            want = O.forward(oc, A[i], int(toks[i]), int(poss[i]))
            check_logits(got[i], want, (step, i), (0.0, 0.0))
            agree += int(np.argmax(got[i]) == np.argmax(want))
    allowed = max(1, steps * nb // 20) if flips is None else flips
    assert agree >= steps * nb - allowed, agree


@pytest.mark.parametrize("nb", [4, 16])
def test_batch_engine_matches_oracle(nb):
    cfg = SMALL_QWEN3
    W = synthetic_host_weights(cfg, seed=11)
    eng = Engine(cfg, host=W, batch=nb)
    # sequences at different positions (sequence i starts at position 3 i; its earlier rows are zero, as the
    # oracle's cache is)
    run_against_oracle(cfg, eng, W, 12, [3 * i for i in range(nb)], seed=nb)
    eng.close()


def test_batch_engine_qwen3_8b_widths():
    """BASELINE.json configs[3]'s widths (two layers) at batch 16: every product on the batched form, w2 (K 12288)
    with its activations read from global memory. The logits at the line; the greedy token may differ where the
    random 151,936-wide vocabulary's two largest logits lie within the line of each other (as measured: 2 of 32)."""
    cfg = replace(QWEN3_8B, layers=2, seq_len=32)
    eng = Engine(cfg, seed=2, batch=16)
    W = eng.host_weights()
    run_against_oracle(cfg, eng, W, 2, [i for i in range(16)], seed=5, flips=4)
    eng.close()


def test_batch_next_tokens_are_the_argmax():
    cfg = SMALL_QWEN3
    a, b = Engine(cfg, seed=6, batch=4), Engine(cfg, seed=6, batch=4)
    toks = np.array([5, 6, 7, 8])
    for pos in range(5):
        poss = np.full(4, pos)
        logits = a.forward_batch(toks, poss)
        nxt = b.next_tokens(toks, poss)
        assert np.array_equal(nxt, logits.argmax(axis=1))
        toks = nxt
    a.close()
    b.close()


def test_batch_prefill_fills_its_sequence():
    """A batch engine's prefill of sequence i (its cache alone), then a step of all: sequence i sees its prompt,
    the others their own (empty) caches."""
    cfg = replace(SMALL_QWEN3, seq_len=128)
    W = synthetic_host_weights(cfg, seed=13)
    eng = Engine(cfg, host=W, batch=4)
    prompt = np.random.default_rng(3).integers(0, cfg.vocab, 40)
    eng.prefill(prompt, 0, need_logits=False, seq=2)
    single = Engine(cfg, host=W)
    single.prefill(prompt, 0, need_logits=False)
    want = single.forward(9, 40)
    got = eng.forward_batch([9, 9, 9, 9], [40, 40, 40, 40])
    check_logits(got[2], want, "prefilled", (0.0, 0.0))
    assert np.abs(got[0] - want).max() > 1e-3  # the others did not see the prompt
    eng.close()
    single.close()
