"""Generates tests/golden/sampling.npz: tokens the reference's NumPy sampler draws (src/python/engine/sampler.py's
NumpySampler.drawing, the sampler the reference's sample kernel restates: kernels/kernel/sample.ts:1-2), to pin the
oracle's sample (or_sample) and through it the device's.

Run in a container that holds the reference read-only (its path in the environment variable PLLM_REFERENCE, which must be set):
    python tests/golden/make_sampling.py
The output is committed; no test reads the reference at run time.

Seeded logits of three vocabularies (normal, of a few spreads, with ties), a grid of settings (temperature, topp,
top_k, min_p; no penalties), and random numbers handed to the sampler in place of its generator's: every draw's token.
"""
import itertools
import os
import sys

import numpy as np

REF = os.environ.get("PLLM_REFERENCE")
if not REF:
    sys.exit("set PLLM_REFERENCE to the reference's source tree (read-only)")
sys.path.insert(0, os.path.join(REF, "src", "python"))
from engine.sampler import NumpySampler, Sampling  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sampling.npz")


class Numbers:
    """An rng whose random() hands out the given numbers."""

    def __init__(self, numbers):
        self.numbers = list(numbers)

    def random(self):
        return self.numbers.pop(0)


def main():
    rng = np.random.default_rng(7)
    vocabularies = []
    for n, spread in ((50, 1.0), (1000, 3.0), (4096, 6.0)):
        x = (rng.standard_normal(n) * spread).astype(np.float32)
        x[n // 3] = x[n // 5]  # a tie
        vocabularies.append(x)
    settings = list(itertools.product((0.7, 1.0, 1.3), (0.0, 0.5, 0.9, 1.0), (0, 1, 40), (0.0, 0.05)))
    randoms = rng.random(6)
    rows = []
    for v, x in enumerate(vocabularies):
        for (temperature, topp, top_k, min_p) in settings:
            draw = NumpySampler().drawing(Sampling(temperature=temperature, topp=topp, top_k=top_k, min_p=min_p),
                                          Numbers(randoms))
            for r in randoms:
                token = draw(x.copy(), [], [])
                rows.append((v, temperature, topp, top_k, min_p, r, token))
    a = np.array(rows, dtype=np.float64)
    np.savez_compressed(OUT, logits0=vocabularies[0], logits1=vocabularies[1], logits2=vocabularies[2], draws=a)
    print("wrote", OUT, os.path.getsize(OUT), "bytes,", len(rows), "draws")


if __name__ == "__main__":
    main()
