"""Generates tests/golden/superblocks.npz: llama.cpp's blocks of 256 weights read by the reference's own NumPy reader
(src/python/convert/superblocks.py SUPERBLOCKS), to pin the oracle's reading of the ten types the reference's block
kernels multiply (kernels/blocks/types.ts) and, through it, the device's.

Run in a container that holds the reference read-only (its path in the environment variable PLLM_REFERENCE, which must be set):
    python tests/golden/make_superblocks.py
The output is committed; no test reads the reference at run time.

For each type: seeded random block bytes (any bytes are blocks, kernels/blocks/types.ts's head), with the float16
scales (d, dmin; IQ1_M's four nibbles of d) set to finite values of a model's size, and the float32 weights the
reader makes of them; plus the checkpoint's codebooks row (convert/grids.py's codebooks(), the bytes the reference's
kernels build their tables from: sb_tables, kernels/blocks/types.ts:294-322).
"""
import os
import sys

import numpy as np

REF = os.environ.get("PLLM_REFERENCE")
if not REF:
    sys.exit("set PLLM_REFERENCE to the reference's source tree (read-only)")
sys.path.insert(0, os.path.join(REF, "src", "python"))
from convert.grids import codebooks  # noqa: E402
from convert.superblocks import SUPERBLOCKS  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "superblocks.npz")
BLOCKS_EACH = 12
# where each type's float16 scales are (bytes): d (and dmin for the K types)
HALVES = {"Q2_K": (80, 82), "Q4_K": (0, 2), "IQ2_XXS": (0,), "IQ2_XS": (0,), "IQ2_S": (0,), "IQ3_XXS": (0,),
          "IQ3_S": (0,), "IQ1_S": (0,), "IQ4_XS": (0,), "IQ1_M": ()}


def main():
    rng = np.random.default_rng(11)
    out = {}
    books, places = codebooks()
    out["codebooks"] = np.frombuffer(books, dtype=np.uint8).copy()
    for name, (ggml, size, read) in SUPERBLOCKS.items():
        raw = rng.integers(0, 256, (BLOCKS_EACH, size), dtype=np.uint8)
        for at in HALVES[name]:
            d = (rng.uniform(0.002, 0.05, BLOCKS_EACH) * np.where(rng.random(BLOCKS_EACH) < 0.2, -1, 1))
            raw[:, at:at + 2] = d.astype("<f2").view(np.uint8).reshape(BLOCKS_EACH, 2)
        if name == "IQ1_M":  # d: the top four bits of the four scale words, the first word's the lowest
            d = rng.uniform(0.002, 0.05, BLOCKS_EACH).astype("<f2").view("<u2")
            for w in range(4):
                word = raw[:, 48 + 2 * w:50 + 2 * w].copy().view("<u2").reshape(-1)
                word = (word & 0x0fff) | (((d >> (4 * w)) & 15) << 12)
                raw[:, 48 + 2 * w:50 + 2 * w] = word.astype("<u2").view(np.uint8).reshape(BLOCKS_EACH, 2)
        out[f"{name}/ggml"] = np.array(ggml)
        out[f"{name}/blocks"] = raw
        out[f"{name}/weights"] = np.asarray(read(raw.tobytes()), np.float32).reshape(BLOCKS_EACH, 256)
        print(name, ggml, size)
    np.savez_compressed(OUT, **out)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
