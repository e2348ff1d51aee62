"""Generates tests/golden/checkpoints.npz: checkpoint files written by the reference's own code, and what the reference
reads from them, to pin the checkpoint reader (pyodide-llm_b200/pllm/checkpoint.py) and the forward driver on them.

Run in a container that holds the reference read-only (its path in the environment variable PLLM_REFERENCE, which must be set):
    python tests/golden/make_checkpoints.py
The output is committed; no test reads the reference at run time.

For each file: the bytes of tests/made_up.py's `quantized` (a made-up model of drawn() values, written through
made_up.checkpoint with the reference's packers: engine/packing.py's quantize, six, ternary, binary) in one dtype; then
what the reference's NumPy model (src/python/engine/model.py's Llama, no kernels) holds and computes:
  - the SHA-256 of the float32 bytes of every matrix it widened (wq ... w3, wcls: values times their group's scale);
  - the rows of a few tokens of its embedding (Llama.embedding);
  - its logits after each token of a short sequence at positions 0, 1, ... (Llama.forward): float32 weights and
    activations, a float32 cache; the int8 forward driver quantizes its activations in groups of 32 (quantize_x) and
    keeps a float16 cache, so these are met within the reference's own line for its int8 kernels against NumPy.
"""
import hashlib
import os
import sys

import numpy as np

REF = os.environ.get("PLLM_REFERENCE")
if not REF:
    sys.exit("set PLLM_REFERENCE to the reference's source tree (read-only)")
sys.path.insert(0, os.path.join(REF, "src", "python"))
sys.path.insert(0, os.path.join(REF, "tests"))
import made_up  # noqa: E402  (the reference's own made-up models)
from engine.model import Llama  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "checkpoints.npz")
MATRICES = ("wq", "wk", "wv", "wo", "w1", "w2", "w3", "wcls")
TOKENS = np.array([5, 17, 3, 60, 41, 8], dtype=np.int32)

# name: (dtype, made_up.quantized's arguments, the form)
FILES = {
    "int8_qwen3": ("int8", dict(dim=64, hidden=128, layers=2, heads=2, kv_heads=1, vocab=-96, seq_len=64, seed=0),
                   dict(qk_norm=True)),
    "int8_llama_shared": ("int8", dict(dim=64, hidden=96, layers=2, heads=2, kv_heads=2, vocab=96, seq_len=64, seed=1),
                          dict()),
    "int6_qwen3": ("int6", dict(dim=64, hidden=128, layers=2, heads=2, kv_heads=1, vocab=-96, seq_len=64, seed=2),
                   dict(qk_norm=True)),
    "ternary_qwen3": ("ternary", dict(dim=128, hidden=128, layers=2, heads=4, kv_heads=2, vocab=-96, seq_len=64,
                                      seed=3), dict(qk_norm=True)),
    "binary_llama": ("binary", dict(dim=128, hidden=128, layers=2, heads=4, kv_heads=2, vocab=-96, seq_len=64,
                                    seed=4), dict()),
}


def main():
    out = {}
    for name, (dtype, args, form) in FILES.items():
        data, tokenizer = made_up.quantized(dtype=dtype, **args, **form)
        model = Llama(data, tokenizer, dtype=dtype, **form)
        out[f"{name}/file"] = np.frombuffer(data, dtype=np.uint8).copy()
        for m in MATRICES:
            w = getattr(model, m, None)
            if w is not None:
                out[f"{name}/sha256/{m}"] = np.array(hashlib.sha256(np.ascontiguousarray(w, np.float32).tobytes())
                                                     .hexdigest())
        out[f"{name}/embedding"] = np.stack([np.asarray(model.embedding(int(t)), np.float32) for t in TOKENS])
        logits = [np.asarray(model.forward(int(t), pos), np.float32) for pos, t in enumerate(TOKENS)]
        out[f"{name}/logits"] = np.stack(logits)
        out[f"{name}/dtype"] = np.array(dtype)
        out[f"{name}/form"] = np.array(repr(sorted(form.items())))
        print(name, dtype, len(data), "bytes")
    out["tokens"] = TOKENS
    np.savez_compressed(OUT, **out)
    print("wrote", OUT, os.path.getsize(OUT), "bytes")


if __name__ == "__main__":
    main()
