"""One rank of a tensor-parallel check (launched by tests/test_gpu_tp.py under torch.distributed.run, one process a
GPU): the rank's share of a synthetic model decodes a few tokens with the exchange, then prefills a prompt on the tensor
cores (NCCL all-reduce of the row-parallel partials) and decodes after it, greedy tokens from next_token; rank 0
gathers the logits, runs the same with the whole model on its own GPU (no exchange), and writes the distances and
the tokens to --out."""
import argparse
import datetime
import json
import os
import sys
from dataclasses import replace

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "pyodide-llm_b200")]

import numpy as np  # noqa: E402
import torch.distributed as dist  # noqa: E402

from pllm.device import init  # noqa: E402
from pllm.forward import QWEN3_8B, Engine  # noqa: E402
from pllm.lib import L  # noqa: E402
from pllm.tp import Exchange, gather_logits  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--layers", type=int, default=4)
    ap.add_argument("--tokens", type=int, default=6)
    ap.add_argument("--prompt", type=int, default=40)
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    cfg = replace(QWEN3_8B, layers=args.layers, seq_len=64)
    init(local)
    xg = Exchange(cfg, rank, world)
    eng = Engine(cfg, seed=5, device=local, exchange=xg)
    tokens = np.random.default_rng(1).integers(0, cfg.vocab, args.tokens)
    got = [gather_logits(eng.forward(int(t), pos), eng.shard) for pos, t in enumerate(tokens)]
    # the tensor-core prefill across the ranks (NCCL all-reduce after wo and w2), then decode steps after it, each
    # step's logits gathered and its greedy token from next_token (the ranks' keys' max on the devices)
    prompt = np.random.default_rng(2).integers(0, cfg.vocab, args.prompt)
    eng.close()
    eng = Engine(cfg, seed=5, device=local, exchange=xg)
    pre = gather_logits(eng.prefill(prompt, 0), eng.shard)
    after, greedy = [], []
    for i, t in enumerate(tokens[:3]):
        pos = args.prompt + i
        after.append(gather_logits(eng.forward(int(t), pos), eng.shard))
        greedy.append(eng.next_token(int(t), pos))
    statuses = [None] * world
    dist.all_gather_object(statuses, int(L.pllm_device_status()))
    tokens_of = [None] * world
    dist.all_gather_object(tokens_of, greedy)
    eng.close()
    xg.close()
    if rank == 0:
        ref = Engine(cfg, seed=5, device=local)
        rows = []
        for pos, t in enumerate(tokens):
            want, g = ref.forward(int(t), pos), got[pos]
            rows.append({"pos": pos, "rel": float(np.linalg.norm(g - want) / np.linalg.norm(want)),
                         "peak": float(np.abs(g - want).max() / np.abs(want).max()),
                         "argmax": [int(np.argmax(g)), int(np.argmax(want))]})
        ref.close()
        ref = Engine(cfg, seed=5, device=local)
        prefill_rows = []
        want = ref.prefill(prompt, 0)
        prefill_rows.append({"pos": "prefill", "rel": float(np.linalg.norm(pre - want) / np.linalg.norm(want)),
                             "peak": float(np.abs(pre - want).max() / np.abs(want).max()),
                             "argmax": [int(np.argmax(pre)), int(np.argmax(want))]})
        for i, t in enumerate(tokens[:3]):
            want, g = ref.forward(int(t), args.prompt + i), after[i]
            prefill_rows.append({"pos": args.prompt + i, "rel": float(np.linalg.norm(g - want) / np.linalg.norm(want)),
                                 "peak": float(np.abs(g - want).max() / np.abs(want).max()),
                                 "argmax": [int(np.argmax(g)), int(np.argmax(want))]})
        ref.close()
        with open(args.out, "w") as f:
            json.dump({"world": world, "statuses": statuses, "rows": rows, "prefill_rows": prefill_rows,
                       "greedy": tokens_of, "gathered_argmax": [int(np.argmax(g)) for g in after]}, f)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
