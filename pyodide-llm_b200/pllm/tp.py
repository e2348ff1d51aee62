"""Tensor-parallel decode across the GPUs of one node, one process a GPU (no counterpart in the reference, whose engine
splits a product's rows across the CPU threads of one memory: src/runtime/forward/threads.ts:90-133).

The split is Megatron's column / row parallelism over the reference's own unit of work (a product's row range,
jobs.ts's [r0, r1)): q/k/v by whole heads and w1/w3 by hidden rows (column-parallel: each rank makes its rows of the
output), wo and w2 by K at head and hidden boundaries (row-parallel: each rank makes a partial of every output row
from its share of the groups of 32, so every group's integer is the reference's), the classifier by vocab rows. A
layer then has two reductions, after wo and after w2: the exchange (exchange.cu) sends every rank's partial into
every rank's receive region over NVLink in the product's epilogue and sums them, in rank order, in the next
product's prologue. Attention, its cache and the head norms stay per rank (its heads).
"""
import ctypes
from dataclasses import dataclass

import numpy as np

from .lib import L, PllmError, check


@dataclass
class Shard:
    """Rank rank of world's share of a configuration's shapes."""
    cfg: object
    rank: int = 0
    world: int = 1

    def __post_init__(self):
        c, w = self.cfg, self.world
        if not 1 <= w <= 8 or not 0 <= self.rank < w:
            raise ValueError(f"rank {self.rank} of {w}: 1 to 8 ranks")
        bad = [name for name, v in (("heads", c.heads), ("kv_heads", c.kv_heads), ("hidden", c.hidden),
                                    ("vocab", c.vocab)) if v % w]
        if bad:
            raise ValueError(f"{', '.join(bad)} not divisible by {w} ranks")
        # the row-parallel products' K (a rank's q heads, its hidden rows) must suit the bulk-copy product (K % 128)
        if w > 1 and ((c.heads // w * c.head_size) % 128 or (c.hidden // w) % 128 or c.dim % 128):
            raise ValueError(f"a rank's K ({c.heads // w * c.head_size}, {c.hidden // w}) is not a multiple of 128")

    @property
    def heads(self):
        return self.cfg.heads // self.world

    @property
    def kv_heads(self):
        return self.cfg.kv_heads // self.world

    @property
    def qdim(self):
        return self.heads * self.cfg.head_size

    @property
    def kvdim(self):
        return self.kv_heads * self.cfg.head_size

    @property
    def rows_qkv(self):
        return self.qdim + 2 * self.kvdim

    @property
    def hidden(self):
        return self.cfg.hidden // self.world

    @property
    def vocab(self):
        return self.cfg.vocab // self.world

    def q_rows(self):
        return slice(self.rank * self.qdim, (self.rank + 1) * self.qdim)

    def kv_rows(self):
        return slice(self.rank * self.kvdim, (self.rank + 1) * self.kvdim)

    def hidden_rows(self):
        return slice(self.rank * self.hidden, (self.rank + 1) * self.hidden)

    def vocab_rows(self):
        return slice(self.rank * self.vocab, (self.rank + 1) * self.vocab)

    def host_share(self, W):
        """This rank's part of a host-weights dict (synthetic_host_weights' layout): per layer the q/k/v rows of its
        heads, wo's columns of its heads, w1/w3 rows of its hidden rows, w2's columns of them, its vocab rows of the
        classifier; the embedding, the norms and the RoPE tables whole."""
        g = lambda s: slice(s.start // 32, s.stop // 32)  # noqa: E731  the scales of a column range
        S = dict(W)
        q, kv, h, v = self.q_rows(), self.kv_rows(), self.hidden_rows(), self.vocab_rows()
        for k, rows in (("q", q), ("k", kv), ("v", kv), ("1", h), ("3", h)):
            S["w" + k], S["s" + k] = W["w" + k][:, rows], W["s" + k][:, rows]
        for k, cols in (("o", q), ("2", h)):
            S["w" + k], S["s" + k] = W["w" + k][:, :, cols], W["s" + k][:, :, g(cols)]
        S["cls"], S["cls_s"] = W["cls"][v], W["cls_s"][v]
        return {k: (np.ascontiguousarray(a) if isinstance(a, np.ndarray) else a) for k, a in S.items()}


class Exchange:
    """A rank's exchange region (pllm_tp_open), mapped into every other rank's process: the handles go round through
    a torch.distributed group (gloo is enough: 64 bytes a rank, once)."""

    def __init__(self, cfg, rank=0, world=1, group=None):
        self.rank, self.world, self.group = rank, world, group
        self.h = L.pllm_tp_open(world, rank, cfg.dim, cfg.layers)
        if not self.h:
            check("pllm_tp_open")
            raise PllmError(1, "pllm_tp_open failed")
        mine = ctypes.create_string_buffer(64)
        if L.pllm_tp_handle(self.h, mine):
            check("pllm_tp_handle")
        handles = [mine.raw]
        if world > 1:
            import torch.distributed as dist
            handles = [None] * world
            dist.all_gather_object(handles, mine.raw, group=group)
        joined = ctypes.create_string_buffer(b"".join(handles), 64 * world)
        if L.pllm_tp_connect(self.h, joined):
            check("pllm_tp_connect")
        self.barrier()

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier(group=self.group)

    def collectives(self, device):
        """The ranks' NCCL group for the prefill's reductions and the greedy step's key (made on first use: every rank
        reaches it in the same call, in the same order)."""
        if getattr(self, "_nccl", None) is None:
            import torch
            import torch.distributed as dist
            torch.cuda.set_device(device)
            self._nccl = dist.new_group(list(range(self.world)), backend="nccl")
            self._device = device
        return self._nccl

    def all_reduce(self, ptr, count, dtype, stream, op="sum"):
        """count elements (float32 or int64) of the library's device memory at ptr, summed (or their max) over the
        ranks in place, NCCL over NVLink, in order on the library's stream (its kernels before, after)."""
        import torch
        import torch.distributed as dist
        group = self.collectives(self._device if getattr(self, "_device", None) is not None else 0)
        typestr = {"f4": "<f4", "i8": "<i8"}[dtype]
        view = _DeviceView(ptr, count, typestr)
        t = torch.as_tensor(view, device=f"cuda:{self._device}")
        with torch.cuda.stream(torch.cuda.ExternalStream(stream, device=f"cuda:{self._device}")):
            dist.all_reduce(t, op=dist.ReduceOp.SUM if op == "sum" else dist.ReduceOp.MAX, group=group)

    def close(self):
        """Every rank stops using the exchange, then each unmaps the others' regions and frees its own."""
        if self.h:
            L.pllm_sync()
            self.barrier()
            L.pllm_tp_close(self.h)
            self.h = 0


class _DeviceView:
    """The CUDA array interface of count elements of the library's device memory (no copy; torch reads the pointer)."""

    def __init__(self, ptr, count, typestr):
        self.__cuda_array_interface__ = {"shape": (count,), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "stream": None}


def gather_logits(local, shard, group=None):
    """The ranks' vocab slices of the logits, whole on rank 0 (None on the others)."""
    if shard.world == 1:
        return local
    import torch
    import torch.distributed as dist
    parts = [torch.empty(shard.vocab, dtype=torch.float32) for _ in range(shard.world)] if shard.rank == 0 else None
    dist.gather(torch.from_numpy(np.ascontiguousarray(local)), parts, dst=0, group=group)
    return torch.cat(parts).numpy() if shard.rank == 0 else None
