"""Tensor parallelism's host side, on the CPU: the ranks' shares of a model (pllm.tp.Shard), the arithmetic of the
K split (every group's integer unchanged, the partials summing to the whole product), and the exchange's handle
round and the logits gather over a 2-rank gloo group (the library faked: no GPU here)."""
import datetime
import os
import socket
from dataclasses import replace

import numpy as np
import pytest

import oracle as O
from pllm.forward import QWEN3_8B, STORIES15M, Config, quantize_rows, synthetic_host_weights
from pllm.tp import Shard

SMALL = Config(dim=256, hidden=512, layers=2, heads=8, kv_heads=4, head_size=64, vocab=1024, seq_len=64,
               qk_norm=True, rope_theta=1e6, eps=1e-6)


def test_shard_shapes_qwen3_8b():
    for world in (1, 2, 4, 8):
        shares = [Shard(QWEN3_8B, r, world) for r in range(world)]
        assert sum(s.qdim for s in shares) == QWEN3_8B.qdim
        assert sum(s.kvdim for s in shares) == QWEN3_8B.kvdim
        assert sum(s.hidden for s in shares) == QWEN3_8B.hidden
        assert sum(s.vocab for s in shares) == QWEN3_8B.vocab
        assert shares[-1].vocab_rows().stop == QWEN3_8B.vocab
        assert all(s.kv_heads >= 1 and s.heads // s.kv_heads == 4 for s in shares)  # GQA ratio kept


def test_shard_refusals():
    with pytest.raises(ValueError):
        Shard(QWEN3_8B, 0, 3)  # 32 heads over 3 ranks
    with pytest.raises(ValueError):
        Shard(QWEN3_8B, 2, 2)
    with pytest.raises(ValueError):
        Shard(STORIES15M, 0, 2)  # a rank's K (3 heads of 48) is not a multiple of 128
    Shard(STORIES15M)  # one rank: any shape


def test_host_shares_reassemble():
    cfg = replace(SMALL, kv_heads=8)
    W = synthetic_host_weights(cfg, seed=3)
    world = 2
    S = [Shard(cfg, r, world).host_share(W) for r in range(world)]
    for k in ("q", "k", "v", "1", "3"):  # column-parallel: rows
        assert np.array_equal(np.concatenate([s["w" + k] for s in S], axis=1), W["w" + k])
        assert np.array_equal(np.concatenate([s["s" + k] for s in S], axis=1), W["s" + k])
    for k in ("o", "2"):  # row-parallel: K (whole groups: scales follow)
        assert np.array_equal(np.concatenate([s["w" + k] for s in S], axis=2), W["w" + k])
        assert np.array_equal(np.concatenate([s["s" + k] for s in S], axis=2), W["s" + k])
    assert np.array_equal(np.concatenate([s["cls"] for s in S]), W["cls"])
    assert all(np.array_equal(s["emb"], W["emb"]) for s in S)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_k_split_keeps_group_integers(world):
    """wo / w2 split along K at group boundaries: the groups' integers are the whole product's, and the ranks'
    partials sum to its output within float32 rounding (only the order of the float32 sums changes)."""
    rng = np.random.default_rng(world)
    rows, K = 96, 1024
    w, s = quantize_rows(rng.normal(0, 0.02, (rows, K)).astype(np.float32))
    xq, xs = O.quantize_x(rng.normal(0, 1, K).astype(np.float32))
    whole = O.group_sums_q8(xq, w)
    step = K // world
    total = np.zeros(rows, np.float32)
    for r in range(world):  # rank order, as the exchange sums them
        cols, groups = slice(r * step, (r + 1) * step), slice(r * step // 32, (r + 1) * step // 32)
        assert np.array_equal(O.group_sums_q8(xq[cols], w[:, cols]), whole[:, groups])
        total += O.matmul_q8(xq[cols], xs[groups], w[:, cols], s[:, groups])
    full = O.matmul_q8(xq, xs, w, s)
    assert np.allclose(total, full, rtol=1e-5, atol=1e-6 * np.abs(full).max())


def test_activation_quantization_splits_at_groups():
    """A rank quantizes its slice of the attention output (or of hb) itself: quantize_x works group by group, so the
    slices' bytes and scales are the whole vector's."""
    x = np.random.default_rng(1).normal(0, 1, 4096).astype(np.float32)
    xq, xs = O.quantize_x(x)
    for world in (2, 4, 8):
        step = 4096 // world
        for r in range(world):
            q, sc = O.quantize_x(x[r * step:(r + 1) * step])
            assert np.array_equal(q, xq[r * step:(r + 1) * step])
            assert np.array_equal(sc, xs[r * step // 32:(r + 1) * step // 32])


# ---- the handle round and the gather over gloo (2 ranks, the library faked)

class FakeLib:
    """What Exchange calls of the library, on the host: a handle is 64 bytes naming its rank."""

    def __init__(self, rank):
        self.rank, self.connected, self.closed = rank, None, None

    def pllm_tp_open(self, world, rank, dim, layers):
        assert rank == self.rank
        return 1000 + rank

    def pllm_tp_handle(self, h, buf):
        buf.raw = bytes([self.rank]) * 64
        return 0

    def pllm_tp_connect(self, h, joined):
        self.connected = bytes(joined.raw)
        return 0

    def pllm_sync(self):
        return 0

    def pllm_tp_close(self, h):
        self.closed = h


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import torch.distributed as dist
    import pllm.tp as tp
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    fake = FakeLib(rank)
    tp.L = fake
    x = tp.Exchange(SMALL, rank, world)
    ok = fake.connected == b"".join(bytes([r]) * 64 for r in range(world))
    shard = Shard(SMALL, rank, world)
    local = np.arange(shard.vocab, dtype=np.float32) + rank * shard.vocab
    whole = tp.gather_logits(local, shard)
    if rank == 0:
        ok = ok and whole is not None and np.array_equal(whole, np.arange(SMALL.vocab, dtype=np.float32))
    else:
        ok = ok and whole is None
    x.close()
    ok = ok and fake.closed == 1000 + rank
    dist.destroy_process_group()
    out.put((rank, bool(ok)))


def test_exchange_round_over_gloo():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: True, 1: True}
