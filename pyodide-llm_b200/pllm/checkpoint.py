"""The reference's checkpoint files, read into the forward driver's host weights (Engine(cfg, host=W)).

A checkpoint is llama2.c's file as the reference extends it: a header of 7 int32 (dim, hidden_dim, n_layers, n_heads,
n_kv_heads, vocab_size, seq_len; a negative vocabulary says the classifier is a tensor of its own), then every tensor
in file order, each stored by its kind (src/python/engine/layout.py:689-713 `placed`):
  - the Llama / Qwen3 rows in file order (layout.py:378-388 `llama`, :342-370 the parts): the embedding, the stacks of
    rms_att_weight, wq, wk, wv, wo, rms_ffn_weight, w1, w2, w3 (a tensor for all layers, layer after layer), the final
    norm, the RoPE tables (freq_cis_real, freq_cis_imag), the classifier where the header says so, the q / k / v biases
    (form "bias"), the heads' norms q_norm and k_norm (form "qk_norm");
  - a row's kind (layout.py:658-668 `kind_of`): in a file of a quantized dtype the vectors are float32 and the RoPE
    tables are left out (computed from rope_theta), everything else is the file's dtype; in a float32 or float16 file
    every row is of that type;
  - a quantized kind (src/python/engine/dtypes.py:39-80, :125-140) stores a tensor's values in groups along the row,
    then one scale a group: int8 (groups of 32, or of the largest power of two below that divides the row:
    packing.py:32-37; float32 scales), int6 (24 bytes a group of 32, packing.py:56-71; float32 scales), ternary (2 bits
    a weight, 32 bytes a group of 128, packing.py:102-115; float16 scales), binary (1 bit a weight, 16 bytes a group of
    128, packing.py:148-162; float16 scales).
The dtype is the one whose file size the header gives (engine/checkpoint.py's checkpoint_dtype reads it the same way).

The forward driver multiplies int8 groups of 32. The other kinds become exactly such groups where they are exactly
such groups: an int6 group is an int8 group of multiples of 4 and a quarter of the scale (packing.py:48-53: the same
products to the bit); a ternary or binary group of 128 is four int8 groups of -1 / 0 / 1 with the group's scale (the
integer sums the reference's t2 / b1 products make, summed in float32 in another order). A float32 or float16 file is
quantized as the reference's quantize.py writes an int8 file (packing.py:40-45).

What this engine does not run is refused by name: the q / k / v biases (Qwen2), another architecture than a Llama
(with or without Qwen3's head norms), and a final norm whose largest weight is 4 times its median (the reference takes
8 outlier channels of such a norm apart in the classifier: engine/checkpoint.py OUTLIER_RATIO)."""
import math
import struct
from dataclasses import dataclass

import numpy as np

from .forward import Config, quantize_rows, rope_tables

HEADER = 28
MATRIX, VECTOR, TABLE, EMBEDDING, CLASSIFIER = "matrix", "vector", "table", "embedding", "classifier"
OUTLIER_RATIO = 4.0


@dataclass(frozen=True)
class Form:
    """What the header cannot say, as the caller says it (the reference's FORM options of a Llama)."""
    qk_norm: bool = False      # Qwen3: the RMSNorm weights of q's and k's heads after the rows (layout.py:353-355)
    bias: bool = False         # Qwen2: q / k / v biases (refused: this engine has none)
    head_dim: int = 0          # a head's size where it is not dim / n_heads
    rope_theta: float = 10000.0
    eps: float = 1e-5          # rms_norm_eps
    arch: str = "llama"


@dataclass(frozen=True)
class Row:
    name: str
    role: str
    shape: tuple


def llama_rows(header, form):
    """The tensors of a Llama / Qwen3 checkpoint, in file order (layout.py:378-388)."""
    dim, hidden, layers, heads, kv_heads, vocab, seq_len = header
    hs = form.head_dim or dim // heads
    q, kv, v = heads * hs, kv_heads * hs, abs(vocab)
    rows = [Row("token_embedding_table", EMBEDDING, (v, dim)),
            Row("rms_att_weight", VECTOR, (layers, dim)),
            Row("wq", MATRIX, (layers, q, dim)), Row("wk", MATRIX, (layers, kv, dim)),
            Row("wv", MATRIX, (layers, kv, dim)), Row("wo", MATRIX, (layers, dim, q)),
            Row("rms_ffn_weight", VECTOR, (layers, dim)),
            Row("w1", MATRIX, (layers, hidden, dim)), Row("w2", MATRIX, (layers, dim, hidden)),
            Row("w3", MATRIX, (layers, hidden, dim)),
            Row("rms_final_weight", VECTOR, (dim,)),
            Row("freq_cis_real", TABLE, (seq_len, hs // 2)), Row("freq_cis_imag", TABLE, (seq_len, hs // 2))]
    if vocab < 0:
        rows.append(Row("wcls", CLASSIFIER, (v, dim)))
    if form.bias:
        rows += [Row("bq", VECTOR, (layers, q)), Row("bk", VECTOR, (layers, kv)), Row("bv", VECTOR, (layers, kv))]
    if form.qk_norm:
        rows += [Row("q_norm", VECTOR, (layers, hs)), Row("k_norm", VECTOR, (layers, hs))]
    return rows


def group32(length):
    """An int8 row's group: 32, or the largest power of two below it that divides the row (packing.py:32-37)."""
    size = 32
    while length % size:
        size //= 2
    return size


@dataclass(frozen=True)
class Kind:
    """How a tensor is stored (dtypes.py:39-80): itemsize for a plain one; else bits a value in groups, a scale of
    scale_bytes (4: float32, 2: float16) after all the values."""
    name: str
    itemsize: int = 0
    bits: int = 0
    group: int = 0        # 0: group32 of the row (int8)
    scale_bytes: int = 4

    def group_of(self, length):
        return group32(length) if self.group == 0 else self.group

    def stored(self, count, length):
        """(bytes of the values, bytes of the scales) of count values in rows of this length (dtypes.py:75-77)."""
        if not self.bits:
            return count * self.itemsize, 0
        g = self.group_of(length)
        return count // g * (g * self.bits // 8), self.scale_bytes * (count // g)


KINDS = {k.name: k for k in (Kind("float32", itemsize=4), Kind("float16", itemsize=2), Kind("int8", bits=8),
                             Kind("int6", bits=6, group=32), Kind("ternary", bits=2, group=128, scale_bytes=2),
                             Kind("binary", bits=1, group=128, scale_bytes=2))}
QUANTIZED = ("int8", "int6", "ternary", "binary")


def kind_of(row, dtype):
    """A row's kind in a file of this dtype, None where the file leaves it out (layout.py:658-668)."""
    if dtype not in QUANTIZED:
        return dtype
    return "float32" if row.role == VECTOR else None if row.role == TABLE else dtype


@dataclass(frozen=True)
class Place:
    row: Row
    kind: str      # None: not in the file
    offset: int    # of its values
    size: int      # all its bytes
    scales: int    # offset of its scales (quantized kinds), else 0


def placed(rows, dtype, offset=HEADER):
    """Every row's place, one tensor after the other behind the header (layout.py:689-707)."""
    out = []
    for row in rows:
        kind = kind_of(row, dtype)
        if kind is None:
            out.append(Place(row, None, offset, 0, 0))
            continue
        values, scales = KINDS[kind].stored(math.prod(row.shape), row.shape[-1])
        out.append(Place(row, kind, offset, values + scales, offset + values if scales else 0))
        offset += values + scales
    return out


def file_size(rows, dtype):
    return HEADER + sum(p.size for p in placed(rows, dtype))


def suits(rows, dtype):
    """Whether every row of the file's kinds is whole groups (dtypes.py:82-84)."""
    for row in rows:
        kind = kind_of(row, dtype)
        if kind is not None and KINDS[kind].bits and row.shape[-1] % KINDS[kind].group_of(row.shape[-1]):
            return False
    return True


def unpack6(raw):
    """24 bytes a group of 32 -> its int8 values (multiples of 4): value j's low four bits in byte j % 16 (j < 16 the
    low nibble, else the high one), its top two bits in byte 16 + j % 8 at bits 2 (j // 8) (packing.py:56-71)."""
    b = np.asarray(raw, dtype=np.uint8).reshape(-1, 24)
    low = np.concatenate([b[:, :16] & 15, b[:, :16] >> 4], axis=1)
    top = np.concatenate([(b[:, 16:] >> s) & 3 for s in (0, 2, 4, 6)], axis=1)
    return ((low | (top << 4)) << 2).astype(np.uint8).view(np.int8)


def unpack_ternary(raw):
    """A byte for four weights, weight j's code (w + 1) at bits 2 (j % 4) of byte j // 4 (packing.py:102-115)."""
    b = np.asarray(raw, dtype=np.uint8).reshape(-1, 1)
    return (((b >> np.array([0, 2, 4, 6], dtype=np.uint8)) & 3).astype(np.int8) - 1).reshape(-1)


def unpack_binary(raw):
    """16 bytes a group of 128, weight 64 h + 4 c + p at bit 4 h + p of byte c, set for +1 (packing.py:148-162)."""
    b = np.asarray(raw, dtype=np.uint8).reshape(-1, 16)
    bits = (b[:, :, None] >> np.arange(8, dtype=np.uint8)) & 1          # [group][c][4 h + p]
    signs = bits.reshape(-1, 16, 2, 4).transpose(0, 2, 1, 3).reshape(-1)  # [group][h][c][p] = weight 64 h + 4 c + p
    return signs.astype(np.int8) * np.int8(2) - np.int8(1)


class Checkpoint:
    """A checkpoint file: its header, form, dtype and every row's place; the tensors read on request."""

    def __init__(self, path, form=Form(), dtype=None):
        self.path, self.form = path, form
        self.data = np.memmap(path, dtype=np.uint8, mode="r")
        if self.data.size < HEADER:
            raise ValueError(f"{path}: {self.data.size} bytes, no header")
        self.header = struct.unpack_from("<7i", bytes(self.data[:HEADER]), 0)
        dim, hidden, layers, heads, kv_heads, vocab, seq_len = self.header
        if min(dim, hidden, layers, heads, kv_heads, abs(vocab), seq_len) <= 0 or heads % kv_heads:
            raise ValueError(f"{path}: not a checkpoint header {self.header}")
        if form.arch != "llama":
            raise ValueError(f"architecture {form.arch!r}: this engine runs a Llama (with or without Qwen3's head norms)")
        self.rows = llama_rows(self.header, form)
        sizes = {d: file_size(self.rows, d) for d in KINDS if suits(self.rows, d)}
        if dtype is None:
            found = [d for d, s in sizes.items() if s == self.data.size]
            if not found:
                raise ValueError(f"{path}: {self.data.size} bytes is the size of no dtype of this header and form "
                                 f"({sizes})")
            dtype = found[0]
        elif sizes.get(dtype) != self.data.size:
            raise ValueError(f"{path}: {self.data.size} bytes, a {dtype} file of this header is {sizes.get(dtype)}")
        self.dtype = dtype
        self.places = {p.row.name: p for p in placed(self.rows, dtype)}

    def raw(self, name):
        """(the kind, the values' bytes or array, the scales or None) of a row as the file holds it."""
        p = self.places[name]
        if p.kind is None:
            return None, None, None
        k, n = KINDS[p.kind], math.prod(p.row.shape)
        if not k.bits:
            dt = np.float32 if p.kind == "float32" else np.float16
            return p.kind, np.frombuffer(self.data, dtype=dt, count=n, offset=p.offset).reshape(p.row.shape), None
        g = k.group_of(p.row.shape[-1])
        values = np.frombuffer(self.data, dtype=np.uint8, count=p.scales - p.offset, offset=p.offset)
        st = np.float32 if k.scale_bytes == 4 else np.float16
        scales = np.frombuffer(self.data, dtype=st, count=n // g, offset=p.scales)
        return p.kind, values, scales

    def int8(self, name):
        """A matrix as int8 groups of 32: (values [.., rows, K] int8, scales [.., rows, K / 32] float32)."""
        shape = self.places[name].row.shape
        kind, values, scales = self.raw(name)
        K = shape[-1]
        if K % 32:
            raise ValueError(f"{name}: rows of {K} values; the products take whole groups of 32")
        if kind in ("float32", "float16"):  # quantize.py's int8 (packing.py:40-45)
            return quantize_rows(np.asarray(values, dtype=np.float32).reshape(shape))
        if kind == "int8":
            g = group32(K)
            if g != 32:
                raise ValueError(f"{name}: int8 groups of {g}; the products take groups of 32")
            return values.view(np.int8).reshape(shape), scales.astype(np.float32).reshape(shape[:-1] + (K // 32,))
        if kind == "int6":  # the same products to the bit: 4 v and s / 4 (packing.py:48-53)
            return unpack6(values).reshape(shape), scales.astype(np.float32).reshape(shape[:-1] + (K // 32,))
        q = unpack_ternary(values) if kind == "ternary" else unpack_binary(values)
        if kind == "ternary" and np.any(q > 1):
            raise ValueError(f"{name}: a ternary code 3, which no ternary file holds")
        s = np.repeat(scales.astype(np.float32).reshape(-1, 1), 4, axis=1)  # a group of 128: four groups of 32
        return q.reshape(shape), s.reshape(shape[:-1] + (K // 32,))

    def floats(self, name):
        kind, values, _ = self.raw(name)
        if kind not in ("float32", "float16"):
            raise ValueError(f"{name}: a vector stored as {kind}")
        return np.asarray(values, dtype=np.float32).reshape(self.places[name].row.shape)

    def config(self, seq_len=None, **more):
        dim, hidden, layers, heads, kv_heads, vocab, file_seq = self.header
        f = self.form
        return Config(dim=dim, hidden=hidden, layers=layers, heads=heads, kv_heads=kv_heads,
                      head_size=f.head_dim or dim // heads, vocab=abs(vocab), seq_len=seq_len or file_seq,
                      qk_norm=f.qk_norm, rope_theta=f.rope_theta, eps=f.eps, **more)

    def host_weights(self, cfg):
        """The forward driver's host weights (the keys synthetic_host_weights makes) of this checkpoint."""
        if self.form.bias:
            raise ValueError("q / k / v biases (Qwen2): this engine has none")
        W = {}
        for ours, theirs in (("q", "wq"), ("k", "wk"), ("v", "wv"), ("o", "wo"), ("1", "w1"), ("2", "w2"),
                             ("3", "w3")):
            W["w" + ours], W["s" + ours] = self.int8(theirs)
        W["emb"], W["emb_s"] = self.int8("token_embedding_table")
        W["cls"], W["cls_s"] = self.int8("wcls") if "wcls" in self.places else (W["emb"], W["emb_s"])
        W["att_norm"] = self.floats("rms_att_weight")
        W["ffn_norm"] = self.floats("rms_ffn_weight")
        W["final_norm"] = self.floats("rms_final_weight")
        w = np.abs(W["final_norm"])
        if w.max() >= OUTLIER_RATIO * np.median(w):
            raise ValueError("the final norm's largest weight is 4 times its median: the reference takes its outlier "
                             "channels apart in the classifier, which this engine does not")
        W["q_norm"] = self.floats("q_norm") if self.form.qk_norm else None
        W["k_norm"] = self.floats("k_norm") if self.form.qk_norm else None
        if self.places["freq_cis_real"].kind is not None and cfg.seq_len <= self.header[6]:
            W["cos_t"] = np.ascontiguousarray(self.floats("freq_cis_real")[:cfg.seq_len])
            W["sin_t"] = np.ascontiguousarray(self.floats("freq_cis_imag")[:cfg.seq_len])
        else:
            W["cos_t"], W["sin_t"] = rope_tables(cfg)
        return {k: (np.ascontiguousarray(v) if v is not None else None) for k, v in W.items()}


def load(path, form=Form(), seq_len=None, **engine_options):
    """An Engine of a checkpoint file: (engine, its Config)."""
    from .forward import Engine
    ck = Checkpoint(path, form)
    cfg = ck.config(seq_len)
    return Engine(cfg, host=ck.host_weights(cfg), **engine_options), cfg
