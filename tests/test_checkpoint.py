"""The checkpoint reader (pllm/checkpoint.py) against files the reference wrote and what the reference read from them
(tests/golden/checkpoints.npz, made by tests/golden/make_checkpoints.py from tests/made_up.py's `quantized` and
src/python/engine/model.py's Llama):
  - the dtype found from the file's size, and every row's place (a misplaced row reads as other numbers);
  - every matrix widened to float32 (values times their group's scale) equal to the reference's to the bit (SHA-256 of
    the bytes), for int8, int6, ternary and binary files, with and without a classifier of its own;
  - the embedding's rows equal to the reference's;
  - the oracle's int8 forward (quantize_x activations, a float16 cache) on the weights read, against the reference's
    NumPy forward (float32 throughout) on the same file: the reference's own line for its int8 kernels against NumPy
    (tests/forward-check.ts:1-15: the greedy token at 85 % of the positions or more), and a relative distance of the
    logits of 5e-2 on average (0.12 at most).
And the refusals: a file of no dtype's size, a form this engine does not run."""
import hashlib
import os

import numpy as np
import pytest

import oracle as O
from pllm.checkpoint import Checkpoint, Form, llama_rows, placed, unpack6, unpack_binary, unpack_ternary

from test_gpu_forward import oracle_arrays, oracle_config

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "checkpoints.npz"))
NAMES = sorted({k.split("/")[0] for k in GOLDEN.files if "/" in k})
OURS = (("wq", "q"), ("wk", "k"), ("wv", "v"), ("wo", "o"), ("w1", "1"), ("w2", "2"), ("w3", "3"), ("wcls", "cls"))


def form_of(name):
    return Form(**dict(eval(str(GOLDEN[f"{name}/form"]))))


@pytest.fixture(scope="module")
def files(tmp_path_factory):
    d = tmp_path_factory.mktemp("checkpoints")
    out = {}
    for name in NAMES:
        p = str(d / f"{name}.bin")
        GOLDEN[f"{name}/file"].tofile(p)
        out[name] = p
    return out


def widened(w, s):
    K = w.shape[-1]
    return (w.astype(np.float32).reshape(*w.shape[:-1], K // 32, 32) * s[..., None]).reshape(w.shape)


@pytest.mark.parametrize("name", NAMES)
def test_reads_the_reference_files(files, name):
    ck = Checkpoint(files[name], form_of(name))
    assert ck.dtype == str(GOLDEN[f"{name}/dtype"])
    cfg = ck.config()
    W = ck.host_weights(cfg)
    checked = 0
    for theirs, ours in OURS:
        key = f"{name}/sha256/{theirs}"
        if key not in GOLDEN.files:
            continue
        w, s = (W["cls"], W["cls_s"]) if ours == "cls" else (W["w" + ours], W["s" + ours])
        assert hashlib.sha256(widened(w, s).tobytes()).hexdigest() == str(GOLDEN[key]), theirs
        checked += 1
    assert checked == len(OURS)
    rows = np.stack([widened(W["emb"][t], W["emb_s"][t]) for t in GOLDEN["tokens"]])
    assert np.array_equal(rows, GOLDEN[f"{name}/embedding"])


def test_oracle_forward_on_the_files_meets_the_reference(files):
    agree, total, rels = 0, 0, []
    for name in NAMES:
        ck = Checkpoint(files[name], form_of(name))
        cfg = ck.config()
        A, oc = oracle_arrays(cfg, ck.host_weights(cfg)), oracle_config(cfg)
        for pos, t in enumerate(GOLDEN["tokens"]):
            got, want = O.forward(oc, A, int(t), pos), GOLDEN[f"{name}/logits"][pos]
            rels.append(float(np.linalg.norm(got - want) / np.linalg.norm(want)))
            agree += int(np.argmax(got) == np.argmax(want))
            total += 1
    print(f"greedy token agreement {agree}/{total}, relative distance mean {np.mean(rels):.2e} max {max(rels):.2e}")
    assert agree >= 0.85 * total and np.mean(rels) <= 5e-2 and max(rels) <= 0.12


def test_places_follow_the_layout():
    """The rows of a Qwen3 int8 file, one after the other behind the header: values then scales; vectors float32;
    no RoPE tables in a quantized file; the classifier where the vocabulary is negative."""
    header = (64, 128, 2, 2, 1, -96, 64)
    rows = llama_rows(header, Form(qk_norm=True))
    names = [r.name for r in rows]
    assert names[:3] == ["token_embedding_table", "rms_att_weight", "wq"] and names[-3:] == ["wcls", "q_norm", "k_norm"]
    places = {p.row.name: p for p in placed(rows, "int8")}
    assert places["token_embedding_table"].offset == 28
    assert places["token_embedding_table"].size == 96 * 64 + 96 * 2 * 4
    assert places["freq_cis_real"].kind is None and places["freq_cis_real"].size == 0
    assert places["rms_att_weight"].kind == "float32"
    wq = places["wq"]
    assert wq.scales == wq.offset + 2 * 64 * 64 and wq.size == 2 * 64 * 64 * 9 // 8
    assert places["wcls"].offset == places["freq_cis_imag"].offset
    assert "wcls" not in [r.name for r in llama_rows((64, 128, 2, 2, 1, 96, 64), Form())]


def test_unpacking_round_trips():
    """The packings' layouts, written here in the other direction: int6's low nibbles and top bits, ternary's codes,
    binary's bit of weight 64 h + 4 c + p."""
    rng = np.random.default_rng(0)
    v = rng.integers(-32, 32, (3, 32)).astype(np.int8)
    b = (v.view(np.uint8) & 63).astype(np.uint8)
    packed = np.concatenate([(b[:, :16] & 15) | ((b[:, 16:] & 15) << 4),
                             (b[:, 0:8] >> 4) | ((b[:, 8:16] >> 4) << 2) | ((b[:, 16:24] >> 4) << 4) |
                             ((b[:, 24:32] >> 4) << 6)], axis=1)
    assert np.array_equal(unpack6(packed), (v * 4).astype(np.int8))
    t = rng.integers(-1, 2, 256).astype(np.int8)
    codes = (t.reshape(-1, 4) + 1).astype(np.uint8)
    assert np.array_equal(unpack_ternary(codes[:, 0] | codes[:, 1] << 2 | codes[:, 2] << 4 | codes[:, 3] << 6), t)
    s = np.where(rng.random(256) < 0.5, -1, 1).astype(np.int8)
    raw = np.zeros((2, 16), np.uint8)
    for g in range(2):
        for j in range(128):
            h, c, p = j // 64, (j % 64) // 4, j % 4
            if s[128 * g + j] > 0:
                raw[g, c] |= 1 << (4 * h + p)
    assert np.array_equal(unpack_binary(raw), s)


def test_refusals(files, tmp_path):
    name = NAMES[0]
    short = tmp_path / "short.bin"
    GOLDEN[f"{name}/file"][:-4].tofile(str(short))
    with pytest.raises(ValueError, match="size of no dtype"):
        Checkpoint(str(short), form_of(name))
    with pytest.raises(ValueError, match="architecture"):
        Checkpoint(files[name], Form(arch="gpt2"))
    with pytest.raises(ValueError, match="size of no dtype"):  # a form whose rows the file does not hold
        Checkpoint(files["int8_qwen3"], Form(qk_norm=False))
    with pytest.raises(ValueError):
        Checkpoint(files["int8_qwen3"], Form(qk_norm=True), dtype="int6")
