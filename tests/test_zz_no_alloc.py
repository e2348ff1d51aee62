"""The attention variant for callers that cannot allocate device memory (pllm_attention_f16_noalloc): a caller that
owns a fixed device arena, or runs where an allocation is not allowed, gets the same attention as attention_f16
without handing it a scratch buffer; the partials live in the library's own 4 MiB device array. Checked through the
C ABI against attention_f16 (the existing entry point, with its att scratch) and against the oracle's attention
(the reference's attentionOf restated on the CPU), within the attention's tolerance (1e-4 relative, 2e-5 absolute),
on two calls in a row; and a shape whose partials exceed the array is refused.
This file is collected last, so that a failure here comes after every other test has run."""
import numpy as np
import pytest

import oracle as O
from pllm.device import Buffer, init
from pllm.lib import L, PllmError, check

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def device():
    init(0)
    L.pllm_set_stream(0)
    yield
    L.pllm_device_sync()


def test_noalloc_attention_matches_attention_f16():
    rng = np.random.default_rng(17)
    nh, nkv, hs = 32, 8, 128
    keep = []
    for call, pos in enumerate((700, 2047)):  # two calls in a row, the second with more slices than the first
        count = pos + 1
        q = rng.normal(0, 1, nh * hs).astype(np.float32)
        kc, _ = O.to_f16(rng.normal(0, 1, (count, nkv * hs)).astype(np.float32))
        vc, _ = O.to_f16(rng.normal(0, 1, (count, nkv * hs)).astype(np.float32))
        Q, K, V = Buffer.of(q), Buffer.of(kc), Buffer.of(vc)
        want, got = Buffer(nh * hs * 4), Buffer(nh * hs * 4)
        att = Buffer(nh * count * 4)
        keep += [Q, K, V, want, got, att]
        L.attention_f16(want.ptr, Q.ptr, K.ptr, V.ptr, att.ptr, pos, nh, nkv, hs, 0, nh)
        check("attention_f16")
        L.pllm_attention_f16_noalloc(got.ptr, Q.ptr, K.ptr, V.ptr, pos, nh, nkv, hs, 0, nh)
        check("pllm_attention_f16_noalloc")
        a, b = want.download(np.float32), got.download(np.float32)
        np.testing.assert_allclose(b, a, rtol=1e-4, atol=2e-5, err_msg=f"call {call}")
        ref, _ = O.attention(q, kc, vc, pos, nh, nkv, hs, half=True)
        np.testing.assert_allclose(b, ref, rtol=1e-4, atol=2e-5, err_msg=f"call {call} against the oracle")


def test_noalloc_attention_refuses_what_does_not_fit():
    out = Buffer(64)
    pos = 40000  # 32 heads of 128: the 4 MiB array holds the partials of 31,744 positions at most
    L.pllm_attention_f16_noalloc(out.ptr, out.ptr, out.ptr, out.ptr, pos, 32, 8, 128, 0, 32)
    with pytest.raises(PllmError, match="static scratch"):
        check("refused")
