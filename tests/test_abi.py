"""The drop-in boundary without a GPU: libpllm.so loads, exports every function include/pllm.h declares (the
reference's registry names among them, src/runtime/jobs.ts:82-142), and the Python binding's table matches the
header. No kernel is called here."""
import ctypes
import os
import re
import subprocess

import pytest

from conftest import PKG, ROOT

LIB = os.path.join(PKG, "pllm", "libpllm.so")
HEADER = os.path.join(ROOT, "include", "pllm.h")


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(LIB):
        subprocess.run(["make", "-s", "-j8", "-C", PKG], check=True)
    return ctypes.CDLL(LIB)


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*([a-z_0-9]+)\s*\(", text, flags=re.M)


def test_header_declares_the_registry():
    names = set(declared())
    registry = {"quantize_x", "interleave", "int8_sums", "six_sums", "matmul_q8", "matmul_q8r", "matmul_q8r_tile",
                "matmul_q6", "matmul_q6r", "matmul_t2", "matmul_t2r", "matmul_t2r_tile", "matmul_b1", "matmul_b1r",
                "matmul_b1r_tile", "matmul_f32", "rope", "attention", "attention_f16", "attention_capped",
                "attention_f16_capped", "to_f16", "from_f16", "finite_f16", "rmsnorm", "swiglu", "add_inplace", "gate",
                "convolve", "short_conv", "delta_rule", "argmax", "penalize", "sample",
                "sb_tables", "sums_x", "matmul_sb", "matmul_sbr", "matmul_sbr_tile", "matmul_sbw_tile", "signed_dots",
                "sb_row"}
    assert registry <= names, registry - names


def test_library_exports_every_declared_symbol(lib):
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_exports_nothing_undeclared():
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    extra = {n for n in exported if not n.startswith("_")} - set(declared())
    assert not extra, f"exported but not in include/pllm.h: {sorted(extra)}"


def test_binding_table_matches_header(lib):
    import pllm.lib as pl
    assert set(pl.SIGNATURES) == set(declared()), set(pl.SIGNATURES) ^ set(declared())


def test_reference_signature_arity():
    """Each registry function takes the reference's argument count (jobs.ts:82-142's Arguments)."""
    import pllm.lib as pl
    arity = {"rmsnorm": 5, "swiglu": 4, "add_inplace": 3, "rope": 6, "attention": 11, "attention_f16": 11,
             "attention_capped": 12, "attention_f16_capped": 12, "to_f16": 3, "from_f16": 3, "finite_f16": 2,
             "matmul_f32": 6, "six_sums": 3, "int8_sums": 3, "matmul_q8": 8, "interleave": 3, "matmul_t2": 9,
             "matmul_q6": 8, "quantize_x": 5, "gate": 4, "convolve": 5, "short_conv": 6, "delta_rule": 11,
             "matmul_q8r": 9, "matmul_q8r_tile": 12, "matmul_q6r": 9, "matmul_t2r": 9, "matmul_t2r_tile": 12,
             "matmul_b1": 9, "matmul_b1r": 9, "matmul_b1r_tile": 12, "argmax": 2, "penalize": 5, "sample": 9,
             "sb_tables": 2, "sums_x": 3, "matmul_sb": 9, "matmul_sbr": 9, "matmul_sbr_tile": 12, "matmul_sbw_tile": 13,
             "signed_dots": 3, "sb_row": 5}
    for name, n in arity.items():
        assert len(pl.SIGNATURES[name][0]) == n, name

