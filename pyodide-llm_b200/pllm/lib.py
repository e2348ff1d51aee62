"""libpllm.so through ctypes: the registry's kernels with the reference's names and argument order
(src/python/engine/kernels.py:31-66 binds the reference's WASM kernels the same way: an address a c_void_p there, a
uint64 device pointer here; i32 and f32 as they are).

There is no fallback: if the library is missing or cannot load, importing this module raises. Build it with
`make -C pyodide-llm_b200` (nvcc, sm_100a) or __graft_entry__.build().
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpllm.so")

U64, I64, I32, F32, P = ctypes.c_uint64, ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_void_p

# name: (argument types, return type). The registry kernels first (their types: src/runtime/jobs.ts:82-142).
SIGNATURES = {
    # ---- the registry (include/pllm.h)
    "rmsnorm": ([U64, U64, U64, I32, F32], None),
    "swiglu": ([U64, U64, U64, I32], None),
    "add_inplace": ([U64, U64, I32], None),
    "rope": ([U64, U64, U64, I32, I32, I32], None),
    "attention": ([U64, U64, U64, U64, U64, I32, I32, I32, I32, I32, I32], None),
    "attention_f16": ([U64, U64, U64, U64, U64, I32, I32, I32, I32, I32, I32], None),
    "attention_capped": ([U64, U64, U64, U64, U64, I32, I32, I32, I32, I32, I32, F32], None),
    "attention_f16_capped": ([U64, U64, U64, U64, U64, I32, I32, I32, I32, I32, I32, F32], None),
    "to_f16": ([U64, U64, I32], I32),
    "from_f16": ([U64, U64, I32], None),
    "finite_f16": ([U64, I32], I32),
    "matmul_f32": ([U64, U64, U64, I32, I32, I32], None),
    "six_sums": ([U64, U64, I32], None),
    "int8_sums": ([U64, U64, I32], None),
    "matmul_q8": ([U64, U64, U64, U64, U64, I32, I32, I32], None),
    "interleave": ([U64, U64, I32], None),
    "matmul_t2": ([U64, U64, U64, U64, U64, I32, I32, I32, I32], None),
    "matmul_q6": ([U64, U64, U64, U64, U64, I32, I32, I32], None),
    "quantize_x": ([U64, U64, U64, I32, I32], None),
    "gate": ([U64, U64, U64, I32], None),
    "convolve": ([U64, U64, U64, I32, I32], None),
    "short_conv": ([U64, U64, U64, U64, I32, I32], None),
    "delta_rule": ([U64, U64, U64, U64, U64, I32, I32, I32, I32, I32, I32], None),
    "matmul_q8r": ([U64, U64, U64, U64, U64, U64, I32, I32, I32], None),
    "matmul_q8r_tile": ([U64, U64, U64, U64, U64, U64, I32, I32, I32, I32, I32, I32], None),
    "matmul_q6r": ([U64, U64, U64, U64, U64, U64, I32, I32, I32], None),
    "matmul_t2r": ([U64, U64, U64, U64, U64, I32, I32, I32, I32], None),
    "matmul_t2r_tile": ([U64, U64, U64, U64, U64, I32, I32, I32, I32, I32, I32, I32], None),
    "matmul_b1": ([U64, U64, U64, U64, U64, I32, I32, I32, I32], None),
    "matmul_b1r": ([U64, U64, U64, U64, U64, I32, I32, I32, I32], None),
    "matmul_b1r_tile": ([U64, U64, U64, U64, U64, I32, I32, I32, I32, I32, I32, I32], None),
    # ---- device, memory, streams, graphs, errors
    "pllm_init": ([I32], I32),
    "pllm_last_error": ([ctypes.c_char_p, I32], I32),
    "pllm_clear_error": ([], None),
    "pllm_num_sms_of_device": ([], I32),
    "pllm_alloc": ([U64], U64),
    "pllm_free": ([U64], None),
    "pllm_alloc_host": ([U64], U64),
    "pllm_free_host": ([U64], None),
    "pllm_h2d": ([U64, P, U64], None),
    "pllm_d2h": ([P, U64, U64], None),
    "pllm_d2d": ([U64, U64, U64], None),
    "pllm_memset": ([U64, I32, U64], None),
    "pllm_stream_create": ([], U64),
    "pllm_stream_destroy": ([U64], None),
    "pllm_set_stream": ([U64], None),
    "pllm_get_stream": ([], U64),
    "pllm_sync": ([], I32),
    "pllm_device_sync": ([], I32),
    "pllm_graph_begin": ([], I32),
    "pllm_graph_end": ([], U64),
    "pllm_graph_launch": ([U64], I32),
    "pllm_graph_destroy": ([U64], None),
    "pllm_event_create": ([], U64),
    "pllm_event_record": ([U64], None),
    "pllm_event_ms": ([U64, U64], F32),
    "pllm_event_destroy": ([U64], None),
    "pllm_version": ([], ctypes.c_char_p),
    # ---- the device engine's additions
    "pllm_group_sums": ([U64, U64, U64, U64, I32, I32, I32, I32, I32], None),
    "pllm_quantize_tokens": ([U64, U64, U64, I32, I32, I32], None),
    "pllm_to_f16_async": ([U64, U64, I32, U64], None),
    "pllm_rmsnorm_rows": ([U64, U64, U64, I32, F32, I32, I64], None),
    "pllm_embed_q8": ([U64, U64, U64, U64, I32, I32, I32, I64], None),
    "pllm_gemv": ([U64, I64, U64, U64, I64, I64, U64, I64, U64, F32, I32, U64, U64, I32, I32, I32, I32, I32, I32, I32,
                   I64, I32], None),
    "pllm_qk_rope_cache": ([U64, U64, U64, U64, U64, U64, U64, U64, I32, U64, U64, I32, I32, I32, I32, F32, I32, U64,
                            I32], None),
    "pllm_attention_scratch_bytes": ([I32, I32, I32, I32], U64),
    "pllm_attention_f16_noalloc": ([U64, U64, U64, U64, I32, I32, I32, I32, I32, I32], None),
    "pllm_attention_step": ([U64, U64, U64, U64, U64, U64, I32, I32, I32, I32, I32, F32, I32, U64, U64, U64, U64, I32,
                             F32, U64, I32], None),
    "pllm_attention_dev": ([U64, U64, U64, U64, U64, U64, I32, I32, I32, I32, I32, F32, I32, I32], None),
    "pllm_attention_step_batch": ([U64, I64, U64, I64, U64, U64, I64, U64, U64, I32, I32, I32, I32, I32, F32, I32, U64,
                                   U64, U64, U64, I32, F32, U64, I32], None),
    "pllm_device_status": ([], I32),
    "pllm_set_gemv_mode": ([I32], I32),
    "pllm_set_stage_budget": ([I32], I32),
    "pllm_set_attention_mode": ([I32], I32),
    "pllm_synth_f32": ([U64, I64, U64, F32, F32], None),
    "pllm_synth_q8": ([U64, U64, I64, I32, U64, F32], None),
    "pllm_synth_q8_block": ([U64, U64, I64, I32, U64, F32, I64, I64, I64], None),
    "pllm_gemm_q8": ([U64, I64, U64, U64, U64, U64, I32, I32, I32, I64, I32, I64], None),
    "pllm_norm_quantize_rows": ([U64, U64, U64, I64, U64, F32, I32, I32, I32], None),
    "pllm_transpose_scales": ([U64, U64, I64, I32], None),
    "pllm_qk_rope_cache_rows": ([U64, I64, U64, U64, U64, U64, I32, I32, U64, U64, I32, I32, I32, I32, F32, I32, U64],
                                None),
    "pllm_attention_prefill": ([U64, I64, U64, I64, U64, U64, I32, I32, I32, I32, I32], None),
    "pllm_tp_open": ([I32, I32, I32, I32], U64),
    "pllm_tp_handle": ([U64, P], I32),
    "pllm_tp_connect": ([U64, P], I32),
    "pllm_tp_close": ([U64], None),
    "pllm_tp_step": ([U64], None),
    "argmax": ([U64, I32], I32),
    "penalize": ([U64, U64, I32, F32, F32], None),
    "pllm_argmax_dev": ([U64, U64, I32, U64], None),
    "pllm_argmax_key_dev": ([U64, U64, I32, I64, U64], None),
    "pllm_key_token_dev": ([U64, U64], None),
    "sb_tables": ([U64, U64], I32),
    "sums_x": ([U64, U64, I32], None),
    "matmul_sb": ([U64, U64, U64, U64, U64, I32, I32, I32, I32], None),
    "matmul_sbr": ([U64, U64, U64, U64, U64, I32, I32, I32, I32], None),
    "matmul_sbr_tile": ([U64, U64, U64, U64, U64, I32, I32, I32, I32, I32, I32, I32], None),
    "matmul_sbw_tile": ([U64, U64, U64, U64, U64, I32, I32, I32, I32, I32, I32, I32, U64], None),
    "signed_dots": ([U64, U64, U64], None),
    "sb_row": ([U64, U64, U64, I32, I32], None),
    "sample": ([U64, I32, F32, F32, ctypes.c_double, U64, U64, I32, F32], I32),
    "pllm_sample_dev": ([U64, U64, I32, F32, F32, U64, U64, U64, I32, F32], None),
    "pllm_gemv_tp": ([U64, U64, U64, U64, F32, I32, U64, U64, I32, I32, I32, I32, I64, I32, U64, I32], None),
    "pllm_synth_t2": ([U64, U64, I64, I32, U64, F32, F32], None),
    "pllm_delta_rule_block": ([U64, I64, U64, U64, U64, I64, U64, I64, I32, I32, I32, I32, I32, I32, I32], None),
    "pllm_shift_rows": ([U64, I32, I32], None),
    "pllm_conv_step": ([U64, I64, U64, U64, I64, U64, I64, I32, I32, U64, I32], None),
    "pllm_delta_gates": ([U64, U64, U64, I32], None),
    "pllm_scale_rows": ([U64, I32, I32, I64, U64], None),
    "pllm_softcap": ([U64, I32, F32], None),
    "pllm_exact_prepare": ([U64, U64, U64, U64, U64, I32, F32, I32, I32], None),
    "pllm_exact_product": ([U64, U64, U64, U64, U64, U64, I32, I32, I32], None),
    "pllm_exact_qk_rope_cache": ([U64, U64, U64, U64, U64, U64, I32, U64, U64, I32, I32, I32, F32, I32, U64], None),
    "pllm_exact_attention": ([U64, U64, U64, U64, U64, U64, I32, I32, I32, I32, I32, I32, F32], None),
}

# the registry's names: what a drop-in for the reference's kernel modules exports (tests check each is there)
REGISTRY = [name for name in SIGNATURES if not name.startswith("pllm_")]


class PllmError(RuntimeError):
    pass


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"libpllm.so is not built ({LIB_PATH}): run `make -C pyodide-llm_b200`; there is no CPU fallback")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(lib, name)  # AttributeError: a symbol of include/pllm.h the library does not export
        fn.argtypes, fn.restype = args, res
    return lib


L = _load()


def last_error():
    buf = ctypes.create_string_buffer(512)
    code = L.pllm_last_error(buf, 512)
    return code, buf.value.decode(errors="replace")


def check(what=""):
    """Raise the sticky error, if any, and clear it."""
    code, msg = last_error()
    if code:
        L.pllm_clear_error()
        raise PllmError(f"{what + ': ' if what else ''}{msg} (code {code})")
