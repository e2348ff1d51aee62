"""pllm: takano32/pyodide-llm's quantized forward hot path on a B200 (sm_100a).

    lib      libpllm.so through ctypes: the registry's kernels (the reference's names and arguments) and the runtime
    device   device buffers over pllm_alloc / pllm_h2d / pllm_d2h
    jobs     the registry's job table and row runner (src/runtime/jobs.ts's WORK, PACKED, runner) over the C ABI
    forward  a decoder's forward pass on the device: one decode step a CUDA graph
"""
from . import lib  # noqa: F401  (raises if libpllm.so is missing: no CPU fallback)
