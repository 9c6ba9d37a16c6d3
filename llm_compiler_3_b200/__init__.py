"""llm_compiler_3_b200: B200-native (sm_100a) execution backend for the FP16
Llama/Qwen3 decode computation LLM_Compiler_3 lowers.

The product is ``libnpu_b200.so`` (C ABI in ``include/npu_b200.h``); this package
holds its build script, the ctypes binding and the host-side mirror of the
reference's interface for this path.
"""
from ._native import NativeUnavailable, NpuError  # noqa: F401

__version__ = "0.1.0"
