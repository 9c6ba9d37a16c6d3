"""ctypes binding of libnpu_b200.so (the C ABI declared in include/npu_b200.h).

The library is loaded from ``llm_compiler_3_b200/lib/`` only.  There is no
fallback: if the shared library is missing or fails to load, every entry point
raises ``NativeUnavailable``, so a GPU run can never silently compute on the
CPU or through another library.
"""
from __future__ import annotations

import ctypes
from ctypes import (POINTER, c_char_p, c_float, c_int, c_int32, c_int64, c_size_t, c_uint32,
                    c_uint64, c_void_p)
from pathlib import Path

LIBRARY = Path(__file__).resolve().parent / "lib" / "libnpu_b200.so"
HEADER = Path(__file__).resolve().parent.parent / "include" / "npu_b200.h"

OK = 0
ERRORS = {
    -1: "NPU_B200_E_INVALID",
    -2: "NPU_B200_E_CUDA",
    -3: "NPU_B200_E_NCCL",
    -4: "NPU_B200_E_UNSUPPORTED",
    -5: "NPU_B200_E_NOMEM",
    -6: "NPU_B200_E_PLAN",
    -7: "NPU_B200_E_DEVICE",
    -8: "NPU_B200_E_STATE",
}


class NativeUnavailable(RuntimeError):
    """libnpu_b200.so could not be loaded; build it with llm_compiler_3_b200.build."""


class NpuError(RuntimeError):
    """A C-ABI call returned a negative status."""

    def __init__(self, code: int, message: str):
        super().__init__(f"{ERRORS.get(code, code)}: {message}")
        self.code = code


# (name, restype, argtypes)
_SIGNATURES = [
    ("npu_b200_abi_version", c_int, []),
    ("npu_b200_last_error", c_char_p, []),
    ("npu_b200_device_status", c_int, [POINTER(c_uint32)]),
    ("npu_b200_flash_decode_workspace_size", c_size_t, [c_int, c_int, c_int, c_int, c_int]),
    ("npu_b200_flash_decode", c_int,
     [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
      c_float, c_int, c_void_p, c_size_t, c_void_p]),
    ("npu_b200_flash_decode_noalloc", c_int,
     [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
      c_float, c_int, c_void_p]),
    ("npu_b200_prefill_attention", c_int,
     [c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
      c_int, c_int, c_float, c_int, c_void_p]),
    ("npu_b200_linear_workspace_size", c_size_t, [c_int, c_int, c_int]),
    ("npu_b200_linear", c_int,
     [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_size_t,
      c_void_p]),
    ("npu_b200_packed_weight_bytes", c_size_t, [c_int, c_int]),
    ("npu_b200_pack_weight", c_int, [c_void_p, c_int, c_int, c_void_p, c_void_p]),
    ("npu_b200_pack_weight_rows", c_int,
     [c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_int, c_void_p]),
    ("npu_b200_projection", c_int,
     [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_size_t, c_void_p]),
    ("npu_b200_nccl_unique_id", c_int, [c_void_p]),
    ("npu_b200_create", c_int, [c_int, c_int, c_int, c_void_p, POINTER(c_void_p)]),
    ("npu_b200_destroy", c_int, [c_void_p]),
    ("npu_b200_graph_check", c_int, [c_char_p, POINTER(c_int64), c_int]),
    ("npu_b200_shard_info", c_int, [c_char_p, c_int, c_int, POINTER(c_int64), c_int]),
    ("npu_b200_load_graph", c_int, [c_void_p, c_char_p]),
    ("npu_b200_run_graph", c_int, [c_void_p, POINTER(c_void_p), POINTER(c_void_p), c_void_p]),
    ("npu_b200_load_plan", c_int, [c_void_p, c_char_p]),
    ("npu_b200_plan_info", c_int, [c_void_p, POINTER(c_int64), c_int]),
    ("npu_b200_plan_check", c_int, [c_char_p, POINTER(c_int64), c_int]),
    ("npu_b200_set_weight", c_int, [c_void_p, c_char_p, c_void_p, c_size_t]),
    ("npu_b200_load_capture", c_int, [c_void_p, c_char_p]),
    ("npu_b200_save_image", c_int, [c_void_p, c_char_p]),
    ("npu_b200_load_image", c_int, [c_void_p, c_char_p]),
    ("npu_b200_kv_cache", c_int, [c_void_p, c_int, POINTER(c_void_p), POINTER(c_void_p)]),
    ("npu_b200_decode_step", c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    ("npu_b200_decode_step_device", c_int,
     [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    ("npu_b200_forward_hidden", c_int, [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
    ("npu_b200_forward_hidden_device", c_int,
     [c_void_p, c_void_p, c_void_p, c_int, c_void_p, c_void_p]),
]

LINEAR_RELU = 1
LINEAR_OUT_F32 = 2
LINEAR_PACKED_W = 4

EPI_STORE, EPI_RESID, EPI_SWIGLU, EPI_QKV, EPI_ARGMAX = range(5)
PACK_IDENTITY, PACK_INTERLEAVE, PACK_HEAD_PAIRS = range(3)


class Epilogue(ctypes.Structure):
    """Mirror of npu_b200_epilogue (include/npu_b200.h)."""

    _fields_ = [
        ("kind", c_int), ("ssq_in", c_void_p), ("ssq_parts", c_int), ("ssq_ld", c_int),
        ("hidden", c_int), ("ssq_eps", c_float), ("out", c_void_p), ("ld_out", c_int),
        ("out_f32", c_int), ("relu", c_int), ("bias", c_void_p), ("resid", c_void_p),
        ("ld_resid", c_int), ("norm_w", c_void_p), ("xw", c_void_p), ("ld_xw", c_int),
        ("ssq_out", c_void_p), ("ssq_out_ld", c_int), ("q_heads", c_int), ("kv_heads", c_int),
        ("positions", c_void_p), ("inv_freq", c_void_p), ("k_cache", c_void_p),
        ("v_cache", c_void_p), ("max_seq", c_int), ("q_norm_w", c_void_p), ("k_norm_w", c_void_p),
        ("qk_eps", c_float), ("am_val", c_void_p), ("am_idx", c_void_p), ("am_ld", c_int),
        ("ssq_out_rows", c_int), ("am_rows", c_int),
    ]

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library, with argument types declared; raises if unavailable."""
    global _lib
    if _lib is None:
        if not LIBRARY.exists():
            raise NativeUnavailable(
                f"{LIBRARY} is missing: run `python -m llm_compiler_3_b200.build`")
        try:
            handle = ctypes.CDLL(str(LIBRARY), mode=ctypes.RTLD_GLOBAL)
        except OSError as exc:  # pragma: no cover - depends on the machine
            raise NativeUnavailable(f"cannot load {LIBRARY}: {exc}") from exc
        for name, restype, argtypes in _SIGNATURES:
            fn = getattr(handle, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = handle
    return _lib


def exported_symbols() -> list[str]:
    """Every C-ABI function this binding declares."""
    return [name for name, _, _ in _SIGNATURES]


def check(rc: int) -> None:
    """Raise NpuError for a negative status, with the library's message."""
    if rc != OK:
        message = lib().npu_b200_last_error() or b""
        raise NpuError(rc, message.decode(errors="replace"))


def device_status() -> int:
    """Synchronize and return (and clear) the device error bits; raise if any."""
    bits = c_uint32(0)
    check(lib().npu_b200_device_status(ctypes.byref(bits)))
    return bits.value


__all__ = ["lib", "check", "device_status", "exported_symbols", "NativeUnavailable", "NpuError",
           "LIBRARY", "HEADER", "c_void_p", "c_int", "c_int32", "c_float", "c_size_t", "c_uint64"]
