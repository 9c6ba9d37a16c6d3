"""CPU checks of the C-ABI boundary: the library loads without a GPU and exports
exactly what include/npu_b200.h declares; argument errors come back as status
codes with a message, never as a crash."""
import ctypes
import re
import subprocess

import pytest

from llm_compiler_3_b200 import _native


def _declared():
    text = _native.HEADER.read_text()
    return sorted(set(re.findall(r"NPU_B200_API\s+[\w\s\*]+?\b(npu_b200_\w+)\s*\(", text)))


def test_header_declares_entry_points():
    names = _declared()
    assert "npu_b200_flash_decode" in names and "npu_b200_last_error" in names


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in npu_b200.h but not exported"
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIBRARY)],
                         capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r"\bT (npu_b200_\w+)", out))
    assert exported == set(_declared()), f"exports differ from header: {exported ^ set(_declared())}"


def test_binding_covers_header():
    assert set(_native.exported_symbols()) == set(_declared())


def test_abi_version_and_errors_without_gpu():
    lib = _native.lib()
    assert lib.npu_b200_abi_version() == 1
    # Invalid arguments are rejected on the host before any CUDA call.
    rc = lib.npu_b200_flash_decode(None, None, None, None, None, 1, 32, 8, 128, 4096,
                                   ctypes.c_float(0.088), 0, None, 0, None)
    assert rc == -1
    assert b"null" in lib.npu_b200_last_error()
    with pytest.raises(_native.NpuError, match="NPU_B200_E_INVALID"):
        _native.check(rc)


def test_flash_decode_workspace_sizes():
    lib = _native.lib()
    # One split needs no workspace; more splits need counters + partials.
    assert lib.npu_b200_flash_decode_workspace_size(64, 8, 128, 4096, 1) == 0
    size = lib.npu_b200_flash_decode_workspace_size(1, 8, 128, 4096, 16)
    assert size == 16384 * 4 + 8 * 16 * (8 * 128 + 16) * 4
    assert lib.npu_b200_flash_decode_workspace_size(1, 8, 128, 4096, 0) > 0
