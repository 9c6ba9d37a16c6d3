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


@pytest.mark.parametrize("batch,kv_heads,keys,splits", [
    (1, 1, 4096, 32),   # a TP=8 rank's single KV head: 32 CTAs of 128 keys
    (1, 2, 4096, 32),
    (1, 8, 4096, 16),   # config 2: 128 CTAs, one per SM
    (16, 8, 8192, 8),   # config 4
    (64, 8, 4096, 2),   # the batch-64 step: 1024 CTAs in ~7 waves
    (1, 1, 300, 5),     # short cache: 64-key splits
])
def test_flash_decode_split_choice(batch, kv_heads, keys, splits):
    """The automatic split count (waves of one CTA per SM on 148 SMs, ~96 keys of
    start-up per CTA and ~6 keys of merge per split), read back from the
    workspace it needs: counters + units x splits x (8 x head_dim + 16) floats."""
    lib = _native.lib()
    lib.npu_b200_flash_decode_workspace_size.restype = ctypes.c_size_t
    size = lib.npu_b200_flash_decode_workspace_size(batch, kv_heads, 128, keys, 0)
    per_split = batch * kv_heads * (8 * 128 + 16) * 4
    assert (size - 16384 * 4) % per_split == 0
    assert (size - 16384 * 4) // per_split == splits
