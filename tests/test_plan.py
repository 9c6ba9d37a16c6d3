"""Plan files and host-side checks of the runtime boundary (CPU)."""
import ctypes
import hashlib

import pytest

from llm_compiler_3_b200 import _native
from llm_compiler_3_b200.plan import DecodePlan, llama3_8b, qwen3_8b, rope_inv_freq


def _check(path):
    out = (ctypes.c_int64 * 12)()
    rc = _native.lib().npu_b200_plan_check(str(path).encode(), out, 12)
    return rc, list(out)


def _fnv1a(text: str) -> int:
    h = 1469598103934665603
    for c in text.encode():
        h ^= c
        h = (h * 1099511628211) % (1 << 64)
    return h & 0x7FFFFFFFFFFFFFFF


def test_llama_plan_parses(tmp_path):
    plan = llama3_8b()
    path = plan.write(tmp_path / "plan.txt")
    rc, info = _check(path)
    assert rc == 0, _native.lib().npu_b200_last_error()
    assert info[:6] == [32, 4096, 32, 8, 14336, 128256]
    assert info[7:10] == [64, 4096, 128]
    assert info[10] == _fnv1a(path.read_text())


def test_qwen3_plan_parses(tmp_path):
    rc, info = _check(qwen3_8b().write(tmp_path / "p.txt"))
    assert rc == 0 and info[4] == 12288


def test_inv_freq_round_trips_exactly(tmp_path):
    plan = llama3_8b()
    text = plan.text()
    line = next(l for l in text.splitlines() if l.startswith("inv_freq"))
    values = [float.fromhex(v) for v in line.split("=")[1].split()]
    assert values == rope_inv_freq(500000.0, 128)


@pytest.mark.parametrize("edit,message", [
    (("stage = cuda-plan", "stage = target"), "stage"),
    (("schema = 1", "schema = 2"), "schema"),
    (("head_dim = 128", "head_dim = 64"), "head_dim"),
    (("arch = llama", "arch = gpt2"), "arch"),
    (("max_seq = 4096", "max_seq = 4096\nmax_seq = 8"), "duplicate"),
    (("vocab = 128256", "vocab = 128256\nbogus = 1"), "unknown key"),
    (("ffn = 14336", "ffn = 100"), "inconsistent"),
    (("qk_norm = 0", "qk_norm = 1"), "qk_norm"),
    (("hidden = 4096", "hidden = many"), "integer"),
])
def test_plan_rejections(tmp_path, edit, message):
    """Fail-closed like the reference's stage / schema / fingerprint checks
    (tools/npu-compile/npu-compile.cpp:226-316) and strict TOML
    (lib/Target/HardwareConfig.cpp:18-71)."""
    text = llama3_8b().text().replace(*edit)
    path = tmp_path / "bad.txt"
    path.write_text(text)
    rc, _ = _check(path)
    assert rc == -6 or rc == -4
    assert message in _native.lib().npu_b200_last_error().decode()


def test_missing_plan_file(tmp_path):
    rc, _ = _check(tmp_path / "absent.txt")
    assert rc == -6


def test_tp_context_without_nccl_fails_cleanly(monkeypatch):
    """NCCL that cannot be loaded is reported as NPU_B200_E_NCCL before any CUDA
    call (host-side fault injection: a bad library path)."""
    monkeypatch.setenv("NPU_B200_NCCL_LIBRARY", "/nonexistent/libnccl.so.2")
    ctx = ctypes.c_void_p()
    rc = _native.lib().npu_b200_create(0, 0, 2, ctypes.create_string_buffer(128),
                                       ctypes.byref(ctx))
    assert rc == -3 and not ctx.value
    assert b"NCCL" in _native.lib().npu_b200_last_error()


def test_tp_arguments_validated():
    ctx = ctypes.c_void_p()
    assert _native.lib().npu_b200_create(0, 2, 2, None, ctypes.byref(ctx)) == -1
    assert _native.lib().npu_b200_create(0, 0, 2, None, ctypes.byref(ctx)) == -1
