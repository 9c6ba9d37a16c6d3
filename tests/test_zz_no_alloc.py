"""The allocation-free flash-decoding entry point (npu_b200_flash_decode_noalloc).

It exists for callers that may not allocate device memory at call time (a host
application owning all HBM through its own pool, a latency-critical path that
cannot afford cudaMalloc's device synchronization).  It must give what the
allocating entry point gives, call after call, from its static scratch array.
This file is collected last so a failure here never hides an earlier test."""
import ctypes

import pytest
import torch

import oracle
from conftest import seeded

pytestmark = pytest.mark.gpu

ATOL = 2e-2


def _noalloc(q, k, v, lens, num_splits=0):
    from llm_compiler_3_b200 import _native
    out = torch.empty_like(q)
    batch, q_heads, dim = q.shape
    _, kv_heads, max_seq, _ = k.shape
    rc = _native.lib().npu_b200_flash_decode_noalloc(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
        ctypes.c_void_p(v.data_ptr()), ctypes.c_void_p(lens.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), batch, q_heads, kv_heads, dim, max_seq,
        ctypes.c_float(dim ** -0.5), num_splits,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _native.check(rc)
    return out


@pytest.mark.parametrize("batch,seq,lens,splits", [
    (1, 4096, [4096], 0),              # the flash-decoding config: split count chosen by the library
    (4, 4096, [4096, 3000, 1, 2048], 0),  # chosen splits merged through the static scratch
    (4, 1000, [1000, 1, 517, 0], 5),   # ragged lengths, an empty sequence
])
def test_noalloc_matches_allocating_entry(cuda, batch, seq, lens, splits):
    """Two calls in a row: each must match the allocating entry point and the
    CPU oracle within the flash-decoding tolerance."""
    from llm_compiler_3_b200 import _native, ops
    dev = torch.device("cuda", 0)
    q_h = seeded((batch, 32, 128), 61)
    k_h = seeded((batch, 8, seq, 128), 62)
    v_h = seeded((batch, 8, seq, 128), 63)
    q, k, v = q_h.to(dev), k_h.to(dev), v_h.to(dev)
    lens_d = torch.tensor(lens, dtype=torch.int32, device=dev)
    expected = ops.flash_decode(q, k, v, lens_d, num_splits=splits).float().cpu()
    ref = oracle.attention_decode(q_h, k_h, v_h, lens, 128 ** -0.5)
    for _ in range(2):  # the second call sees the scratch the first one left
        got = _noalloc(q, k, v, lens_d, splits).float().cpu()
        assert float((got - expected).abs().max()) <= ATOL
        assert oracle.cosine(got, expected) >= 0.9999
        assert float((got - ref).abs().max()) <= ATOL
        assert oracle.cosine(got, ref) >= 0.9999
    assert _native.device_status() == 0


def test_noalloc_rejects_oversized_scratch(cuda):
    from llm_compiler_3_b200 import _native
    dev = torch.device("cuda", 0)
    q = torch.zeros(64, 32, 128, dtype=torch.float16, device=dev)
    k = torch.zeros(64, 8, 4096, 128, dtype=torch.float16, device=dev)
    lens = torch.full((64,), 4096, dtype=torch.int32, device=dev)
    with pytest.raises(_native.NpuError, match="static scratch"):
        _noalloc(q, k, k, lens, num_splits=64)
