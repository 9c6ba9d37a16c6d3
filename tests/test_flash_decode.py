"""Split-KV flash-decoding kernel against the CPU oracle (GPU tests).

Tolerances: FP16 outputs within max-abs 2e-2 and cosine >= 0.9999 of the
FP32-accumulated oracle (the FP16 parity bar); the reference's own SDPA bound
is 2e-2 max-abs (test/Integration/attention.py:99-104,170)."""
import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN, seeded

ATOL = 2e-2
COS = 0.9999

pytestmark = pytest.mark.gpu


def _run(q, k, v, lens, num_splits=0, scale=None):
    from llm_compiler_3_b200 import _native, ops
    dev = torch.device("cuda", 0)
    out = ops.flash_decode(q.to(dev), k.to(dev), v.to(dev),
                           torch.tensor(lens, dtype=torch.int32, device=dev),
                           scale=scale, num_splits=num_splits)
    assert _native.device_status() == 0
    return out.float().cpu()


def _check(got, ref):
    err = float((got - ref).abs().max())
    assert err <= ATOL, f"max-abs {err}"
    assert oracle.cosine(got, ref) >= COS


def test_config2_attention(cuda):
    """Flash-decoding config: 32 query / 8 KV heads, d 128, 4096 cached keys, batch 1."""
    q = seeded((1, 32, 128), 1)
    k = seeded((1, 8, 4096, 128), 2)
    v = seeded((1, 8, 4096, 128), 3)
    ref = oracle.attention_decode(q, k, v, [4096], 128 ** -0.5)
    for splits in (0, 1, 7, 16):
        _check(_run(q, k, v, [4096], splits), ref)


@pytest.mark.parametrize("group,dim", [(1, 64), (2, 128), (4, 64), (8, 128)])
def test_groups_and_head_dims(cuda, group, dim):
    kv = 2
    q = seeded((3, kv * group, dim), 10 + group)
    k = seeded((3, kv, 300, dim), 20 + group)
    v = seeded((3, kv, 300, dim), 30 + group)
    lens = [300, 1, 97]
    ref = oracle.attention_decode(q, k, v, lens, dim ** -0.5)
    _check(_run(q, k, v, lens), ref)
    _check(_run(q, k, v, lens, 3), ref)


def test_ragged_and_empty_sequences(cuda):
    """Ragged lengths (not multiples of the 32-key tile), a sequence with no keys
    (zeros by convention) and garbage past each length, which must not leak."""
    q = seeded((4, 8, 128), 5)
    k = seeded((4, 2, 200, 128), 6)
    v = seeded((4, 2, 200, 128), 7)
    lens = [200, 33, 0, 161]
    for b, n in enumerate(lens):   # plant non-finite values past the valid range
        k[b, :, n:] = float("nan")
        v[b, :, n:] = float("inf")
    ref = oracle.attention_decode(q, k, v, lens, 128 ** -0.5)
    for splits in (0, 1, 4):
        got = _run(q, k, v, lens, splits)
        assert torch.isfinite(got).all()
        assert float(got[2].abs().max()) == 0.0
        _check(got, ref)


@pytest.mark.parametrize("batch,kv,dim,lens", [(1, 1, 128, [4096]), (2, 2, 128, [700, 0]),
                                                (1, 4, 64, [333]), (4, 1, 128, [1, 31, 32, 1000]),
                                                (2, 2, 64, [4096, 2500]),
                                                (4, 1, 128, [3000, 0, 4096, 17])])
def test_small_batch_many_splits(cuda, batch, kv, dim, lens):
    """At most 4 (sequence, KV head) units with automatic splits: 16-64 splits
    per unit, merged by the unit's last CTA from one bulk copy of the unit's
    partials (ragged and empty sequences, garbage past each length)."""
    group = 4
    max_seq = max(max(lens), 64)
    q = seeded((batch, kv * group, dim), 40 + batch)
    k = seeded((batch, kv, max_seq, dim), 50 + kv)
    v = seeded((batch, kv, max_seq, dim), 60 + dim)
    for b, n in enumerate(lens):
        k[b, :, n:] = float("nan")
        v[b, :, n:] = float("inf")
    ref = oracle.attention_decode(q, k, v, lens, dim ** -0.5)
    got = _run(q, k, v, lens)
    assert torch.isfinite(got).all()
    for b, n in enumerate(lens):
        if n == 0:
            assert float(got[b].abs().max()) == 0.0
    _check(got, ref)


def test_sdpa_reference_cases(cuda):
    """The reference's SDPA cases with a supported head size, decode query row."""
    z = dict(np.load(GOLDEN / "sdpa_decode.npz"))
    for name in z["names"]:
        q = torch.from_numpy(z[f"{name}.q"])[None]
        if q.shape[-1] not in (64, 128):
            continue
        k = torch.from_numpy(z[f"{name}.k"])
        v = torch.from_numpy(z[f"{name}.v"])
        got = _run(q, k, v, [k.shape[2]])[0]
        expected = torch.from_numpy(z[f"{name}.expected"])
        assert float((got - expected).abs().max()) < 2e-2, name


def test_workspace_reuse_and_determinism(cuda):
    """The kernel leaves its split counters at zero: repeated calls on one
    workspace agree bit for bit."""
    q = seeded((2, 32, 128), 41)
    k = seeded((2, 8, 1024, 128), 42)
    v = seeded((2, 8, 1024, 128), 43)
    first = _run(q, k, v, [1024, 700], 5)
    for _ in range(3):
        assert torch.equal(_run(q, k, v, [1024, 700], 5), first)


def test_long_cache_batch64_shape(cuda):
    """Decode-stack attention shape: batch 64, 8 KV heads, 4096 keys, checked on a
    subset of sequences against the oracle (size-independent per sequence)."""
    from llm_compiler_3_b200 import ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(7)
    q = torch.randn(64, 32, 128, device=dev, generator=g).half()
    k = torch.randn(64, 8, 4096, 128, device=dev, generator=g).half()
    v = torch.randn(64, 8, 4096, 128, device=dev, generator=g).half()
    lens = torch.full((64,), 4096, dtype=torch.int32, device=dev)
    out = ops.flash_decode(q, k, v, lens).float().cpu()
    for b in (0, 17, 63):
        ref = oracle.attention_decode(q[b:b + 1].cpu(), k[b:b + 1].cpu(), v[b:b + 1].cpu(),
                                      [4096], 128 ** -0.5)
        _check(out[b:b + 1], ref)
