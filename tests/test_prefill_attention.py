"""Multi-query (prefill) attention: the oracle pinned to torch's SDPA -- the
reference's own golden for npu.attention (test/Integration/attention.py:93) --
on the reference's four SDPA cases, and the tcgen05 kernel against the oracle.

Tolerances: FP16 outputs within max-abs 2e-2 of the FP32 oracle, the
reference's SDPA bound (test/Integration/attention.py:99-104,170), and cosine
>= 0.9999."""
import pytest
import torch

import oracle
from conftest import seeded

ATOL = 2e-2
COS = 0.9999

# name, query heads, key/value heads, queries, keys, head size, causal
# (the reference's cases, test/Integration/attention.py:28-33)
REFERENCE_CASES = [
    ("mha", 2, 2, 64, 128, 32, False),
    ("gqa", 8, 2, 64, 256, 64, False),
    ("causal", 4, 1, 128, 128, 64, True),
    ("gqa_causal_d128", 8, 2, 256, 256, 128, True),
]


def _inputs(heads, kv_heads, queries, keys, dim, batch=1, capacity=None, seed=1):
    capacity = capacity or keys
    q = seeded((batch, heads, queries, dim), seed, 0.5)
    k = seeded((batch, kv_heads, capacity, dim), seed + 1, 0.5)
    v = seeded((batch, kv_heads, capacity, dim), seed + 2, 0.5)
    return q, k, v


@pytest.mark.parametrize("case", REFERENCE_CASES, ids=[c[0] for c in REFERENCE_CASES])
def test_oracle_matches_sdpa(case):
    _, heads, kv_heads, queries, keys, dim, causal = case
    q, k, v = _inputs(heads, kv_heads, queries, keys, dim)
    want = torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.float(), v.float(), is_causal=causal, enable_gqa=heads != kv_heads)
    got = oracle.attention_prefill(q, k, v, keys, dim ** -0.5, causal)
    torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-5)


def test_oracle_cache_positions_and_empty_rows():
    """q_start shifts the causal diagonal (a prompt appended to a cached prefix);
    a row that sees no key (no keys at all) is zero."""
    q, k, v = _inputs(4, 2, 6, 20, 32, batch=2, capacity=24)
    got = oracle.attention_prefill(q, k, v, 20, 0.3, True, q_start=[10, 0])
    for b, start in enumerate((10, 0)):
        for i in range(6):
            n = min(start + i + 1, 20)
            want = oracle.attention_decode(q[b:b + 1, :, i], k[b:b + 1], v[b:b + 1], [n], 0.3)
            torch.testing.assert_close(got[b, :, i], want[0], atol=1e-6, rtol=0)
    assert torch.count_nonzero(oracle.attention_prefill(q, k, v, 0, 0.3, False)) == 0


def _run(q, k, v, keys, causal, q_start=None, scale=None):
    from llm_compiler_3_b200 import _native, ops
    dev = torch.device("cuda", 0)
    qs = None if q_start is None else torch.tensor(q_start, dtype=torch.int32, device=dev)
    out = ops.prefill_attention(q.to(dev), k.to(dev), v.to(dev), keys=keys, q_start=qs,
                                causal=causal, scale=scale)
    torch.cuda.synchronize()
    assert _native.device_status() == 0
    return out.float().cpu()


def _check(got, want):
    err = float((got - want).abs().max())
    assert err <= ATOL, f"max-abs {err}"
    assert oracle.cosine(got, want) >= COS


@pytest.mark.gpu
@pytest.mark.parametrize("case", REFERENCE_CASES, ids=[c[0] for c in REFERENCE_CASES])
def test_reference_cases(cuda, case):
    _, heads, kv_heads, queries, keys, dim, causal = case
    q, k, v = _inputs(heads, kv_heads, queries, keys, dim)
    _check(_run(q, k, v, keys, causal), oracle.attention_prefill(q, k, v, keys, dim ** -0.5, causal))


@pytest.mark.gpu
@pytest.mark.parametrize("dim", [32, 64, 128])
def test_prompt_after_cached_prefix(cuda, dim):
    """Ragged prompt (37 queries, not a multiple of the 64-row block) appended at
    different cache positions; the cache holds garbage past `keys`, which must not
    leak in."""
    q, k, v = _inputs(8, 2, 37, 150, dim, batch=3, capacity=160, seed=7)
    k[:, :, 150:] = float("nan")
    v[:, :, 150:] = float("nan")
    starts = [100, 0, 113]
    got = _run(q, k, v, 150, True, q_start=starts)
    _check(got, oracle.attention_prefill(q, k, v, 150, dim ** -0.5, True, q_start=starts))


@pytest.mark.gpu
def test_small_query_blocks_and_wide_groups(cuda):
    """5 queries per head, group 8: eight heads share one CTA's 128 rows."""
    q, k, v = _inputs(16, 2, 5, 70, 64, batch=2, capacity=80, seed=11)
    got = _run(q, k, v, 70, True, q_start=[60, 0])
    _check(got, oracle.attention_prefill(q, k, v, 70, 64 ** -0.5, True, q_start=[60, 0]))
    got = _run(q, k, v, 70, False, scale=0.05)
    _check(got, oracle.attention_prefill(q, k, v, 70, 0.05, False))


@pytest.mark.gpu
@pytest.mark.parametrize("scale", [128 ** -0.5, -0.05])
def test_head128_paths(cuda, scale):
    """Head size 128: a positive scale runs the two-tile pipelined kernel, a
    negative one the single-tile kernel; both against the oracle, including a
    key count that is not a multiple of the 64-key tile."""
    q, k, v = _inputs(8, 2, 300, 333, 128, batch=2, capacity=352, seed=31)
    for causal in (False, True):
        got = _run(q, k, v, 333, causal, q_start=[33, 0], scale=scale)
        _check(got, oracle.attention_prefill(q, k, v, 333, scale, causal, q_start=[33, 0]))


@pytest.mark.gpu
def test_no_keys_and_rejections(cuda):
    from llm_compiler_3_b200 import _native
    q, k, v = _inputs(2, 1, 16, 16, 32)
    assert torch.count_nonzero(_run(q, k, v, 0, False)) == 0
    q, k, v = _inputs(2, 1, 16, 16, 128)
    assert torch.count_nonzero(_run(q, k, v, 0, True)) == 0
    with pytest.raises(_native.NpuError, match="head_dim"):
        _run(seeded((1, 2, 4, 48), 1), seeded((1, 1, 8, 48), 2), seeded((1, 1, 8, 48), 3), 8, False)
    with pytest.raises(_native.NpuError, match="keys"):
        _run(q, k, v, 17, False)


@pytest.mark.gpu
def test_long_prompt_matches_decode_kernel(cuda):
    """A 1024-token causal prompt over a 4096-slot cache (prefix of 3000): the
    last query's row equals the flash-decoding kernel's output at that position."""
    from llm_compiler_3_b200 import ops
    q, k, v = _inputs(32, 8, 1024, 4024, 128, capacity=4096, seed=21)
    got = _run(q, k, v, 4024, True, q_start=[3000])
    want = oracle.attention_prefill(q[:, :, -64:], k, v, 4024, 128 ** -0.5, True, q_start=[3960])
    _check(got[:, :, -64:], want)
    dev = torch.device("cuda", 0)
    dec = ops.flash_decode(q[:, :, -1].contiguous().to(dev), k.to(dev), v.to(dev),
                           torch.tensor([4024], dtype=torch.int32, device=dev))
    _check(got[:, :, -1], dec.float().cpu())
