"""Pin the CPU oracle (oracle/decode.py) before any kernel is checked against it.

Each expected value comes from the reference's own ground truth: transformers'
decoder layers, torch SDPA and the MLP module (fixtures in tests/golden/, made by
tests/golden/make_golden.py), plus the reference's known-answer matmul grid.
"""
import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN


def _load(name):
    return dict(np.load(GOLDEN / name))


@pytest.mark.parametrize("family", ["llama", "qwen3"])
def test_decoder_layer_matches_transformers(family):
    z = _load(f"{family}_layer_decode.npz")
    hidden, heads, kv, hd, ffn = (int(v) for v in z["shape"])
    shape = oracle.DecoderShape(hidden=hidden, heads=heads, kv_heads=kv, head_dim=hd, ffn=ffn,
                                eps=float(z["eps"]), rope_theta=float(z["rope_theta"]),
                                qk_norm=family == "qwen3")
    weights = {k[2:]: torch.from_numpy(v) for k, v in z.items() if k.startswith("w.")}
    k_cache = torch.from_numpy(z["k_cache"]).clone()
    v_cache = torch.from_numpy(z["v_cache"]).clone()
    positions = torch.from_numpy(z["positions"])
    y, k_new, v_new = oracle.decoder_layer_decode(weights, torch.from_numpy(z["x"]), positions,
                                                  k_cache, v_cache, shape)
    np.testing.assert_allclose(y.numpy(), z["expected_y"], atol=2e-5, rtol=1e-5)
    np.testing.assert_allclose(k_new.numpy(), z["expected_k_new"], atol=2e-5, rtol=1e-5)
    np.testing.assert_allclose(v_new.numpy(), z["expected_v_new"], atol=2e-5, rtol=1e-5)
    # KV indexing is exact: the new entry lands at `position`, nothing else moves.
    original_k = torch.from_numpy(z["k_cache"])
    for b, p in enumerate(positions.tolist()):
        assert torch.equal(k_cache[b, :, p], k_new[b].half())
        assert torch.equal(v_cache[b, :, p], v_new[b].half())
        mask = torch.ones(k_cache.shape[2], dtype=torch.bool)
        mask[p] = False
        assert torch.equal(k_cache[b][:, mask], original_k[b][:, mask])


def test_attention_matches_sdpa_cases():
    z = _load("sdpa_decode.npz")
    for name in z["names"]:
        q = torch.from_numpy(z[f"{name}.q"])[None]          # [1, Hq, D]
        k = torch.from_numpy(z[f"{name}.k"])                 # [1, Hkv, S, D]
        v = torch.from_numpy(z[f"{name}.v"])
        expected = z[f"{name}.expected"]
        got = oracle.attention_decode(q, k, v, [k.shape[2]], q.shape[-1] ** -0.5)[0]
        np.testing.assert_allclose(got.numpy(), expected, atol=1e-5, rtol=1e-5, err_msg=name)
        online = oracle.attention_online(q, k, v, [k.shape[2]], q.shape[-1] ** -0.5)[0]
        np.testing.assert_allclose(online.numpy(), expected, atol=1e-5, rtol=1e-5, err_msg=name)


def test_online_softmax_on_grid_values():
    """elementwise.py:142-146 style: blockwise online softmax equals dense attention
    on 1/16-grid operands (< 5e-3 is the reference's bound; the FP32 oracle is exact
    to rounding)."""
    q = oracle.grid_values(4 * 64, 7).reshape(1, 4, 64)
    k = oracle.grid_values(2 * 256 * 64, 3).reshape(1, 2, 256, 64)
    v = oracle.grid_values(2 * 256 * 64, 5).reshape(1, 2, 256, 64)
    dense = oracle.attention_decode(q, k, v, [256], 0.125)
    for block in (32, 64, 128):
        online = oracle.attention_online(q, k, v, [256], 0.125, block=block)
        assert float((online - dense).abs().max()) < 1e-5


def test_grid_matmul_is_exact():
    """test/Integration/matmul.py:18-26: |x| <= 1/2 on the 1/16 grid, K <= 512 keeps
    every FP32 partial sum exact, so the FP16 result is bit-exact."""
    a = oracle.grid_values(64 * 512, 7).reshape(64, 512)
    w = oracle.grid_values(96 * 512, 3).reshape(96, 512)
    got = oracle.linear(a, w).half()
    exact = (a.double() @ w.double().t()).half()
    assert torch.equal(got.view(torch.int16), exact.view(torch.int16))


def test_mlp_matches_module():
    z = _load("mlp.npz")
    t = {k: torch.from_numpy(v) for k, v in z.items()}
    got = oracle.mlp_forward(t["x"], t["w1"], t["b1"], t["w2"], t["b2"], round_hidden=False)
    np.testing.assert_allclose(got.numpy(), z["expected"], atol=1e-4, rtol=1e-4)


def test_rope_tables_match_transformers_default():
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    config = LlamaConfig(hidden_size=4096, num_attention_heads=32, head_dim=128,
                         rope_parameters={"rope_type": "default", "rope_theta": 500000.0})
    rotary = LlamaRotaryEmbedding(config)
    assert torch.equal(rotary.inv_freq, oracle.rope_inv_freq(500000.0, 128))
    pos = torch.tensor([[0, 1, 2047, 4095]])
    cos, sin = rotary(torch.zeros(1, 4, 8), pos)
    c2, s2 = oracle.rope_cos_sin(oracle.rope_inv_freq(500000.0, 128), pos[0])
    assert torch.equal(cos[0], c2) and torch.equal(sin[0], s2)


def test_argmax_ties_break_low():
    logits = torch.tensor([[1.0, 3.0, 3.0, 2.0], [5.0, 5.0, 5.0, 5.0]])
    assert oracle.greedy_argmax(logits).tolist() == [1, 0]
    assert torch.equal(oracle.greedy_argmax(logits), torch.argmax(logits, dim=-1))


@pytest.mark.parametrize("family", ["llama", "qwen3"])
def test_fp16_handoff_variant_stays_within_tolerance(family):
    """The variant that rounds where the kernels hand tensors over in FP16 is the
    same layer to within the FP16 tolerance, yet not the FP32 result itself."""
    z = _load(f"{family}_layer_decode.npz")
    hidden, heads, kv, hd, ffn = (int(v) for v in z["shape"])
    shape = oracle.DecoderShape(hidden=hidden, heads=heads, kv_heads=kv, head_dim=hd, ffn=ffn,
                                eps=float(z["eps"]), rope_theta=float(z["rope_theta"]),
                                qk_norm=family == "qwen3")
    weights = {k[2:]: torch.from_numpy(v) for k, v in z.items() if k.startswith("w.")}
    positions = torch.from_numpy(z["positions"])
    runs = [oracle.decoder_layer_decode(weights, torch.from_numpy(z["x"]), positions,
                                        torch.from_numpy(z["k_cache"]).clone(),
                                        torch.from_numpy(z["v_cache"]).clone(), shape,
                                        fp16_handoff=h) for h in (False, True)]
    (y32, k32, _), (y16, k16, _) = runs
    assert float((y16 - torch.from_numpy(z["expected_y"])).abs().max()) < 2e-2
    assert oracle.cosine(y16, torch.from_numpy(z["expected_y"])) >= 0.9999
    assert not torch.equal(y16, y32)
    assert torch.equal(k16, k16.half().float())  # new keys leave in FP16


def test_norm_for_projection_scales_after_rounding():
    x = torch.tensor([[3.0, 4.0, 0.001, -2.0]])
    w = torch.tensor([1.0, 0.5, 2.0, 1.5]).half()
    scale = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-5)
    expected = scale * (x * w.float()).half().float()
    assert torch.equal(oracle.norm_for_projection(x, w, 1e-5, fp16=True), expected)
    assert torch.equal(oracle.norm_for_projection(x, w, 1e-5), oracle.rms_norm(x, w, 1e-5))
