"""Decode-step capture (llm_compiler_3_b200/capture.py): the flat-cache decode
step of a transformers decoder layer, pinned to transformers' own DynamicCache
decode (the golden fixtures), exportable with torch.export, written as the
reference's capture directory (python/npu/capture/export.py:30-40) with a plan
the runtime parses -- and, on a GPU, run by the runtime from that directory."""
import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from conftest import GOLDEN


def _layer(family):
    """A transformers layer of the golden fixture's shape with its weights."""
    from transformers import LlamaConfig, Qwen3Config
    from transformers.models.llama.modeling_llama import LlamaDecoderLayer
    from transformers.models.qwen3.modeling_qwen3 import Qwen3DecoderLayer
    z = dict(np.load(GOLDEN / f"{family}_layer_decode.npz"))
    hidden, heads, kv, hd, ffn = (int(v) for v in z["shape"])
    common = dict(hidden_size=hidden, intermediate_size=ffn, num_attention_heads=heads,
                  num_key_value_heads=kv, head_dim=hd, rms_norm_eps=float(z["eps"]),
                  rope_parameters={"rope_type": "default", "rope_theta": float(z["rope_theta"])},
                  attn_implementation="eager")
    config = LlamaConfig(**common) if family == "llama" else Qwen3Config(**common)
    cls = LlamaDecoderLayer if family == "llama" else Qwen3DecoderLayer
    layer = cls(config, layer_idx=0).float().eval()
    with torch.no_grad():
        for name, param in layer.named_parameters():
            param.copy_(torch.from_numpy(z["w." + name]).float())
    return layer, config, z


def _step(family):
    from llm_compiler_3_b200.capture import DecodeStep
    layer, config, z = _layer(family)
    return DecodeStep(layer, float(z["rope_theta"])), config, z


def _inputs(z, dtype=torch.float32):
    return (torch.from_numpy(z["x"]).to(dtype), torch.from_numpy(z["k_cache"]).to(dtype),
            torch.from_numpy(z["v_cache"]).to(dtype),
            torch.from_numpy(z["positions"]).to(torch.int64))


@pytest.mark.parametrize("family", ["llama", "qwen3"])
def test_decode_step_matches_transformers(family):
    """Output, new cache entries at each position, and every other entry untouched."""
    step, _, z = _step(family)
    x, k, v, pos = _inputs(z)
    with torch.no_grad():
        y, k2, v2 = step(x, k, v, pos)
    torch.testing.assert_close(y, torch.from_numpy(z["expected_y"]), atol=2e-5, rtol=0)
    for b, p in enumerate(z["positions"].tolist()):
        torch.testing.assert_close(k2[b, :, p], torch.from_numpy(z["expected_k_new"][b]),
                                   atol=2e-5, rtol=0)
        torch.testing.assert_close(v2[b, :, p], torch.from_numpy(z["expected_v_new"][b]),
                                   atol=2e-5, rtol=0)
        keep = torch.ones(k.shape[2], dtype=torch.bool)
        keep[p] = False
        assert torch.equal(k2[b][:, keep], k[b][:, keep]) and torch.equal(v2[b][:, keep], v[b][:, keep])


@pytest.mark.parametrize("family", ["llama", "qwen3"])
def test_decode_step_exports(family):
    """torch.export at fixed shapes (flat cache in and out, no DynamicCache);
    the exported program computes what the module does."""
    from llm_compiler_3_b200.capture import export_decode_step
    step, _, z = _step(family)
    example = _inputs(z)
    exported = export_decode_step(step, example)
    with torch.no_grad():
        want = step(*example)
        got = exported.module()(*example)
    for a, b in zip(got, want):
        torch.testing.assert_close(a, b, atol=1e-6, rtol=0)


def test_capture_directory_layout(tmp_path):
    """Activations first, then parameters and buffers sorted by name, each as
    little-endian arg<N>.bin; the plan parses with the library's own checks."""
    from llm_compiler_3_b200 import _native
    from llm_compiler_3_b200.capture import write_decode_capture
    step, config, z = _step("llama")
    step = step.half()
    example = _inputs(z, torch.float16)
    plan_path = write_decode_capture(step, config, example, tmp_path)
    lines = (tmp_path / "arguments.txt").read_text().splitlines()
    names = [line.split()[1] for line in lines]
    assert names[:4] == ["input0", "input1", "input2", "input3"]
    params = names[4:]
    assert params == sorted(params) and "layer.self_attn.q_proj.weight" in params
    for line in lines[4:]:
        index, name, shape, dtype = line.split()
        n = int(np.prod([int(s) for s in shape.split("x")]))
        size = (tmp_path / f"arg{index}.bin").stat().st_size
        assert size == n * (2 if dtype == "float16" else 4)
        if name == "layer.self_attn.q_proj.weight":
            got = np.frombuffer((tmp_path / f"arg{index}.bin").read_bytes(), dtype="<f2")
            assert np.array_equal(got, z["w.self_attn.q_proj.weight"].reshape(-1))
    info = (ctypes.c_int64 * 12)()
    _native.check(_native.lib().npu_b200_plan_check(str(plan_path).encode(), info, 12))
    assert list(info)[:4] == [1, int(z["shape"][0]), int(z["shape"][1]), int(z["shape"][2])]
    assert info[8] == z["k_cache"].shape[2]


@pytest.mark.gpu
@pytest.mark.parametrize("family", ["llama", "qwen3"])
def test_runtime_runs_capture_directory(cuda, tmp_path, family):
    """The runtime loads the written directory and plan and computes the step's
    output and cache entries (FP16 storage, FP32 accumulation tolerances)."""
    import oracle
    from llm_compiler_3_b200.capture import write_decode_capture
    from llm_compiler_3_b200.runtime import Decoder
    step, config, z = _step(family)
    example16 = _inputs(z, torch.float16)
    with torch.no_grad():
        want_y, want_k, want_v = step(*_inputs(z))
    plan_path = write_decode_capture(step.half(), config, example16, tmp_path)
    with Decoder(plan_path) as dec:
        dec.load_capture(tmp_path)
        k, v = dec.kv_cache(0)
        k.copy_(example16[1].cuda())
        v.copy_(example16[2].cuda())
        y = dec.forward_hidden(example16[0], z["positions"])
        k_after, v_after = k.cpu(), v.cpu()
    assert float((y.float() - want_y).abs().max()) <= 2e-2
    assert oracle.cosine(y.float(), want_y) >= 0.9999
    for b, p in enumerate(z["positions"].tolist()):
        assert float((k_after[b, :, p].float() - want_k[b, :, p]).abs().max()) <= 2e-2
        assert float((v_after[b, :, p].float() - want_v[b, :, p]).abs().max()) <= 2e-2
