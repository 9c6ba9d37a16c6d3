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
    import json
    meta = json.loads((tmp_path / "metadata.json").read_text())
    assert meta["stage"] == "cuda-plan" and meta["plan"] == "plan.txt"
    assert [a["name"] for a in meta["arguments"]] == names
    assert meta["param_bytes"] == sum(
        (tmp_path / f"arg{a['index']}.bin").stat().st_size for a in meta["arguments"]
        if a["role"] == "param")


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


def test_plan_from_capture_block(tmp_path):
    """The plan read off a captured block's argument shapes (and its lifted
    inv_freq buffer) is the plan of the layer's config."""
    from llm_compiler_3_b200.capture import write_decode_capture
    from llm_compiler_3_b200.plan import DecodePlan, plan_from_capture
    step, config, z = _step("qwen3")
    write_decode_capture(step, config, _inputs(z), tmp_path)
    got = plan_from_capture(tmp_path, max_batch=2, max_seq=48)
    want = DecodePlan.from_hf_config(config, max_batch=2, max_seq=48, layers=1, with_vocab=False)
    assert got.text() == want.text()


def test_plan_from_capture_stack_cli(tmp_path):
    """A whole-model capture (layers.<i>. names, embedding, RoPE buffer): layer
    count, vocabulary and the exact inverse frequencies; the CLI's plan parses
    with the library's own checks."""
    import ctypes
    from llm_compiler_3_b200 import _native
    from llm_compiler_3_b200.plan import main, plan_from_capture, rope_inv_freq
    H, F, V, D = 512, 1024, 1000, 128
    shapes = {"self_attn.q_proj.weight": (4 * D, H), "self_attn.k_proj.weight": (2 * D, H),
              "self_attn.v_proj.weight": (2 * D, H), "self_attn.o_proj.weight": (H, 4 * D),
              "mlp.gate_proj.weight": (F, H), "mlp.up_proj.weight": (F, H),
              "mlp.down_proj.weight": (H, F), "input_layernorm.weight": (H,),
              "post_attention_layernorm.weight": (H,)}
    names = {"model.embed_tokens.weight": (V, H), "model.norm.weight": (H,),
             "lm_head.weight": (V, H), "model.rotary_emb.inv_freq": (D // 2,)}
    for layer in range(3):
        for name, shape in shapes.items():
            names[f"model.layers.{layer}.{name}"] = shape
    lines = ["0 input0 1x7 int64"]
    for i, name in enumerate(sorted(names), start=1):
        dtype = "float32" if name.endswith("inv_freq") else "float16"
        lines.append(f"{i} {name} {'x'.join(map(str, names[name]))} {dtype}")
        if name.endswith("inv_freq"):
            inv = np.asarray(rope_inv_freq(250000.0, D), dtype="<f4")
            (tmp_path / f"arg{i}.bin").write_bytes(inv.tobytes())
    (tmp_path / "arguments.txt").write_text("\n".join(lines) + "\n")
    plan = plan_from_capture(tmp_path, max_batch=8, max_seq=512)
    assert (plan.layers, plan.hidden, plan.heads, plan.kv_heads, plan.ffn, plan.vocab) == \
        (3, H, 4, 2, F, V)
    assert plan.arch == "llama" and plan.inv_freq == rope_inv_freq(250000.0, D)
    assert abs(plan.rope_theta - 250000.0) / 250000.0 < 1e-4
    assert main(["--from-capture", str(tmp_path), "--max-batch", "8", "--max-seq", "512"]) == 0
    info = (ctypes.c_int64 * 12)()
    _native.check(_native.lib().npu_b200_plan_check(str(tmp_path / "plan.txt").encode(), info, 12))
    assert list(info)[:6] == [3, H, 4, 2, F, V]
