"""Decode runtime (libnpu_b200 contexts) against the CPU oracle and transformers.

Exact checks: the new K/V entry lands at `position` and no other cache entry
changes; greedy token ids.  Toleranced: FP16 outputs within max-abs 2e-2 and
cosine >= 0.9999 of the FP32-accumulated oracle."""
import os
import tempfile
import warnings
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN, seeded

pytestmark = pytest.mark.gpu

ATOL = 2e-2
COS = 0.9999


def _check(got, ref, atol=ATOL):
    got = got.float()
    err = float((got - ref).abs().max())
    cos = oracle.cosine(got, ref)
    assert err <= atol and cos >= COS, f"max-abs {err:.3e}, cosine {cos:.6f}"


def _golden(family):
    return dict(np.load(GOLDEN / f"{family}_layer_decode.npz"))


def _golden_plan(z, family, max_batch):
    from llm_compiler_3_b200.plan import DecodePlan
    hidden, heads, kv, hd, ffn = (int(v) for v in z["shape"])
    return DecodePlan(arch=family, hidden=hidden, heads=heads, kv_heads=kv, head_dim=hd, ffn=ffn,
                      layers=1, vocab=0, rms_eps=float(z["eps"]),
                      rope_theta=float(z["rope_theta"]), max_batch=max_batch,
                      max_seq=z["k_cache"].shape[2])


@pytest.mark.parametrize("family", ["llama", "qwen3"])
def test_layer_matches_transformers(cuda, family):
    """One decode step of the transformers decoder layer (golden fixture) through
    the runtime: output, new K/V entries, and exact cache indexing."""
    from llm_compiler_3_b200.runtime import Decoder
    z = _golden(family)
    with Decoder(_golden_plan(z, family, max_batch=2)) as dec:
        for name, arr in z.items():
            if name.startswith("w."):
                dec.set_weight(name[2:], torch.from_numpy(arr))
        k, v = dec.kv_cache(0)
        k.copy_(torch.from_numpy(z["k_cache"]).cuda())
        v.copy_(torch.from_numpy(z["v_cache"]).cuda())
        y = dec.forward_hidden(torch.from_numpy(z["x"]), z["positions"])
        _check(y, torch.from_numpy(z["expected_y"]))
        k_after, v_after = k.cpu(), v.cpu()
    before_k, before_v = torch.from_numpy(z["k_cache"]), torch.from_numpy(z["v_cache"])
    for b, p in enumerate(z["positions"].tolist()):
        _check(k_after[b, :, p], torch.from_numpy(z["expected_k_new"][b]))
        _check(v_after[b, :, p], torch.from_numpy(z["expected_v_new"][b]))
        keep = torch.ones(before_k.shape[2], dtype=torch.bool)
        keep[p] = False
        assert torch.equal(k_after[b][:, keep], before_k[b][:, keep])
        assert torch.equal(v_after[b][:, keep], before_v[b][:, keep])


def test_capture_directory_boundary(cuda):
    """Weights read from a capture directory in the reference's format
    (arguments.txt + arg<N>.bin, python/npu/capture/export.py:30-40) give the
    same step as weights set one by one."""
    from llm_compiler_3_b200.runtime import Decoder
    z = _golden("llama")
    names = [k[2:] for k in z if k.startswith("w.")]
    with tempfile.TemporaryDirectory() as tmp:
        lines = [f"0 input0 2x{z['x'].shape[1]} float16"]
        for i, name in enumerate(names, start=1):
            arr = z["w." + name]
            (Path(tmp) / f"arg{i}.bin").write_bytes(arr.astype("<f2").tobytes())
            lines.append(f"{i} block.{name} {'x'.join(map(str, arr.shape))} float16")
        (Path(tmp) / "arguments.txt").write_text("\n".join(lines) + "\n")
        with Decoder(_golden_plan(z, "llama", max_batch=2)) as dec:
            dec.load_capture(tmp)
            k, v = dec.kv_cache(0)
            k.copy_(torch.from_numpy(z["k_cache"]).cuda())
            v.copy_(torch.from_numpy(z["v_cache"]).cuda())
            y = dec.forward_hidden(torch.from_numpy(z["x"]), z["positions"])
    _check(y, torch.from_numpy(z["expected_y"]))


def _layer_weights(shape, seed, qk_norm=False):
    H, D = shape.hidden, shape.head_dim
    w = {
        "self_attn.q_proj.weight": seeded((shape.heads * D, H), seed + 1, 0.02),
        "self_attn.k_proj.weight": seeded((shape.kv_heads * D, H), seed + 2, 0.02),
        "self_attn.v_proj.weight": seeded((shape.kv_heads * D, H), seed + 3, 0.02),
        "self_attn.o_proj.weight": seeded((H, shape.heads * D), seed + 4, 0.02),
        "mlp.gate_proj.weight": seeded((shape.ffn, H), seed + 5, 0.02),
        "mlp.up_proj.weight": seeded((shape.ffn, H), seed + 6, 0.02),
        "mlp.down_proj.weight": seeded((H, shape.ffn), seed + 7, 0.02),
        "input_layernorm.weight": torch.ones(H, dtype=torch.float16),
        "post_attention_layernorm.weight": torch.ones(H, dtype=torch.float16),
    }
    if qk_norm:
        w["self_attn.q_norm.weight"] = torch.ones(D, dtype=torch.float16)
        w["self_attn.k_norm.weight"] = torch.ones(D, dtype=torch.float16)
    return w


def _run_layer_config(plan, shape, batch, position, seed, qk_norm):
    from llm_compiler_3_b200.runtime import Decoder
    weights = _layer_weights(shape, seed, qk_norm)
    x = seeded((batch, shape.hidden), seed + 10)
    kc = seeded((batch, shape.kv_heads, plan.max_seq, shape.head_dim), seed + 11)
    vc = seeded((batch, shape.kv_heads, plan.max_seq, shape.head_dim), seed + 12)
    kc[:, :, position:] = 0
    vc[:, :, position:] = 0
    positions = torch.full((batch,), position, dtype=torch.int32)
    with Decoder(plan) as dec:
        dec.set_weights(weights)
        k, v = dec.kv_cache(0)
        k[:batch].copy_(kc.cuda())
        v[:batch].copy_(vc.cuda())
        y = dec.forward_hidden(x, positions)
        k_after, v_after = k[:batch].cpu(), v[:batch].cpu()
    ref, k_new, v_new = oracle.decoder_layer_decode(weights, x, positions, kc.clone(), vc.clone(),
                                                    shape)
    _check(y, ref)
    _check(k_after[:, :, position], k_new)
    _check(v_after[:, :, position], v_new)
    keep = torch.ones(plan.max_seq, dtype=torch.bool)
    keep[position] = False
    assert torch.equal(k_after[:, :, keep], kc[:, :, keep])
    assert torch.equal(v_after[:, :, keep], vc[:, :, keep])


def test_llama_layer_batch1(cuda):
    """Llama-3-8B-shaped layer, batch 1, position 2047 over a 2047-token cache."""
    from llm_compiler_3_b200.plan import llama3_8b
    plan = llama3_8b(layers=1, vocab=0, max_batch=1, max_seq=2048)
    _run_layer_config(plan, oracle.LLAMA3_8B, batch=1, position=2047, seed=300, qk_norm=False)


def test_qwen3_layer_batch16(cuda):
    """Qwen3-8B-shaped layer (QK-norm, theta 1e6), batch 16, 8191 cached + 1 new."""
    from llm_compiler_3_b200.plan import qwen3_8b
    plan = qwen3_8b(layers=1, vocab=0, max_batch=16, max_seq=8192)
    _run_layer_config(plan, oracle.QWEN3_8B, batch=16, position=8191, seed=400, qk_norm=True)


def test_ragged_positions_batch(cuda):
    """Different positions per sequence in one step (ragged KV lengths)."""
    from llm_compiler_3_b200.plan import llama3_8b
    from llm_compiler_3_b200.runtime import Decoder
    shape = oracle.LLAMA3_8B
    plan = llama3_8b(layers=1, vocab=0, max_batch=4, max_seq=512)
    weights = _layer_weights(shape, 500)
    x = seeded((3, shape.hidden), 510)
    kc = seeded((3, 8, 512, 128), 511)
    vc = seeded((3, 8, 512, 128), 512)
    positions = torch.tensor([0, 300, 511], dtype=torch.int32)
    with Decoder(plan) as dec:
        dec.set_weights(weights)
        k, v = dec.kv_cache(0)
        k[:3].copy_(kc.cuda())
        v[:3].copy_(vc.cuda())
        y = dec.forward_hidden(x, positions)
    ref, _, _ = oracle.decoder_layer_decode(weights, x, positions, kc.clone(), vc.clone(), shape)
    _check(y, ref)


def _stack_setup(layers, batch, max_seq, position, seed):
    from llm_compiler_3_b200.plan import llama3_8b
    shape = oracle.LLAMA3_8B
    plan = llama3_8b(layers=layers, max_batch=batch, max_seq=max_seq)
    gen = torch.Generator().manual_seed(seed)
    tokens = torch.randint(0, shape.vocab, (batch,), generator=gen, dtype=torch.int64).int()
    positions = torch.full((batch,), position, dtype=torch.int32)
    top = {"model.embed_tokens.weight": seeded((shape.vocab, shape.hidden), seed + 1, 0.02),
           "model.norm.weight": torch.ones(shape.hidden, dtype=torch.float16),
           "lm_head.weight": seeded((shape.vocab, shape.hidden), seed + 2, 0.02)}
    return shape, plan, tokens, positions, top


def test_stack_argmax_two_layers(cuda):
    """The full-stack path (embedding, layers, final norm, LM head, argmax) at
    the stack config's widths and batch 64 with 2 layers: ids must equal the
    oracle's; any mismatch is reported with the oracle's top-2 gap."""
    from llm_compiler_3_b200.runtime import Decoder
    layers, batch, max_seq, position = 2, 64, 512, 511
    shape, plan, tokens, positions, top = _stack_setup(layers, batch, max_seq, position, 900)
    per_layer = [_layer_weights(shape, 1000 + 100 * i) for i in range(layers)]
    caches = [(seeded((batch, 8, max_seq, 128), 2000 + i), seeded((batch, 8, max_seq, 128), 3000 + i))
              for i in range(layers)]
    with Decoder(plan) as dec:
        for name, t in top.items():
            dec.set_weight(name, t)
        for i, w in enumerate(per_layer):
            for name, t in w.items():
                dec.set_weight(f"model.layers.{i}.{name}", t)
            k, v = dec.kv_cache(i)
            k.copy_(caches[i][0].cuda())
            v.copy_(caches[i][1].cuda())
        ids = dec.step(tokens.numpy(), positions.numpy())
    ref_ids, logits = oracle.stack_decode(
        lambda i: per_layer[i], layers, top["model.embed_tokens.weight"], top["model.norm.weight"],
        top["lm_head.weight"], tokens, positions,
        lambda i: (caches[i][0].clone(), caches[i][1].clone()), shape, return_logits=True,
        fp16_handoff=True)
    _check_ids(ids, ref_ids, logits)


def _check_ids(ids, ref_ids, logits):
    """Greedy ids must equal the oracle's wherever the oracle's top-2 logit gap
    exceeds what accumulation order alone can move (4e-3 of the logit standard
    deviation; the oracle given here rounds at the kernels' FP16 hand-offs
    wherever a caller can, so only summation order differs).  A closer pair is a
    near-tie: it may only pick the oracle's runner-up, and every such flip is
    reported as a warning with its gap.  Returns the number of flips."""
    ids = np.asarray(ids)
    ref = ref_ids.numpy()
    top2 = logits.topk(2, dim=-1)
    gaps = (top2.values[:, 0] - top2.values[:, 1]).numpy()
    tie_bound = 4e-3 * float(logits.std())
    mism = np.nonzero(ids != ref)[0]
    for b in mism:
        assert gaps[b] < tie_bound, (
            f"sequence {b}: id {ids[b]} != oracle {ref[b]} with top-2 gap {gaps[b]:.3e} "
            f">= bound {tie_bound:.3e}")
        assert ids[b] == int(top2.indices[b, 1]), f"sequence {b}: not the oracle's runner-up"
        warnings.warn(f"near-tie flip, sequence {b}: id {ids[b]} is the oracle's runner-up "
                      f"(oracle {ref[b]}), top-2 gap {gaps[b]:.3e} < bound {tie_bound:.3e}")
    assert len(mism) <= max(1, len(ids) // 16), f"{len(mism)} near-tie flips of {len(ids)}"
    return len(mism)


def test_decode_errors_are_status_codes(cuda):
    from llm_compiler_3_b200 import _native
    from llm_compiler_3_b200.plan import llama3_8b
    from llm_compiler_3_b200.runtime import Decoder
    plan = llama3_8b(layers=1, vocab=0, max_batch=2, max_seq=64)
    with Decoder(plan) as dec:
        with pytest.raises(_native.NpuError, match="never set"):
            dec.forward_hidden(torch.zeros(1, 4096, dtype=torch.float16), [3])
        dec.set_weights(_layer_weights(oracle.LLAMA3_8B, 7))
        with pytest.raises(_native.NpuError, match="outside the cache"):
            dec.forward_hidden(torch.zeros(1, 4096, dtype=torch.float16), [64])
        with pytest.raises(_native.NpuError, match="batch"):
            dec.forward_hidden(torch.zeros(3, 4096, dtype=torch.float16), [1, 2, 3])
        with pytest.raises(_native.NpuError, match="no vocabulary"):
            dec.step([1], [0])


def test_stack_config_full_size(cuda):
    """The stack config at full size: 32 Llama-3-8B-shaped layers, LM head
    4096x128256, batch 64, each sequence at position 4095 over a 4095-token cache.
    Weights and caches are generated on the device (seeded) and read back layer by
    layer for the oracle, so both sides see identical FP16 inputs."""
    from llm_compiler_3_b200.plan import llama3_8b
    from llm_compiler_3_b200.runtime import Decoder
    shape = oracle.LLAMA3_8B
    layers, batch, seq = 32, 64, 4096
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    H, D = shape.hidden, shape.head_dim
    shapes = {"self_attn.q_proj.weight": (shape.heads * D, H),
              "self_attn.k_proj.weight": (shape.kv_heads * D, H),
              "self_attn.v_proj.weight": (shape.kv_heads * D, H),
              "self_attn.o_proj.weight": (H, shape.heads * D),
              "mlp.gate_proj.weight": (shape.ffn, H), "mlp.up_proj.weight": (shape.ffn, H),
              "mlp.down_proj.weight": (H, shape.ffn)}

    def randn(shp, seed, std):
        gen.manual_seed(seed)
        return (torch.randn(shp, device=dev, generator=gen) * std).half()

    def layer(i):
        w = {n: randn(s, 1000 + 16 * i + j, 0.02) for j, (n, s) in enumerate(shapes.items())}
        w["input_layernorm.weight"] = torch.ones(H, dtype=torch.float16, device=dev)
        w["post_attention_layernorm.weight"] = torch.ones(H, dtype=torch.float16, device=dev)
        return w

    embed = randn((shape.vocab, H), 11, 0.02)
    lm = randn((shape.vocab, H), 12, 0.02)
    norm = torch.ones(H, dtype=torch.float16, device=dev)
    gen.manual_seed(7)
    tokens = torch.randint(0, shape.vocab, (batch,), device=dev, generator=gen, dtype=torch.int32)
    positions = torch.full((batch,), seq - 1, dtype=torch.int32)
    with Decoder(llama3_8b(layers=layers, max_batch=batch, max_seq=seq)) as dec:
        dec.set_weight("model.embed_tokens.weight", embed)
        dec.set_weight("lm_head.weight", lm)
        dec.set_weight("model.norm.weight", norm)
        for i in range(layers):
            for name, t in layer(i).items():
                dec.set_weight(f"model.layers.{i}.{name}", t)
            k, v = dec.kv_cache(i)
            gen.manual_seed(50000 + 2 * i)
            k[:, :, : seq - 1].normal_(generator=gen)
            gen.manual_seed(50001 + 2 * i)
            v[:, :, : seq - 1].normal_(generator=gen)
        ids = dec.step(tokens.cpu().numpy(), positions.numpy())
        torch.set_num_threads(os.cpu_count() or 1)
        ref_ids, logits = oracle.stack_decode(
            lambda i: {n: t.cpu() for n, t in layer(i).items()}, layers, embed.cpu(), norm.cpu(),
            lm.cpu(), tokens.cpu(), positions,
            lambda i: tuple(t.cpu() for t in dec.kv_cache(i)), shape, return_logits=True,
            fp16_handoff=True)
    _check_ids(ids, ref_ids, logits)
