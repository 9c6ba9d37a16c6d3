"""Per-rank weight image (npu_b200_save_image / npu_b200_load_image): a context
loaded from the image computes exactly what the context that wrote it does, and
every stamp, size and checksum is checked on load."""
import numpy as np
import pytest
import torch

from conftest import seeded

pytestmark = pytest.mark.gpu


def _plan(arch="qwen3", max_seq=128):
    from llm_compiler_3_b200.plan import DecodePlan
    return DecodePlan(arch=arch, hidden=512, heads=4, kv_heads=2, head_dim=128, ffn=1024,
                      layers=2, vocab=4096, rms_eps=1e-6, rope_theta=1e6, max_batch=4,
                      max_seq=max_seq)


def _fill(dec, plan):
    H, D = plan.hidden, plan.head_dim
    shapes = {"self_attn.q_proj.weight": (plan.heads * D, H),
              "self_attn.k_proj.weight": (plan.kv_heads * D, H),
              "self_attn.v_proj.weight": (plan.kv_heads * D, H),
              "self_attn.o_proj.weight": (H, plan.heads * D),
              "mlp.gate_proj.weight": (plan.ffn, H), "mlp.up_proj.weight": (plan.ffn, H),
              "mlp.down_proj.weight": (H, plan.ffn)}
    seed = 1
    for layer in range(plan.layers):
        for name, shape in shapes.items():
            dec.set_weight(f"model.layers.{layer}.{name}", seeded(shape, seed, 0.03))
            seed += 1
        for name in ("input_layernorm.weight", "post_attention_layernorm.weight",
                     "self_attn.q_norm.weight", "self_attn.k_norm.weight"):
            n = D if "_norm.weight" in name and "self_attn" in name else H
            dec.set_weight(f"model.layers.{layer}.{name}",
                           (1 + 0.1 * seeded((n,), seed).float()).half())
            seed += 1
    dec.set_weight("model.embed_tokens.weight", seeded((plan.vocab, H), 90, 0.02))
    dec.set_weight("model.norm.weight", torch.ones(H, dtype=torch.float16))
    dec.set_weight("lm_head.weight", seeded((plan.vocab, H), 91, 0.02))


def _steps(dec, caches):
    for i, (k, v) in enumerate(caches):
        dk, dv = dec.kv_cache(i)
        dk.copy_(k.cuda())
        dv.copy_(v.cuda())
    ids = dec.step(np.array([3, 4000, 17, 1], dtype=np.int32), [0, 5, 127, 64])
    x = seeded((2, 512), 77)
    y = dec.forward_hidden(x, [9, 100])
    return ids, y


def test_image_round_trip(cuda, tmp_path):
    from llm_compiler_3_b200.runtime import Decoder
    plan = _plan()
    caches = [(seeded((4, 2, 128, 128), 200 + i), seeded((4, 2, 128, 128), 300 + i))
              for i in range(plan.layers)]
    with Decoder(plan) as a:
        _fill(a, plan)
        want_ids, want_y = _steps(a, caches)
        a.save_image(tmp_path)
    assert (tmp_path / "rank0-of-1" / "image.txt").exists()
    with Decoder(plan) as b:
        b.load_image(tmp_path)
        got_ids, got_y = _steps(b, caches)
    assert np.array_equal(got_ids, want_ids)
    assert torch.equal(got_y, want_y)


def test_image_rejects_damage_and_mismatch(cuda, tmp_path):
    from llm_compiler_3_b200 import _native
    from llm_compiler_3_b200.runtime import Decoder
    plan = _plan()
    with Decoder(plan) as a:
        with pytest.raises(_native.NpuError, match="never set"):
            a.save_image(tmp_path)             # weights missing
        _fill(a, plan)
        a.save_image(tmp_path)
    with Decoder(_plan(max_seq=256)) as other:  # another plan: another fingerprint
        with pytest.raises(_native.NpuError, match="another plan"):
            other.load_image(tmp_path)
    blob = tmp_path / "rank0-of-1" / "layers.1.gate_up.bin"
    data = bytearray(blob.read_bytes())
    data[12345] ^= 0x40
    blob.write_bytes(bytes(data))
    with Decoder(plan) as b:
        with pytest.raises(_native.NpuError, match="checksum"):
            b.load_image(tmp_path)
