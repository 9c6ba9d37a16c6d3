"""Generate the golden fixtures that pin the CPU oracle (oracle/decode.py).

Run in a container that has transformers 5.5 and torch (both present in this
image); the fixtures are committed so the tests never need to regenerate them:

    python tests/golden/make_golden.py

Every expected value comes from the module LLM_Compiler_3 itself treats as
ground truth -- the PyTorch module evaluated on the CPU
(examples/llama/verify.py:80-82, test/Integration/attention.py:163-164):

* ``llama_layer_decode.npz`` / ``qwen3_layer_decode.npz`` -- one decode step of a
  small transformers LlamaDecoderLayer / Qwen3DecoderLayer (eager attention,
  FP32 module with FP16-representable weights), run through transformers'
  DynamicCache pre-filled with a random FP16 cache.  Two sequences at different
  positions, each run separately because DynamicCache is rectangular.
* ``sdpa_decode.npz`` -- the last query row of each case in
  test/Integration/attention.py:27-32 (mha, gqa, causal, gqa_causal_d128) against
  torch.nn.functional.scaled_dot_product_attention in FP32 (attention.py:163-164);
  the last row of a causal case sees every key, so it is a decode query.
* ``mlp.npz`` -- the Linear-ReLU-Linear module of examples/pytorch/mlp.py:44-51 at
  the MLP config's shape (batch 64, 256 -> 512 -> 256, biases), FP32 reference from
  the FP16 values (mlp.py:54-61).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _half(shape, generator, std=1.0, mean=0.0):
    return (torch.randn(shape, generator=generator) * std + mean).half()


def _layer_case(family: str, seed: int):
    from transformers import DynamicCache, LlamaConfig, Qwen3Config
    from transformers.models.llama.modeling_llama import LlamaDecoderLayer, LlamaRotaryEmbedding
    from transformers.models.qwen3.modeling_qwen3 import Qwen3DecoderLayer, Qwen3RotaryEmbedding

    if family == "llama":
        config = LlamaConfig(hidden_size=256, intermediate_size=384, num_attention_heads=2,
                             num_key_value_heads=2, head_dim=128, rms_norm_eps=1e-5,
                             rope_parameters={"rope_type": "default", "rope_theta": 500000.0},
                             attn_implementation="eager")
        layer_cls, rotary_cls = LlamaDecoderLayer, LlamaRotaryEmbedding
    else:
        config = Qwen3Config(hidden_size=256, intermediate_size=384, num_attention_heads=2,
                             num_key_value_heads=1, head_dim=128, rms_norm_eps=1e-6,
                             rope_parameters={"rope_type": "default", "rope_theta": 1000000.0},
                             attn_implementation="eager")
        layer_cls, rotary_cls = Qwen3DecoderLayer, Qwen3RotaryEmbedding
    gen = torch.Generator().manual_seed(seed)
    layer = layer_cls(config, layer_idx=0).float().eval()
    arrays = {}
    with torch.no_grad():
        for name, param in layer.named_parameters():
            if name.endswith("norm.weight"):
                value = _half(param.shape, gen, std=0.1, mean=1.0)
            else:
                value = _half(param.shape, gen, std=0.02)
            param.copy_(value.float())
            arrays["w." + name] = value.numpy()
    rotary = rotary_cls(config)
    positions = [5, 37]
    hidden = config.hidden_size
    kv, hd = config.num_key_value_heads, config.head_dim
    max_seq = 48
    x = _half((len(positions), hidden), gen, std=1.0)
    k_cache = _half((len(positions), kv, max_seq, hd), gen)
    v_cache = _half((len(positions), kv, max_seq, hd), gen)
    ys, ks, vs = [], [], []
    with torch.no_grad():
        for b, pos in enumerate(positions):
            cache = DynamicCache()
            cache.update(k_cache[b:b + 1, :, :pos].float(), v_cache[b:b + 1, :, :pos].float(), 0)
            h = x[b:b + 1].float()[:, None, :]
            pid = torch.tensor([[pos]])
            cos, sin = rotary(h, pid)
            out = layer(h, attention_mask=None, position_ids=pid, past_key_values=cache,
                        use_cache=True, position_embeddings=(cos, sin))
            out = out[0] if isinstance(out, tuple) else out
            ys.append(out[0, 0])
            ks.append(cache.layers[0].keys[0, :, pos])
            vs.append(cache.layers[0].values[0, :, pos])
    arrays.update({
        "x": x.numpy(), "positions": np.array(positions, dtype=np.int32),
        "k_cache": k_cache.numpy(), "v_cache": v_cache.numpy(),
        "expected_y": torch.stack(ys).numpy(), "expected_k_new": torch.stack(ks).numpy(),
        "expected_v_new": torch.stack(vs).numpy(),
        "shape": np.array([hidden, config.num_attention_heads, kv, hd, config.intermediate_size],
                          dtype=np.int64),
        "eps": np.array(config.rms_norm_eps, dtype=np.float64),
        "rope_theta": np.array(config.rope_parameters["rope_theta"], dtype=np.float64),
    })
    return arrays


def _sdpa_cases():
    # name, query heads, key/value heads, queries, keys, head size, causal
    # (test/Integration/attention.py:27-32)
    cases = [("mha", 2, 2, 64, 128, 32, False), ("gqa", 8, 2, 64, 256, 64, False),
             ("causal", 4, 1, 128, 128, 64, True), ("gqa_causal_d128", 8, 2, 256, 256, 128, True)]

    def tensor(shape, seed):  # attention.py:33-35
        generator = torch.Generator().manual_seed(seed)
        return (torch.randn(shape, generator=generator) * 0.5).half()

    arrays = {}
    for name, heads, kv_heads, queries, keys, depth, causal in cases:
        q = tensor((1, heads, queries, depth), 1)
        k = tensor((1, kv_heads, keys, depth), 2)
        v = tensor((1, kv_heads, keys, depth), 3)
        expected = torch.nn.functional.scaled_dot_product_attention(
            q.float(), k.float(), v.float(), is_causal=causal, enable_gqa=heads > kv_heads)
        arrays[f"{name}.q"] = q[0, :, -1].numpy()                 # [Hq, D]: last query row
        arrays[f"{name}.k"] = k.numpy()
        arrays[f"{name}.v"] = v.numpy()
        arrays[f"{name}.expected"] = expected[0, :, -1].numpy()   # [Hq, D]
    arrays["names"] = np.array([c[0] for c in cases])
    return arrays


def _mlp_case():
    gen = torch.Generator().manual_seed(11)
    batch, hidden, inner = 64, 256, 512
    x = _half((batch, hidden), gen)
    w1 = _half((inner, hidden), gen, std=(1.0 / hidden) ** 0.5)
    b1 = _half((inner,), gen, std=0.1)
    w2 = _half((hidden, inner), gen, std=(1.0 / inner) ** 0.5)
    b2 = _half((hidden,), gen, std=0.1)
    model = torch.nn.Sequential(torch.nn.Linear(hidden, inner), torch.nn.ReLU(),
                                torch.nn.Linear(inner, hidden))
    with torch.no_grad():
        model[0].weight.copy_(w1.float()); model[0].bias.copy_(b1.float())
        model[2].weight.copy_(w2.float()); model[2].bias.copy_(b2.float())
        expected = model(x.float())
    return {"x": x.numpy(), "w1": w1.numpy(), "b1": b1.numpy(), "w2": w2.numpy(),
            "b2": b2.numpy(), "expected": expected.numpy()}


def main() -> None:
    torch.set_num_threads(max(1, torch.get_num_threads()))
    np.savez_compressed(HERE / "llama_layer_decode.npz", **_layer_case("llama", 1234))
    np.savez_compressed(HERE / "qwen3_layer_decode.npz", **_layer_case("qwen3", 4321))
    np.savez_compressed(HERE / "sdpa_decode.npz", **_sdpa_cases())
    np.savez_compressed(HERE / "mlp.npz", **_mlp_case())
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
