"""Decode-step capture: one decoder layer as an exportable decode step over a
fixed-capacity KV cache, and the capture directory + plan the runtime loads.

The reference's Stage 0 splits a model into a ``@prefill`` and a ``@decode``
entry point before export: decode takes the KV cache, the positions and the
valid lengths and returns the updated cache, as flat fixed-shape tensors rather
than a ``DynamicCache`` object, which ``torch.export`` cannot return
(docs/DESIGN.md §6 Stage 0 and §8.3; the capture itself,
python/npu/capture/export.py:108-139, lifts every parameter and buffer into a
function argument after the activations, sorted by name).  This module is that
decode entry point for transformers' ``LlamaDecoderLayer`` / ``Qwen3DecoderLayer``:

* ``DecodeStep(layer, rope_theta)`` -- forward(x [B, H], k_cache, v_cache
  [B, Hkv, S, D], positions [B]) -> (y [B, H], k_cache', v_cache').  Sequence b
  writes its new key/value at ``positions[b]`` and attends keys
  ``[0, positions[b]]``: the cache layout, capacity (S), position and valid
  length (position + 1) of the runtime's KV-cache ABI (``npu_b200_kv_cache``).
  RoPE angles come from the positions and a persistent inverse-frequency buffer
  (transformers keeps that buffer non-persistent, which export cannot map).
* ``export_decode_step`` -- ``torch.export`` of the step at fixed shapes (the
  graph a torch-mlir import turns into the reference's ``00-imported.mlir``).
* ``write_decode_capture`` -- the reference's capture directory
  (``arguments.txt`` + ``arg<N>.bin``, python/npu/capture/export.py:30-40) for
  the step, and a one-layer ``plan.txt``; ``runtime.Decoder(plan).load_capture``
  runs it on the B200.
"""
from __future__ import annotations

import json
from pathlib import Path
from typing import Sequence

import torch
import torch.nn.functional as F

from .plan import DecodePlan


def _rotate_half(t: torch.Tensor) -> torch.Tensor:
    half = t.shape[-1] // 2
    return torch.cat((-t[..., half:], t[..., :half]), dim=-1)


class DecodeStep(torch.nn.Module):
    """One decode step of a transformers Llama/Qwen3 decoder layer over a flat
    fixed-capacity KV cache (see the module docstring)."""

    def __init__(self, layer: torch.nn.Module, rope_theta: float):
        super().__init__()
        self.layer = layer
        attn = layer.self_attn
        self.head_dim = int(attn.head_dim)
        self.heads = attn.q_proj.out_features // self.head_dim
        self.kv_heads = attn.k_proj.out_features // self.head_dim
        exponents = torch.arange(0, self.head_dim, 2, dtype=torch.float32) / self.head_dim
        self.register_buffer("inv_freq", 1.0 / (float(rope_theta) ** exponents), persistent=True)

    def forward(self, x: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                positions: torch.Tensor):
        layer, attn = self.layer, self.layer.self_attn
        batch, capacity = x.shape[0], k_cache.shape[2]
        d = self.head_dim
        h = layer.input_layernorm(x)
        q = attn.q_proj(h).view(batch, self.heads, d)
        k = attn.k_proj(h).view(batch, self.kv_heads, d)
        v = attn.v_proj(h).view(batch, self.kv_heads, d)
        if hasattr(attn, "q_norm"):  # Qwen3: per-head RMSNorm before RoPE
            q = attn.q_norm(q)
            k = attn.k_norm(k)
        angles = positions.to(torch.float32)[:, None] * self.inv_freq[None, :]
        angles = torch.cat((angles, angles), dim=-1)
        cos, sin = angles.cos()[:, None, :].to(q.dtype), angles.sin()[:, None, :].to(q.dtype)
        q = q * cos + _rotate_half(q) * sin
        k = k * cos + _rotate_half(k) * sin
        # The new entries land at each sequence's position; everything else is kept.
        slot = positions.to(torch.int64).view(batch, 1, 1, 1).expand(batch, self.kv_heads, 1, d)
        k_cache = k_cache.scatter(2, slot, k[:, :, None, :].to(k_cache.dtype))
        v_cache = v_cache.scatter(2, slot, v[:, :, None, :].to(v_cache.dtype))
        # Keys [0, position] of each sequence are valid.
        valid = torch.arange(capacity, device=x.device)[None, :] <= positions.to(torch.int64)[:, None]
        mask = torch.zeros(batch, 1, 1, capacity, dtype=q.dtype, device=x.device)
        mask = mask.masked_fill(~valid[:, None, None, :], float("-inf"))
        o = F.scaled_dot_product_attention(q[:, :, None, :], k_cache.to(q.dtype),
                                           v_cache.to(q.dtype), attn_mask=mask,
                                           scale=d ** -0.5, enable_gqa=True)
        x = x + attn.o_proj(o.reshape(batch, self.heads * d))
        x = x + layer.mlp(layer.post_attention_layernorm(x))
        return x, k_cache, v_cache


def example_inputs(step: DecodeStep, batch: int, capacity: int, dtype=torch.float16,
                   seed: int = 0) -> tuple[torch.Tensor, ...]:
    """Seeded (x, k_cache, v_cache, positions) of the step's shapes."""
    g = torch.Generator().manual_seed(seed)
    hidden = step.layer.input_layernorm.weight.shape[0]
    x = torch.randn(batch, hidden, generator=g).to(dtype)
    k = torch.randn(batch, step.kv_heads, capacity, step.head_dim, generator=g).to(dtype)
    v = torch.randn(batch, step.kv_heads, capacity, step.head_dim, generator=g).to(dtype)
    positions = torch.randint(0, capacity, (batch,), generator=g, dtype=torch.int64)
    return x, k, v, positions


def export_decode_step(step: DecodeStep, example: Sequence[torch.Tensor]):
    """torch.export of the decode step at the example's (fixed) shapes."""
    return torch.export.export(step, tuple(example), strict=False)


def write_decode_capture(step: DecodeStep, config, example: Sequence[torch.Tensor],
                         directory: str | Path, max_batch: int | None = None) -> Path:
    """Write the step as the reference's capture directory -- activations first
    (input0 = x, input1 / input2 = the caches, input3 = positions), then every
    parameter and buffer sorted by name, each as arg<N>.bin little-endian --
    plus a one-layer plan.txt for the runtime and a metadata.json describing the
    package (as npu-compile writes one beside its program,
    tools/npu-compile/npu-compile.cpp:479-507).  Returns the plan's path."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    named = dict(step.named_parameters())
    named.update(dict(step.named_buffers()))
    lines, arguments = [], []
    for i, tensor in enumerate(example):
        shape = "x".join(map(str, tensor.shape))
        lines.append(f"{i} input{i} {shape} {str(tensor.dtype).removeprefix('torch.')}")
        arguments.append({"index": i, "name": f"input{i}", "role": "input",
                          "shape": list(tensor.shape),
                          "dtype": str(tensor.dtype).removeprefix("torch."),
                          "bytes": tensor.numel() * tensor.element_size()})
    for j, name in enumerate(sorted(named), start=len(example)):
        tensor = named[name].detach().contiguous().cpu()
        shape = "x".join(map(str, tensor.shape))
        lines.append(f"{j} {name} {shape} {str(tensor.dtype).removeprefix('torch.')}")
        arguments.append({"index": j, "name": name, "role": "param", "shape": list(tensor.shape),
                          "dtype": str(tensor.dtype).removeprefix("torch."),
                          "bytes": tensor.numel() * tensor.element_size()})
        (directory / f"arg{j}.bin").write_bytes(tensor.numpy().astype(
            tensor.numpy().dtype.newbyteorder("<")).tobytes())
    (directory / "arguments.txt").write_text("\n".join(lines) + "\n")
    batch, capacity = example[0].shape[0], example[1].shape[2]
    plan = DecodePlan.from_hf_config(config, max_batch=max_batch or batch, max_seq=capacity,
                                     layers=1, with_vocab=False)
    path = plan.write(directory / "plan.txt")
    metadata = {"schema": "npu.b200.decode.v1", "stage": "cuda-plan", "numerical_policy": "fp16",
                "plan": path.name, "arguments": arguments,
                "outputs": [{"name": "y", "shape": list(example[0].shape)},
                            {"name": "k_cache", "shape": list(example[1].shape)},
                            {"name": "v_cache", "shape": list(example[2].shape)}],
                "param_bytes": sum(a["bytes"] for a in arguments if a["role"] == "param")}
    (directory / "metadata.json").write_text(json.dumps(metadata, indent=2) + "\n")
    return path
