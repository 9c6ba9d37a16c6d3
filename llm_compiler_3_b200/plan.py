"""Decode plans: the model shape and runtime limits a libnpu_b200 context runs.

A plan file is the B200 path's stamped stage file: strict ``key = value`` lines
(unknown or duplicate keys are rejected, like the reference's HardwareConfig
parser, lib/Target/HardwareConfig.cpp:18-71) carrying ``stage = cuda-plan`` and
``schema = 1`` (the reference stamps ``npu.stage`` / ``npu.schema`` on every stage
file, tools/npu-compile/npu-compile.cpp:226-233).  The library fingerprints the
text with FNV-1a as the reference fingerprints its hardware file
(HardwareConfig.cpp:67-70).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from pathlib import Path

import torch


def rope_inv_freq(theta: float, head_dim: int) -> list[float]:
    """transformers' default RoPE inverse frequencies, bit for bit (FP32)."""
    exponent = torch.arange(0, head_dim, 2, dtype=torch.int64).to(torch.float32) / head_dim
    return (1.0 / (theta ** exponent)).tolist()


@dataclass
class DecodePlan:
    arch: str                 # "llama" | "qwen3"
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    layers: int
    vocab: int                # 0: hidden-state plan (no embedding / LM head)
    rms_eps: float
    rope_theta: float
    max_batch: int
    max_seq: int
    inv_freq: list[float] = field(default_factory=list)

    def __post_init__(self):
        if not self.inv_freq:
            self.inv_freq = rope_inv_freq(self.rope_theta, self.head_dim)

    @property
    def qk_norm(self) -> int:
        return 1 if self.arch == "qwen3" else 0

    def text(self) -> str:
        lines = [
            "# libnpu_b200 decode plan",
            "stage = cuda-plan",
            "schema = 1",
            f"arch = {self.arch}",
            f"hidden = {self.hidden}",
            f"heads = {self.heads}",
            f"kv_heads = {self.kv_heads}",
            f"head_dim = {self.head_dim}",
            f"ffn = {self.ffn}",
            f"layers = {self.layers}",
            f"vocab = {self.vocab}",
            f"rms_eps = {self.rms_eps!r}",
            f"rope_theta = {self.rope_theta!r}",
            f"qk_norm = {self.qk_norm}",
            f"max_batch = {self.max_batch}",
            f"max_seq = {self.max_seq}",
            "inv_freq = " + " ".join(float(f).hex() for f in self.inv_freq),
        ]
        return "\n".join(lines) + "\n"

    def write(self, path: str | Path) -> Path:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        path.write_text(self.text())
        return path

    @classmethod
    def from_hf_config(cls, config, max_batch: int, max_seq: int, layers: int | None = None,
                       with_vocab: bool = True) -> "DecodePlan":
        """Plan for a transformers LlamaConfig / Qwen3Config."""
        name = type(config).__name__.lower()
        arch = "qwen3" if "qwen3" in name else "llama"
        head_dim = getattr(config, "head_dim", None) or config.hidden_size // config.num_attention_heads
        rope = getattr(config, "rope_parameters", None) or {}
        theta = float(rope.get("rope_theta", getattr(config, "rope_theta", 10000.0)))
        if rope.get("rope_type", "default") != "default":
            raise ValueError(f"RoPE type {rope.get('rope_type')} is not supported")
        return cls(arch=arch, hidden=config.hidden_size, heads=config.num_attention_heads,
                   kv_heads=config.num_key_value_heads, head_dim=head_dim,
                   ffn=config.intermediate_size,
                   layers=layers if layers is not None else config.num_hidden_layers,
                   vocab=config.vocab_size if with_vocab else 0, rms_eps=float(config.rms_norm_eps),
                   rope_theta=theta, max_batch=max_batch, max_seq=max_seq)


def llama3_8b(layers: int = 32, vocab: int = 128256, max_batch: int = 64,
              max_seq: int = 4096) -> DecodePlan:
    """Llama-3-8B shape: hidden 4096, 32/8 heads of 128, SwiGLU 14336, eps 1e-5, theta 5e5."""
    return DecodePlan(arch="llama", hidden=4096, heads=32, kv_heads=8, head_dim=128, ffn=14336,
                      layers=layers, vocab=vocab, rms_eps=1e-5, rope_theta=500000.0,
                      max_batch=max_batch, max_seq=max_seq)


def qwen3_8b(layers: int = 36, vocab: int = 151936, max_batch: int = 16,
             max_seq: int = 8192) -> DecodePlan:
    """Qwen3-8B shape: hidden 4096, 32/8 heads of 128, SwiGLU 12288, QK-norm, eps 1e-6, theta 1e6."""
    return DecodePlan(arch="qwen3", hidden=4096, heads=32, kv_heads=8, head_dim=128, ffn=12288,
                      layers=layers, vocab=vocab, rms_eps=1e-6, rope_theta=1000000.0,
                      max_batch=max_batch, max_seq=max_seq)
