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


_DTYPES = {"float16": "<f2", "float32": "<f4", "bfloat16": None}


def plan_from_capture(directory: str | Path, max_batch: int, max_seq: int, *,
                      head_dim: int | None = None, rms_eps: float | None = None,
                      rope_theta: float | None = None) -> DecodePlan:
    """The decode plan of a capture directory (arguments.txt + arg<N>.bin, as
    python/npu/capture/export.py:30-40 writes it), read off its argument shapes.

    The projections give hidden size, heads, KV heads, FFN width and the layer
    count (``layers.<i>.`` names; a captured block without them is one layer);
    ``q_norm`` marks Qwen3 and gives the head dimension (else ``head_dim``,
    default 128); the embedding gives the vocabulary (0 without one).  A lifted
    RoPE ``inv_freq`` buffer is copied into the plan exactly (and gives theta).
    RMSNorm epsilon and theta are not in the weights: pass them, or the family
    defaults apply (Llama 1e-5 / 5e5, Qwen3 1e-6 / 1e6)."""
    import re

    import numpy as np

    directory = Path(directory)
    args: dict[str, tuple[int, tuple[int, ...], str]] = {}
    for line in (directory / "arguments.txt").read_text().splitlines():
        parts = line.split()
        if len(parts) != 4:
            continue
        index, name, shape, dtype = parts
        args[name] = (int(index), tuple(int(s) for s in shape.split("x")), dtype)

    def shapes(suffix: str) -> dict[int, tuple[int, ...]]:
        found = {}
        for name, (_, shape, _) in args.items():
            if name.endswith(suffix):
                m = re.search(r"layers\.(\d+)\.", name)
                found[int(m.group(1)) if m else 0] = shape
        return found

    q = shapes("self_attn.q_proj.weight")
    if not q:
        raise ValueError(f"{directory}: no self_attn.q_proj.weight in arguments.txt")
    layers = sorted(q)
    if layers != list(range(len(layers))):
        raise ValueError(f"{directory}: layers {layers} are not 0..{len(layers) - 1}")
    k, gate = shapes("self_attn.k_proj.weight"), shapes("mlp.gate_proj.weight")
    q_norm = shapes("self_attn.q_norm.weight")
    arch = "qwen3" if q_norm else "llama"
    hidden = q[0][1]
    d = head_dim or (q_norm[0][0] if q_norm else 128)
    heads, kv_heads, ffn = q[0][0] // d, k[0][0] // d, gate[0][0]
    for i in layers:
        if q[i] != q[0] or k.get(i) != k[0] or gate.get(i) != gate[0]:
            raise ValueError(f"{directory}: layer {i} has other projection shapes than layer 0")
    if q[0][0] % d or k[0][0] % d:
        raise ValueError(f"{directory}: q/k rows {q[0][0]}/{k[0][0]} not multiples of head_dim {d}")
    embed = shapes("embed_tokens.weight")
    vocab = embed[0][0] if embed else 0
    inv_freq: list[float] = []
    for name, (index, shape, dtype) in args.items():
        if name.endswith("inv_freq") and _DTYPES.get(dtype) and shape == (d // 2,):
            raw = (directory / f"arg{index}.bin").read_bytes()
            inv_freq = np.frombuffer(raw, dtype=_DTYPES[dtype]).astype(np.float32).tolist()
            break
    if rope_theta is None and len(inv_freq) > 1:
        # theta = inv_freq[1] ** (-d / 2); FP32 inverse frequencies pin it only
        # to ~6 digits, so take the shortest decimal that regenerates the table.
        estimate = float(inv_freq[1]) ** (-d / 2.0)
        rope_theta = estimate
        for digits in range(1, 10):
            candidate = float(f"{estimate:.{digits}g}")
            if rope_inv_freq(candidate, d) == inv_freq:
                rope_theta = candidate
                break
    if rope_theta is None:
        rope_theta = 1e6 if arch == "qwen3" else 5e5
    if rms_eps is None:
        rms_eps = 1e-6 if arch == "qwen3" else 1e-5
    return DecodePlan(arch=arch, hidden=hidden, heads=heads, kv_heads=kv_heads, head_dim=d,
                      ffn=ffn, layers=len(layers), vocab=vocab, rms_eps=float(rms_eps),
                      rope_theta=float(rope_theta), max_batch=max_batch, max_seq=max_seq,
                      inv_freq=inv_freq)


def main(argv=None) -> int:
    import argparse
    ap = argparse.ArgumentParser(description="Write a libnpu_b200 plan from a capture directory.")
    ap.add_argument("--from-capture", required=True, metavar="DIR")
    ap.add_argument("--max-batch", type=int, required=True)
    ap.add_argument("--max-seq", type=int, required=True)
    ap.add_argument("--head-dim", type=int)
    ap.add_argument("--rms-eps", type=float)
    ap.add_argument("--rope-theta", type=float)
    ap.add_argument("--out", help="plan path (default: DIR/plan.txt)")
    a = ap.parse_args(argv)
    plan = plan_from_capture(a.from_capture, a.max_batch, a.max_seq, head_dim=a.head_dim,
                             rms_eps=a.rms_eps, rope_theta=a.rope_theta)
    print(plan.write(a.out or Path(a.from_capture) / "plan.txt"))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
