"""CPU interpreter of a graph plan (graph.txt) -- TEST INFRASTRUCTURE ONLY.

Executes the ops of a capture directory's graph.txt in FP32 on the CPU, with
every op result stored as FP16 as the B200 runtime stores it: ``linear`` is the
reference's matmul (FP16 operands, FP32 accumulation, one FP16 rounding at the
write-out, lib/Transforms/Normalize.cpp:123-192) plus bias and the fused ReLU
(Normalize.cpp:494-507); ``sdpa`` is npu.attention (NPUDialect.td:31-61) with
torch's top-left causal mask (Attention.cpp:70-92).  The parser restates the
file format on its own so the checker shares no code with the product.
"""
from __future__ import annotations

from pathlib import Path
from typing import Sequence

import numpy as np
import torch

from .decode import attention_prefill, linear

__all__ = ["run_graph_plan"]


def _dims(text: str) -> tuple[int, ...]:
    return tuple(int(d) for d in text.split("x"))


def run_graph_plan(directory: str | Path, inputs: Sequence[torch.Tensor]) -> list[torch.Tensor]:
    """Outputs (FP16-valued FP32 tensors, in their graph.txt order) of the plan
    in `directory` for `inputs` (in their graph.txt order)."""
    directory = Path(directory)
    tensors, aliases, ops, ins, outs = {}, {}, [], [], []
    for raw in (directory / "graph.txt").read_text().splitlines():
        f = raw.split()
        if not f or f[0].startswith("npu."):
            continue
        if f[0] == "tensor":
            tensors[f[1]] = (f[2], _dims(f[4]), int(f[6]) if len(f) > 6 else None)
            if f[2] == "input":
                ins.append(f[1])
            elif f[2] == "output":
                outs.append(f[1])
        elif f[0] == "alias":
            aliases[f[1]] = (f[2], _dims(f[3]))
        elif f[0] == "op":
            ops.append(f[1:])
    values: dict[str, torch.Tensor] = {}
    for name, tensor in zip(ins, inputs):
        values[name] = tensor.to(torch.float16).float().reshape(tensors[name][1])
    for name, (role, dims, arg) in tensors.items():
        if role == "param":
            raw = np.frombuffer((directory / f"arg{arg}.bin").read_bytes(), dtype="<f2")
            values[name] = torch.from_numpy(raw.astype(np.float32)).reshape(dims)

    def get(name: str) -> torch.Tensor:
        if name in aliases:
            src, dims = aliases[name]
            return values[src].reshape(dims)
        return values[name]

    for op in ops:
        if op[0] == "linear":
            y, x, w, b, relu = op[1], get(op[2]), get(op[3]), op[4], op[5] == "1"
            rows = x.reshape(-1, x.shape[-1])
            out = linear(rows, w, None if b == "-" else get(b))
            if relu:
                out = out.clamp_min(0.0)
            values[y] = out.half().float().reshape(tensors[y][1])
        elif op[0] == "sdpa":
            o, q, k, v, scale, causal = op[1], get(op[2]), get(op[3]), get(op[4]), float(op[5]), op[6] == "1"
            out = attention_prefill(q, k, v, k.shape[2], scale, causal)
            values[o] = out.half().float().reshape(tensors[o][1])
        else:
            raise ValueError(f"unknown op {op[0]}")
    return [values[name] for name in outs]
