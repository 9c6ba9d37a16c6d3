"""Graph plans: a captured module as a sequence of library kernels.

The reference turns a captured module into a compiled program through MLIR
(python/npu/capture/export.py:108-139 capture, then npu-compile's stages) and
runs it on the NPU simulator with the captured arguments.  Its B200 target
replaces everything after the front end with ``npu_b200_run_graph`` over a plan
(the scope of ``npu-emit-cuda``).  This module writes that plan straight from a
``torch.export`` of the module -- the same graph the reference imports through
torch-mlir -- for graphs built from the ops the library has kernels for:

* ``aten.linear`` (+ bias, + a ReLU that is its only user, fused as the
  reference's normalizeGraph fuses maximumf into the matmul epilogue,
  lib/Transforms/Normalize.cpp:494-507): the tcgen05 linear kernel, 128 rows per
  launch;
* ``aten.matmul`` / ``aten.mm`` / ``aten.addmm`` by a 2-D parameter W [K, N]
  that nothing else reads: the same linear kernel, with W stored transposed
  ([N, K]) in its arg<N>.bin and listed under ``pretransposed`` in metadata.json
  -- the flip the reference's normalizeGraph records for its image builder
  (pretransposeWeights, lib/Transforms/Normalize.cpp:670-701), in the other
  direction, once at capture time;
* ``aten.scaled_dot_product_attention`` (no mask, no dropout, causal or not, GQA,
  any scale) -- npu.attention after canonicalizeAttention
  (lib/Transforms/Attention.cpp:384-419): the flash-decoding kernel for one
  query per head without a causal mask, the prefill attention kernel otherwise;
* views and copies that keep the row-major layout (``view``, ``reshape``,
  ``flatten``, ``squeeze``, ``unsqueeze``, ``contiguous``, ``clone``) and
  dropout in eval mode: aliases, no kernel.

Decoder layers and stacks (RMSNorm, RoPE, SwiGLU, KV cache) run through the
decode plan (``plan.py``, ``runtime.Decoder``) instead.

The capture directory keeps the reference's format (``arguments.txt`` plus
little-endian ``arg<N>.bin``, activations first, then parameters and buffers
sorted by name, export.py:30-40, 117-119, 133-138) and adds ``metadata.json``
(the package's ABI description, as npu-compile writes one beside its program,
tools/npu-compile/npu-compile.cpp:479-507, lib/Transforms/Emit.cpp:1424-1430)
and ``graph.txt``:

    npu.stage cuda-graph
    npu.schema 1
    tensor <name> input|output|param|temp f16 <d0>x<d1>... [arg <N>]
    alias <name> <source> <d0>x<d1>...
    op linear <y> <x> <w> <bias|-> <relu 0|1>
    op sdpa <out> <q> <k> <v> <scale> <causal 0|1>

Inputs bind to the run call's argument pointers and outputs to its output
pointers, each in the order of their lines.
"""
from __future__ import annotations

import json
import math
import operator
from dataclasses import dataclass, field
from pathlib import Path
from typing import Sequence

import torch

STAGE = "cuda-graph"
SCHEMA = 1

# Ops that become aliases of their source (no kernel, no copy).  clone and
# contiguous are among them: this is sound only because no op of a plan writes
# its operands in place and an output must be computed by an op (an alias of
# an input, or of another output, is refused when the outputs are bound), so an
# alias never shares bytes with a tensor that is written after it is read.
_VIEWS = {"aten.view.default", "aten.reshape.default", "aten.contiguous.default",
          "aten.clone.default", "aten._unsafe_view.default", "aten.alias.default",
          "aten.flatten.using_ints", "aten.unsqueeze.default", "aten.squeeze.dim",
          "aten.squeeze.dims", "aten.squeeze.default"}


class GraphUnsupported(ValueError):
    """The module uses an op or a layout the graph plan has no kernel for."""


@dataclass
class GraphPlan:
    """The parsed content of a graph.txt (what the runtime executes)."""

    tensors: dict[str, tuple[str, tuple[int, ...], int | None]] = field(default_factory=dict)
    aliases: dict[str, tuple[str, tuple[int, ...]]] = field(default_factory=dict)
    ops: list[tuple] = field(default_factory=list)
    inputs: list[str] = field(default_factory=list)
    outputs: list[str] = field(default_factory=list)
    pretransposed: set[str] = field(default_factory=set)  # parameters stored as W^T

    def text(self) -> str:
        lines = [f"npu.stage {STAGE}", f"npu.schema {SCHEMA}"]
        for name, (role, dims, arg) in self.tensors.items():
            line = f"tensor {name} {role} f16 {'x'.join(map(str, dims))}"
            if arg is not None:
                line += f" arg {arg}"
            lines.append(line)
        for name, (src, dims) in self.aliases.items():
            lines.append(f"alias {name} {src} {'x'.join(map(str, dims))}")
        for op in self.ops:
            if op[0] == "linear":
                _, y, x, w, b, relu = op
                lines.append(f"op linear {y} {x} {w} {b or '-'} {int(relu)}")
            else:
                _, o, q, k, v, scale, causal = op
                lines.append(f"op sdpa {o} {q} {k} {v} {scale!r} {int(causal)}")
        return "\n".join(lines) + "\n"

    @classmethod
    def parse(cls, text: str) -> "GraphPlan":
        plan = cls()
        for raw in text.splitlines():
            f = raw.split()
            if not f or f[0].startswith("#") or f[0].startswith("npu."):
                continue
            if f[0] == "tensor":
                arg = int(f[6]) if len(f) > 6 and f[5] == "arg" else None
                plan.tensors[f[1]] = (f[2], tuple(int(d) for d in f[4].split("x")), arg)
                if f[2] == "input":
                    plan.inputs.append(f[1])
                elif f[2] == "output":
                    plan.outputs.append(f[1])
            elif f[0] == "alias":
                plan.aliases[f[1]] = (f[2], tuple(int(d) for d in f[3].split("x")))
            elif f[0] == "op" and f[1] == "linear":
                plan.ops.append(("linear", f[2], f[3], f[4], None if f[5] == "-" else f[5],
                                 f[6] == "1"))
            elif f[0] == "op" and f[1] == "sdpa":
                plan.ops.append(("sdpa", f[2], f[3], f[4], f[5], float(f[6]), f[7] == "1"))
            else:
                raise ValueError(f"graph.txt: unknown line {raw!r}")
        return plan


def _shape(node) -> tuple[int, ...]:
    val = node.meta.get("val")
    if not isinstance(val, torch.Tensor):
        raise GraphUnsupported(f"{node.name}: no tensor value")
    if val.dtype != torch.float16:
        raise GraphUnsupported(f"{node.name} is {val.dtype}; graph plans compute in float16")
    return tuple(int(d) for d in val.shape)


def build_graph_plan(exported) -> tuple[GraphPlan, list[str], dict[str, torch.Tensor]]:
    """Map an ExportedProgram onto library ops.  Returns the plan, the user
    input names in order and the parameter tensors by their capture names."""
    sig = exported.graph_signature
    plan = GraphPlan()
    state = dict(exported.state_dict)
    state.update(getattr(exported, "constants", {}) or {})
    params: dict[str, torch.Tensor] = {}
    user_inputs: list[str] = []
    placeholder_target: dict[str, str] = {}
    for spec in sig.input_specs:
        if spec.kind.name == "USER_INPUT":
            user_inputs.append(spec.arg.name)
        else:
            placeholder_target[spec.arg.name] = spec.target
    graph = exported.graph_module.graph
    nodes = list(graph.nodes)
    name_of: dict[str, str] = {}  # fx node -> plan tensor (through aliases)
    fused_relu: set[str] = set()
    pretransposed: set[str] = set()

    def emit_linear(node, x, w, b, weight_kn: bool):
        users = list(node.users)
        relu = len(users) == 1 and str(users[0].target) == "aten.relu.default"
        if relu:
            fused_relu.add(users[0].name)
        wn = name_of[w.name]
        if plan.tensors.get(wn, ("",))[0] != "param" or len(_shape(w)) != 2:
            raise GraphUnsupported(f"{node.name}: the weight must be a 2-D parameter")
        if weight_kn:  # x @ W with W [K, N]: store W^T, the linear kernel's [N, K]
            if len(w.users) != 1 or wn in pretransposed:
                raise GraphUnsupported(f"{node.name}: a matmul weight must have no other reader")
            k, n = _shape(w)
            params[wn] = params[wn].t().contiguous()
            plan.tensors[wn] = ("param", (n, k), None)
            pretransposed.add(wn)
        out = users[0] if relu else node
        plan.tensors[node.name] = ("temp", _shape(out), None)
        name_of[node.name] = node.name
        plan.ops.append(("linear", node.name, name_of[x.name], wn,
                         name_of[b.name] if b is not None else None, relu))

    for node in nodes:
        if node.op == "placeholder":
            dims = _shape(node)
            if node.name in placeholder_target:
                target = placeholder_target[node.name]
                tensor = state[target]
                params[target] = tensor
                plan.tensors[target] = ("param", dims, None)
                name_of[node.name] = target
            else:
                plan.tensors[node.name] = ("input", dims, None)
                plan.inputs.append(node.name)
                name_of[node.name] = node.name
        elif node.op == "call_function":
            target = str(node.target)
            if target in _VIEWS:
                src = name_of[node.args[0].name]
                src = plan.aliases[src][0] if src in plan.aliases else src  # base tensor
                plan.aliases[node.name] = (src, _shape(node))
                name_of[node.name] = node.name
            elif target == "aten.dropout.default":
                train = node.args[2] if len(node.args) > 2 else node.kwargs.get("train", False)
                if train:
                    raise GraphUnsupported(f"{node.name}: dropout in training mode")
                src = name_of[node.args[0].name]
                src = plan.aliases[src][0] if src in plan.aliases else src
                plan.aliases[node.name] = (src, _shape(node))
                name_of[node.name] = node.name
            elif target == "aten.relu.default":
                src = node.args[0]
                if node.name not in fused_relu:
                    raise GraphUnsupported(f"{node.name}: ReLU that does not follow a linear "
                                           "with it as the only user")
                name_of[node.name] = name_of[src.name]
            elif target == "aten.linear.default":
                b = node.args[2] if len(node.args) > 2 else None
                emit_linear(node, node.args[0], node.args[1], b, weight_kn=False)
            elif target in ("aten.matmul.default", "aten.mm.default"):
                emit_linear(node, node.args[0], node.args[1], None, weight_kn=True)
            elif target == "aten.addmm.default":
                beta = node.kwargs.get("beta", 1)
                alpha = node.kwargs.get("alpha", 1)
                bias = node.args[0]
                if beta != 1 or alpha != 1 or len(_shape(bias)) != 1:
                    raise GraphUnsupported(f"{node.name}: addmm needs a [N] bias, beta = alpha = 1")
                emit_linear(node, node.args[1], node.args[2], bias, weight_kn=True)
            elif target == "aten.scaled_dot_product_attention.default":
                a = list(node.args) + [None] * 6
                q, k, v = a[0], a[1], a[2]
                mask = node.kwargs.get("attn_mask", a[3])
                dropout = node.kwargs.get("dropout_p", a[4] if a[4] is not None else 0.0)
                causal = bool(node.kwargs.get("is_causal", a[5] if a[5] is not None else False))
                scale = node.kwargs.get("scale", a[6] if len(node.args) > 6 else None)
                if mask is not None:
                    raise GraphUnsupported(f"{node.name}: attention masks are not supported "
                                           "(use is_causal)")
                if dropout:
                    raise GraphUnsupported(f"{node.name}: dropout is not supported")
                qd, kd = _shape(q), _shape(k)
                if len(qd) != 4 or len(kd) != 4:
                    raise GraphUnsupported(f"{node.name}: q, k, v must be [B, H, L, D]")
                if scale is None:
                    scale = 1.0 / math.sqrt(qd[3])
                plan.tensors[node.name] = ("temp", _shape(node), None)
                name_of[node.name] = node.name
                plan.ops.append(("sdpa", node.name, name_of[q.name], name_of[k.name],
                                 name_of[v.name], float(scale), causal))
            elif target == str(operator.getitem):
                raise GraphUnsupported(f"{node.name}: multi-output ops are not supported")
            else:
                raise GraphUnsupported(f"{node.name}: no kernel for {target}")
        elif node.op == "output":
            outs = node.args[0]
            outs = outs if isinstance(outs, (tuple, list)) else (outs,)
            for out in outs:
                name = name_of[out.name]
                dims = _shape(out)
                while name in plan.aliases:  # the op that produces it writes the output
                    name = plan.aliases[name][0]
                role, base_dims, _ = plan.tensors[name]
                if role == "output":
                    raise GraphUnsupported(f"output {out.name} is returned twice")
                if role != "temp":
                    raise GraphUnsupported(f"output {out.name} is not computed by an op")
                if math.prod(base_dims) != math.prod(dims):
                    raise GraphUnsupported(f"output {out.name} changes size through a view")
                plan.tensors[name] = ("output", base_dims, None)
                plan.outputs.append(name)
    # Drop aliases nothing reads (e.g. the view in front of an output).
    used = {o[2] for o in plan.ops if o[0] == "linear"} | {o[3] for o in plan.ops if o[0] == "linear"}
    used |= {o[4] for o in plan.ops if o[0] == "linear" and o[4]}
    used |= {n for o in plan.ops if o[0] == "sdpa" for n in o[2:5]}
    plan.aliases = {k: v for k, v in plan.aliases.items() if k in used}
    plan.pretransposed = pretransposed
    return plan, user_inputs, params


def _dtype_name(t: torch.Tensor) -> str:
    return str(t.dtype).removeprefix("torch.")


def capture_graph(module: torch.nn.Module, example: Sequence[torch.Tensor],
                  directory: str | Path) -> Path:
    """Export `module` at the example's (fixed) shapes, map it onto library ops
    and write the capture directory plus graph.txt.  Returns graph.txt's path."""
    directory = Path(directory)
    directory.mkdir(parents=True, exist_ok=True)
    exported = torch.export.export(module, tuple(example), strict=False)
    plan, user_inputs, params = build_graph_plan(exported)
    lines = []
    for i, tensor in enumerate(example):
        lines.append(f"{i} input{i} {'x'.join(map(str, tensor.shape))} {_dtype_name(tensor)}")
    for j, name in enumerate(sorted(params), start=len(example)):
        tensor = params[name].detach().contiguous().cpu()
        if tensor.dtype != torch.float16:
            raise GraphUnsupported(f"parameter {name} is {tensor.dtype}; expected float16")
        lines.append(f"{j} {name} {'x'.join(map(str, tensor.shape))} {_dtype_name(tensor)}")
        (directory / f"arg{j}.bin").write_bytes(tensor.numpy().astype("<f2").tobytes())
        role, dims, _ = plan.tensors[name]
        plan.tensors[name] = (role, dims, j)
    (directory / "arguments.txt").write_text("\n".join(lines) + "\n")
    # Inputs bind in the module's argument order, outputs in its return order.
    rank = {n: i for i, n in enumerate(user_inputs)}
    plan.inputs.sort(key=lambda n: rank[n])
    ordered = {n: plan.tensors[n] for n in plan.inputs + plan.outputs}
    ordered.update({n: v for n, v in plan.tensors.items() if n not in ordered})
    plan.tensors = ordered
    path = directory / "graph.txt"
    path.write_text(plan.text())
    arguments = [{"index": i, "name": f"input{i}", "role": "input", "shape": list(t.shape),
                  "dtype": _dtype_name(t), "bytes": t.numel() * t.element_size()}
                 for i, t in enumerate(example)]
    for name, (role, dims, arg) in plan.tensors.items():
        if role == "param":
            arguments.append({"index": arg, "name": name, "role": "param", "shape": list(dims),
                              "dtype": "float16", "bytes": 2 * math.prod(dims)})
    arguments.sort(key=lambda a: a["index"])
    metadata = {
        "schema": "npu.b200.graph.v1", "stage": STAGE, "numerical_policy": "fp16",
        "arguments": arguments,
        "outputs": [{"name": n, "shape": list(plan.tensors[n][1]), "dtype": "float16"}
                    for n in plan.outputs],
        "ops": [op[0] for op in plan.ops],
        "pretransposed": sorted(plan.tensors[n][2] for n in plan.pretransposed),
        "param_bytes": sum(a["bytes"] for a in arguments if a["role"] == "param"),
        "temp_bytes": sum(2 * math.prod(d) for r, d, _ in plan.tensors.values() if r == "temp"),
    }
    (directory / "metadata.json").write_text(json.dumps(metadata, indent=2) + "\n")
    return path


def main(argv=None) -> int:
    """``python -m llm_compiler_3_b200.graph <dir>``: check a graph package on
    the host with the library's own loader checks (no GPU) and summarise it."""
    import argparse
    import ctypes

    from . import _native
    ap = argparse.ArgumentParser(description=main.__doc__.splitlines()[0])
    ap.add_argument("directory", type=Path)
    a = ap.parse_args(argv)
    out = (ctypes.c_int64 * 6)()
    try:
        _native.check(_native.lib().npu_b200_graph_check(str(a.directory).encode(), out, 6))
    except _native.NpuError as err:
        print(f"invalid: {err}")
        return 1
    plan = GraphPlan.parse((a.directory / "graph.txt").read_text())
    inputs, outputs, ops, param_bytes, temp_bytes, decode = list(out)
    print(f"{a.directory}: {inputs} inputs, {outputs} outputs, {ops} ops "
          f"({', '.join(op[0] for op in plan.ops)}; {decode} as flash-decoding), "
          f"{param_bytes} parameter bytes, {temp_bytes} temporary bytes")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
