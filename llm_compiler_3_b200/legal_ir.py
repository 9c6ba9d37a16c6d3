"""Graph plans from the reference's MLIR text: the npu-emit-cuda step, without MLIR.

The reference's front end ends in a module of linalg on tensors: the capture's
``00-imported.mlir`` (torch-mlir's import, python/npu/capture/export.py:54-89)
and, after ``npu-attach-hardware`` and ``npu-legalize``, ``01-legal.mlir``
(tools/npu-compile/npu-compile.cpp:376-381).  Its NPU back end lowers that
module; for the B200 this module maps it onto the library's kernels and writes
a graph package that ``npu_b200_load_graph`` runs, as ``graph.py`` does from a
``torch.export`` graph.  It reads the MLIR text directly, so no MLIR build is
needed; only the subset of the printed form these modules use is parsed.

What is mapped (anything else is refused with ``GraphUnsupported`` naming the
op and the reason):

* ``linalg.matmul`` of an activation by a weight, accumulated from zero -- the
  form ``legalizeGraph`` requires (lib/Transforms/Legalize.cpp:136-161).  The
  weight is a parameter argument: listed in ``npu.pretransposed`` (the legalized
  module's record of pretransposeWeights, lib/Transforms/Normalize.cpp:670-701;
  its capture file keeps torch's [N, K] layout), the result of transposing a
  parameter (torch-mlir's linear), or a parameter stored [K, N] (flipped when
  the package is written).  A per-column add of a parameter vector and a ReLU
  (``arith.maximumf`` with zero, or torch-mlir's ``cmpf ugt`` + ``select``)
  that consume the product fuse into it, as normalizeGraph fuses them
  (Normalize.cpp:494-507).
* ``npu.attention`` in both printed forms: legalized, with ``group``, ``scale``,
  ``causal`` and ``key_transposed`` attributes (include/npu/Dialect/
  NPUDialect.td:31-61), and as imported, with the key/value repeat and the
  causal mask still spelled out, which are recognised the way
  canonicalizeAttention folds them (lib/Transforms/Attention.cpp:42-92,
  384-419).  The default scale is 1/sqrt(head size).
* ``tensor.collapse_shape`` / ``expand_shape``: row-major views, no kernel.

Arguments with an ``arg<N>.bin`` in the capture directory are parameters (the
capture writes files for parameters only, export.py:30-40); the others are the
run call's inputs, in argument order.  An argument listed in
``npu.pretransposed`` is read in its captured, untransposed layout: the
reference flips such arguments only when it writes its device image
(tools/npu-compile/npu-compile.cpp:621-625), which the B200 package does not
have.

    python -m llm_compiler_3_b200.legal_ir <module.mlir> [--capture DIR] --out DIR
"""
from __future__ import annotations

import json
import math
import re
import shutil
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from .graph import STAGE, GraphPlan, GraphUnsupported

_TENSOR = re.compile(r"tensor<([0-9x]*)x?(f16|f32|bf16|i1|i32|i64)>")


def _dims(type_text: str) -> tuple[int, ...]:
    """Shape of a ranked tensor type such as ``tensor<8x128x64xf16>``."""
    m = re.fullmatch(r"\s*tensor<((?:\d+x)*)(\w+)>\s*", type_text)
    if not m:
        raise GraphUnsupported(f"unsupported type {type_text.strip()!r}")
    if m.group(2) != "f16":
        raise GraphUnsupported(f"element type {m.group(2)}: graph plans compute in float16")
    return tuple(int(d) for d in m.group(1).split("x") if d)


def _strip_comments(text: str) -> str:
    out = []
    for line in text.splitlines():
        cut = line.find("//")
        out.append(line if cut < 0 else line[:cut])
    return "\n".join(out)


def _split_top(text: str, sep: str = ",") -> list[str]:
    """Split on `sep` outside (), [], {} and <>."""
    parts, depth, cur = [], 0, []
    for ch in text:
        if ch in "([{<":
            depth += 1
        elif ch in ")]}>":
            depth -= 1
        if ch == sep and depth == 0:
            parts.append("".join(cur))
            cur = []
        else:
            cur.append(ch)
    if "".join(cur).strip():
        parts.append("".join(cur))
    return [p.strip() for p in parts]


def _balanced(text: str, start: int, open_ch: str, close_ch: str) -> int:
    """Index just past the bracket that closes the one at `start`."""
    depth = 0
    for i in range(start, len(text)):
        if text[i] == open_ch:
            depth += 1
        elif text[i] == close_ch:
            depth -= 1
            if depth == 0:
                return i + 1
    raise GraphUnsupported(f"unbalanced {open_ch}{close_ch} in the module")


@dataclass
class Module:
    """The parsed parts of one module: attributes, the entry function's
    arguments and its statements (each one op, regions included)."""

    attrs: dict[str, str] = field(default_factory=dict)
    maps: dict[str, str] = field(default_factory=dict)
    args: list[tuple[str, tuple[int, ...]]] = field(default_factory=list)
    body: list[str] = field(default_factory=list)


# Stages npu-compile stamps on its stage files (tools/npu-compile/npu-compile.cpp:183):
# the B200 path reads a module up to "legal"; later ones are NPU back-end code.
_READABLE_STAGES = ("graph", "legal")


def parse_module(text: str) -> Module:
    text = _strip_comments(text)
    mod = Module()
    for m in re.finditer(r"^\s*#(\w+)\s*=\s*(affine_map<.*>)\s*$", text, re.M):
        mod.maps[m.group(1)] = m.group(2)
    m = re.search(r"module\s+attributes\s*\{", text)
    if m:
        end = _balanced(text, m.end() - 1, "{", "}")
        for item in _split_top(text[m.end():end - 1]):
            if "=" in item:
                key, value = item.split("=", 1)
                mod.attrs[key.strip().strip('"')] = value.strip()
    stage = mod.attrs.get("npu.stage", '"graph"').strip('"')
    if stage not in _READABLE_STAGES:
        raise GraphUnsupported(f'npu.stage = "{stage}" is NPU back-end code; the B200 path '
                               'reads the module as imported ("graph") or legalized ("legal")')
    m = re.search(r"func\.func\s+(?:\w+\s+)?@(\w+)\s*\(", text)
    if not m:
        raise GraphUnsupported("no func.func in the module")
    args_end = _balanced(text, m.end() - 1, "(", ")")
    for item in _split_top(text[m.end():args_end - 1]):
        am = re.match(r"(%[\w.]+)\s*:\s*(tensor<[^>]*>)", item)
        if not am:
            raise GraphUnsupported(f"unsupported function argument {item!r}")
        mod.args.append((am.group(1), _dims(am.group(2))))
    body_start = text.index("{", args_end)
    body_end = _balanced(text, body_start, "{", "}")
    body = text[body_start + 1:body_end - 1]
    # One statement per op: a line that starts a value definition, a quoted
    # generic op or a return begins a new statement once every bracket of the
    # previous one is closed.
    stmt, depth = [], 0
    for line in body.splitlines():
        s = line.strip()
        if not s:
            continue
        if depth == 0 and stmt and re.match(r'(%[\w.:#]+(\s*,\s*%[\w.:#]+)*\s*=|return\b|"|func\.return\b)', s):
            mod.body.append(" ".join(stmt))
            stmt = []
        stmt.append(s)
        depth += s.count("{") + s.count("(") + s.count("[") - s.count("}") - s.count(")") - s.count("]")
    if stmt:
        mod.body.append(" ".join(stmt))
    return mod


# --------------------------------------------------------------------------- values
@dataclass
class Value:
    kind: str                       # arg, param, const, empty, fill, tensor, repeat, mask, transposed
    dims: tuple[int, ...] = ()
    name: str = ""                  # plan tensor (arg, param, tensor)
    scalar: float = 0.0             # const, fill
    src: "Value | None" = None      # repeat, transposed
    group: int = 1                  # repeat
    index: int = -1                 # arg, param: the function argument


def _scalar(text: str) -> float:
    m = re.match(r"\s*(0x[0-9A-Fa-f]+|[-+]?[0-9.]+(?:e[-+]?\d+)?|true|false)\s*:\s*(\w+)", text)
    if not m:
        raise GraphUnsupported(f"unsupported constant {text.strip()!r}")
    lit, ty = m.group(1), m.group(2)
    if lit.startswith("0x"):
        bits = int(lit, 16)
        if ty == "f16":
            return float(np.array([bits], dtype=np.uint16).view(np.float16)[0])
        if ty == "f32":
            return float(np.array([bits], dtype=np.uint32).view(np.float32)[0])
        raise GraphUnsupported(f"hex constant of type {ty}")
    if lit in ("true", "false"):
        return 1.0 if lit == "true" else 0.0
    return float(lit)


def _operands(text: str) -> list[str]:
    return re.findall(r"%[\w.#]+", text)


def _section(stmt: str, word: str) -> str | None:
    """The text inside `word(...)` of a statement (ins / outs)."""
    m = re.search(r"\b" + word + r"\s*\(", stmt)
    if not m:
        return None
    end = _balanced(stmt, m.end() - 1, "(", ")")
    return stmt[m.end():end - 1]


class _Lowering:
    def __init__(self, mod: Module, params: set[int]):
        self.mod = mod
        self.plan = GraphPlan()
        self.values: dict[str, Value] = {}
        self.arg_index: dict[str, int] = {}
        self.flip: set[int] = set()           # parameter files stored [K, N]: write W^T
        self.linear_of: dict[str, int] = {}   # plan tensor -> index of the op writing it
        self.uses: dict[str, int] = {}
        pre = re.findall(r"\d+", mod.attrs.get("npu.pretransposed", ""))
        self.pretransposed = {int(p) for p in pre}
        if "npu.constants" in mod.attrs:
            raise GraphUnsupported("npu.constants: hoisted constant tensors have no slot in a "
                                   "graph plan")
        for i, (name, dims) in enumerate(mod.args):
            self.arg_index[name] = i
            if i in params:
                self.values[name] = Value("param", dims, name=f"arg{i}", index=i)
            else:
                self.values[name] = Value("arg", dims, name=f"input{i}", index=i)
                self.plan.tensors[f"input{i}"] = ("input", dims, None)
                self.plan.inputs.append(f"input{i}")
        for stmt in mod.body:
            for op in _operands(stmt.split("=", 1)[1] if re.match(r"%[\w.]+\s*=", stmt) else stmt):
                self.uses[op] = self.uses.get(op, 0) + 1

    # -- helpers ---------------------------------------------------------------
    def val(self, name: str) -> Value:
        if name not in self.values:
            raise GraphUnsupported(f"{name} is used before it is defined")
        return self.values[name]

    def tensor_name(self, v: Value, what: str) -> str:
        """The plan tensor of an activation operand (params are placed on use)."""
        if v.kind in ("arg", "tensor"):
            return v.name
        raise GraphUnsupported(f"{what}: operand is a {v.kind}, not an activation")

    def param(self, v: Value, dims: tuple[int, ...]) -> str:
        """Declare a parameter argument in the plan with `dims` (its file's layout)."""
        idx = int(v.name[3:])
        self.plan.tensors[v.name] = ("param", dims, idx)
        return v.name

    def view(self, name: str, src: Value, dims: tuple[int, ...]) -> None:
        if src.kind in ("repeat", "mask", "fill", "transposed"):
            self.values[name] = Value(src.kind, dims, name=src.name, scalar=src.scalar,
                                      src=src.src, group=src.group)
            return
        base = self.tensor_name(src, f"{name}: view")
        if math.prod(dims) != math.prod(src.dims):
            raise GraphUnsupported(f"{name}: view changes the element count")
        while base in self.plan.aliases:
            base = self.plan.aliases[base][0]
        alias = name.lstrip("%").replace(".", "_")
        self.plan.aliases[alias] = (base, dims)
        self.values[name] = Value("tensor", dims, name=alias, index=src.index)

    def new_temp(self, name: str, dims: tuple[int, ...]) -> str:
        t = name.lstrip("%").replace(".", "_")
        self.plan.tensors[t] = ("temp", dims, None)
        self.values[name] = Value("tensor", dims, name=t)
        return t

    # -- ops -------------------------------------------------------------------
    def run(self) -> GraphPlan:
        for stmt in self.mod.body:
            self.statement(stmt)
        if not self.plan.ops:
            raise GraphUnsupported("the function computes nothing the library runs")
        used = {o[2] for o in self.plan.ops if o[0] == "linear"} | \
            {o[3] for o in self.plan.ops if o[0] == "linear"} | \
            {o[4] for o in self.plan.ops if o[0] == "linear" and o[4]} | \
            {n for o in self.plan.ops if o[0] == "sdpa" for n in o[2:5]}
        self.plan.aliases = {k: v for k, v in self.plan.aliases.items() if k in used}
        return self.plan

    def statement(self, stmt: str) -> None:
        if stmt.startswith("return") or stmt.startswith("func.return"):
            return self.ret(stmt)
        m = re.match(r"(%[\w.]+)\s*=\s*(.*)$", stmt)
        if not m:
            raise GraphUnsupported(f"unsupported statement {stmt[:60]!r}")
        res, rhs = m.group(1), m.group(2)
        op = re.match(r'("?[\w.]+"?)', rhs).group(1).strip('"')
        handler = {
            "arith.constant": self.constant, "tensor.empty": self.empty,
            "linalg.fill": self.fill, "linalg.matmul": self.matmul,
            "linalg.generic": self.generic, "linalg.transpose": self.transpose,
            "tensor.collapse_shape": self.reshape, "tensor.expand_shape": self.reshape,
            "npu.attention": self.attention,
        }.get(op)
        if handler is None:
            raise GraphUnsupported(f"{res}: no kernel for {op}")
        handler(res, rhs)

    def result_dims(self, rhs: str) -> tuple[int, ...]:
        types = _TENSOR.findall(rhs.rsplit("->", 1)[-1]) if "->" in rhs else []
        if not types:
            types = _TENSOR.findall(rhs.rsplit(":", 1)[-1])
        if not types:
            raise GraphUnsupported(f"no result type in {rhs[:60]!r}")
        d, ty = types[-1]
        if ty != "f16":
            raise GraphUnsupported(f"result type {ty}: graph plans compute in float16")
        return tuple(int(x) for x in d.split("x") if x)

    def constant(self, res, rhs):
        body = rhs[len("arith.constant"):].strip()
        if body.startswith("dense"):
            raise GraphUnsupported(f"{res}: dense tensor constants have no slot in a graph plan")
        self.values[res] = Value("const", scalar=_scalar(body))

    def empty(self, res, rhs):
        self.values[res] = Value("empty", self.result_dims(rhs))

    def fill(self, res, rhs):
        c = self.val(_operands(_section(rhs, "ins"))[0])
        if c.kind != "const":
            raise GraphUnsupported(f"{res}: fill with a non-constant value")
        self.values[res] = Value("fill", self.result_dims(rhs), scalar=c.scalar)

    def reshape(self, res, rhs):
        src = self.val(_operands(rhs)[0])
        self.view(res, src, self.result_dims(rhs.split(" into ")[-1]))

    def transpose(self, res, rhs):
        src = self.val(_operands(_section(rhs, "ins"))[0])
        perm = re.search(r"permutation\s*=\s*\[([^\]]*)\]", rhs)
        if not perm or [int(p) for p in perm.group(1).split(",")] != [1, 0] or src.kind != "param":
            raise GraphUnsupported(f"{res}: only the 2-D transpose of a parameter is folded")
        self.values[res] = Value("transposed", self.result_dims(rhs), src=src)

    def weight(self, res: str, b: Value) -> tuple[str, int, int]:
        """(plan tensor, N, K) of a matmul's right operand B [K, N]."""
        k, n = b.dims
        if b.kind == "transposed":          # B = W^T, W [N, K] as captured
            return self.param(b.src, (n, k)), n, k
        if b.kind == "param":
            idx = int(b.name[3:])
            if idx not in self.pretransposed:  # stored [K, N]: flipped when written
                self.flip.add(idx)
            return self.param(b, (n, k)), n, k
        raise GraphUnsupported(f"{res}: linalg.matmul's right operand is an activation; the "
                               "library's projection multiplies activations by a weight")

    def matmul(self, res, rhs):
        a_name, b_name = _operands(_section(rhs, "ins"))[:2]
        init = self.val(_operands(_section(rhs, "outs"))[0])
        a, b = self.val(a_name), self.val(b_name)
        if len(a.dims) != 2 or len(b.dims) != 2:
            raise GraphUnsupported(f"{res}: only 2-D matmuls are mapped")
        x = self.tensor_name(a, f"{res}: matmul")
        w, n, k = self.weight(res, b)
        if k % 64 != 0:
            raise GraphUnsupported(f"{res}: K = {k} is not a multiple of 64")
        bias = None
        if init.kind == "fill" and init.scalar == 0.0:
            pass
        elif init.kind == "repeat" and init.src is not None and init.src.kind == "param" \
                and init.src.dims == (n,):
            bias = self.param(init.src, (n,))
        else:
            raise GraphUnsupported(f"{res}: the accumulator must start from zero (or the bias)")
        y = self.new_temp(res, self.result_dims(rhs))
        self.linear_of[y] = len(self.plan.ops)
        self.plan.ops.append(("linear", y, x, w, bias, False))

    def generic(self, res, rhs):
        head_end = _balanced(rhs, rhs.index("{"), "{", "}")
        head = rhs[rhs.index("{") + 1:head_end - 1]
        maps = re.search(r"indexing_maps\s*=\s*\[(.*?)\]\s*,\s*iterator_types", head)
        maps = [self.mod.maps.get(x.strip().lstrip("#"), x.strip())
                for x in _split_top(maps.group(1))] if maps else []
        iters = re.findall(r'"(\w+)"', head.split("iterator_types", 1)[-1])
        ins = _operands(_section(rhs, "ins") or "")
        region = rhs[rhs.index("{", head_end):]
        body_ops = re.findall(r"=\s*([\w.]+)", region) + (["linalg.yield"] if "linalg.yield" in region else [])
        dims = self.result_dims(rhs)
        if "reduction" in iters:
            raise GraphUnsupported(f"{res}: linalg.generic reduction ({', '.join(body_ops)}) has "
                                   "no kernel here")
        arith = [o for o in body_ops if o.startswith("arith.") or o.startswith("math.")]

        def affine(m):
            mm = re.search(r"\(([^)]*)\)\s*->\s*\(([^)]*)\)", m)
            return ([d.strip() for d in mm.group(1).split(",") if d.strip()],
                    [d.strip() for d in mm.group(2).split(",") if d.strip()]) if mm else ([], [])

        # Causal mask: no inputs, select(index_q >= index_k, 0, -inf).
        if not ins and "linalg.index" in body_ops and "arith.cmpi" in arith and \
                "arith.select" in arith and re.search(r"cmpi\s+sge", region):
            self.values[res] = Value("mask", dims)
            return
        if not arith and len(ins) == 1:
            src = self.val(ins[0])
            din, dout = affine(maps[0]) if maps else ([], [])
            if dout == din[::-1] and len(din) == 2 and src.kind == "param":
                self.values[res] = Value("transposed", dims, src=src)
                return
            if len(dout) < len(din):
                # Broadcast copy: GQA key/value repeat, or a bias vector
                # spread over rows for a matmul accumulator.
                group = math.prod(dims) // max(1, math.prod(src.dims))
                self.values[res] = Value("repeat", dims, src=src, group=group)
                return
        # Elementwise epilogues of a linear: bias add, ReLU.  The product is
        # the input that a linear op wrote and nothing else reads.
        lin = [o for o in ins if self.val(o).kind == "tensor" and
               self.val(o).name in self.linear_of and self.uses.get(o, 0) == 1]
        if lin:
            ins = lin + [o for o in ins if o != lin[0]]
        producer = self.val(ins[0]) if ins else None
        op_index = self.linear_of.get(producer.name) if lin else None
        if op_index is not None:
            op = list(self.plan.ops[op_index])
            relu = (arith == ["arith.maximumf"] and re.search(r"maximumf", region)) or \
                (sorted(arith) == ["arith.cmpf", "arith.select"] and re.search(r"cmpf\s+ugt", region))
            if relu and len(ins) == 1 and not op[5]:
                zero = [self.values.get(o) for o in _operands(region)]
                if any(z is not None and z.kind == "const" and z.scalar == 0.0 for z in zero):
                    op[5] = True
                    self.plan.ops[op_index] = tuple(op)
                    self.values[res] = self.values[ins[0]]
                    return
            if arith == ["arith.addf"] and len(ins) == 2 and op[4] is None and not op[5]:
                vec = self.val(ins[1])
                # The vector's indexing map must pick the column index alone.
                order = _operands(_section(rhs, "ins") or "")
                vmap = affine(maps[order.index(ins[1])]) if len(maps) > order.index(ins[1]) else ([], [])
                column = len(vmap[0]) == 2 and vmap[1] == [vmap[0][1]]
                if column and vec.kind == "param" and len(vec.dims) == 1 and \
                        vec.dims[0] == producer.dims[-1]:
                    op[4] = self.param(vec, vec.dims)
                    self.plan.ops[op_index] = tuple(op)
                    self.values[res] = self.values[ins[0]]
                    return
        raise GraphUnsupported(f"{res}: linalg.generic ({', '.join(arith) or 'copy'}) has no "
                               "kernel here")

    def attention(self, res, rhs):
        paren = rhs.index("(")
        ops = _operands(rhs[paren:_balanced(rhs, paren, "(", ")")])
        attrs = {}
        am = re.search(r"<\{(.*?)\}>", rhs)
        if am:
            for item in _split_top(am.group(1)):
                key, _, value = item.partition("=")
                attrs[key.strip()] = value.strip()
        vals = [self.val(o) for o in ops]
        init = vals[-1]
        if not (init.kind == "fill" and init.scalar == 0.0):
            raise GraphUnsupported(f"{res}: npu.attention's accumulator must start from zero")
        q, k, v = vals[0], vals[1], vals[2]
        causal = "causal" in attrs
        group = int(attrs["group"].split(":")[0]) if "group" in attrs else 1
        if len(vals) == 5:                 # as imported: mask operand, key/value repeated
            mask = vals[3]
            if mask.kind == "mask":
                causal = True
            elif not (mask.kind == "fill" and mask.scalar == 0.0):
                raise GraphUnsupported(f"{res}: npu.attention mask is neither causal nor absent")
        elif len(vals) != 4:
            raise GraphUnsupported(f"{res}: npu.attention with {len(vals)} operands")
        if k.kind == "repeat" and v.kind == "repeat" and k.group == v.group:
            group, k, v = k.group, k.src, v.src
        # Keys as K^T [Hk, D, N] (key_transposed): the transpose of a computed
        # key is folded; an argument listed in npu.pretransposed is supplied by
        # the caller in its untransposed layout [Hk, N, D].
        keys_last = False
        if "key_transposed" in attrs:
            if k.kind == "transposed":
                k = k.src
            elif k.kind in ("arg", "tensor") and k.index >= 0 and k.index in self.pretransposed:
                keys_last = True
            else:
                raise GraphUnsupported(f"{res}: transposed keys that are computed in the graph")
        heads, queries, dim = q.dims[-3:]
        kv_heads = heads // group
        keys = k.dims[-1] if keys_last else k.dims[-2]
        scale = float(attrs["scale"].split(":")[0]) if "scale" in attrs else 1.0 / math.sqrt(dim)
        qn = self.tensor_name(q, f"{res}: attention query")
        kn = self.tensor_name(k, f"{res}: attention key")
        vn = self.tensor_name(v, f"{res}: attention value")
        names = []
        for nm, val, shape in ((qn, q, (1, heads, queries, dim)),
                               (kn, k, (1, kv_heads, keys, dim)),
                               (vn, v, (1, kv_heads, keys, dim))):
            if math.prod(val.dims) != math.prod(shape):
                raise GraphUnsupported(f"{res}: attention operand {nm} is not {shape}")
            alias = f"{nm}_4d"
            base = nm
            while base in self.plan.aliases:
                base = self.plan.aliases[base][0]
            self.plan.aliases[alias] = (base, shape)
            names.append(alias)
        out = self.new_temp(res + "_4d", (1, heads, queries, dim))
        self.plan.ops.append(("sdpa", out, names[0], names[1], names[2], scale, causal))
        self.plan.aliases[res.lstrip("%").replace(".", "_")] = (out, self.result_dims(rhs))
        self.values[res] = Value("tensor", self.result_dims(rhs),
                                 name=res.lstrip("%").replace(".", "_"))

    def ret(self, stmt):
        names = _operands(stmt.split(":")[0])
        for r in names:
            v = self.val(r)
            if v.kind != "tensor":
                raise GraphUnsupported(f"output {r} is not computed by an op")
            base = v.name
            while base in self.plan.aliases:
                base = self.plan.aliases[base][0]
            role, dims, _ = self.plan.tensors[base]
            if role == "output":
                raise GraphUnsupported(f"output {r} is returned twice")
            self.plan.tensors[base] = ("output", dims, None)
            self.plan.outputs.append(base)


def plan_from_mlir(text: str, params: set[int] | None = None) -> tuple[GraphPlan, set[int]]:
    """Map a module onto the library's ops.  `params`: argument indices that are
    parameters (besides those in npu.pretransposed).  Returns the plan and the
    parameter indices whose capture file must be written transposed."""
    low = _Lowering(parse_module(text), params or set())
    plan = low.run()
    plan.pretransposed = {f"arg{i}" for i in low.flip}
    return plan, low.flip


def write_package(mlir_path: str | Path, out_dir: str | Path,
                  capture_dir: str | Path | None = None) -> Path:
    """Write a graph package (graph.txt, arguments.txt, arg<N>.bin,
    metadata.json) for `mlir_path`, taking parameter files from the capture
    directory.  Returns graph.txt's path."""
    mlir_path, out_dir = Path(mlir_path), Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    cap = Path(capture_dir) if capture_dir else None
    params = set()
    if cap is not None:
        params = {int(p.stem[3:]) for p in cap.glob("arg*.bin") if p.stem[3:].isdigit()}
    plan, flip = plan_from_mlir(mlir_path.read_text(), params)
    mod = parse_module(mlir_path.read_text())
    arguments = []
    for i, (name, dims) in enumerate(mod.args):
        tname = f"arg{i}"
        role = "param" if tname in plan.tensors and plan.tensors[tname][0] == "param" else "input"
        arguments.append({"index": i, "name": f"input{i}" if role == "input" else tname,
                          "role": role, "shape": list(dims), "dtype": "float16",
                          "bytes": 2 * math.prod(dims)})
        if role != "param":
            continue
        src = cap / f"arg{i}.bin" if cap is not None else None
        if src is None or not src.exists():
            raise GraphUnsupported(f"parameter argument {i} has no arg{i}.bin")
        if i in flip:  # stored [K, N] in the capture: the linear kernel reads [N, K]
            k, n = dims
            data = np.fromfile(src, dtype="<f2").reshape(k, n).T.copy()
            (out_dir / f"arg{i}.bin").write_bytes(data.tobytes())
        elif src.resolve() != (out_dir / f"arg{i}.bin").resolve():
            shutil.copyfile(src, out_dir / f"arg{i}.bin")
    lines = [f"{a['index']} {a['name']} {'x'.join(map(str, a['shape']))} float16"
             for a in arguments]
    (out_dir / "arguments.txt").write_text("\n".join(lines) + "\n")
    ordered = {n: plan.tensors[n] for n in plan.inputs + plan.outputs}
    ordered.update({n: v for n, v in plan.tensors.items() if n not in ordered})
    plan.tensors = ordered
    path = out_dir / "graph.txt"
    path.write_text(plan.text())
    metadata = {
        "schema": "npu.b200.graph.v1", "stage": STAGE, "numerical_policy": "fp16",
        "source": mlir_path.name, "arguments": arguments,
        "outputs": [{"name": n, "shape": list(plan.tensors[n][1]), "dtype": "float16"}
                    for n in plan.outputs],
        "ops": [op[0] for op in plan.ops],
        "pretransposed": sorted(flip),
        "param_bytes": sum(a["bytes"] for a in arguments if a["role"] == "param"),
        "temp_bytes": sum(2 * math.prod(d) for r, d, _ in plan.tensors.values() if r == "temp"),
    }
    (out_dir / "metadata.json").write_text(json.dumps(metadata, indent=2) + "\n")
    return path


def main(argv=None) -> int:
    """``python -m llm_compiler_3_b200.legal_ir <module.mlir> --out DIR``: write
    the graph package of a module and check it with the library's loader."""
    import argparse
    from .graph import main as check
    ap = argparse.ArgumentParser(description=main.__doc__.splitlines()[0])
    ap.add_argument("module", type=Path)
    ap.add_argument("--capture", type=Path, default=None,
                    help="capture directory with the parameters' arg<N>.bin")
    ap.add_argument("--out", type=Path, required=True)
    a = ap.parse_args(argv)
    try:
        write_package(a.module, a.out, a.capture)
    except GraphUnsupported as err:
        print(f"unsupported: {err}")
        return 1
    return check([str(a.out)])


if __name__ == "__main__":
    raise SystemExit(main())
