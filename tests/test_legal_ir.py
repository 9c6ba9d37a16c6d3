"""Graph packages from the reference's MLIR text (llm_compiler_3_b200/legal_ir.py).

The reference's own MLIR fixtures (test/Integration/*.mlir and
test/Tools/npu-opt/*.mlir, read in place when the reference tree is present)
must each either become a package that the library's loader accepts
(npu_b200_graph_check) or be refused with a named reason.  The legalized forms
are checked on modules written here in the printed form the reference's lit
checks show (test/Tools/npu-opt/attention.mlir, LEGAL lines: npu.pretransposed,
npu.attention with group / scale / causal / key_transposed).  On the GPU the
packages run against the oracle: the MLP of examples/pytorch/mlp.py at batch 64
(the plumbing config) and SDPA with GQA and a causal mask."""
import ctypes
import math
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from conftest import seeded

REFERENCE = Path("/root/reference")
ATOL, COS = 2e-2, 0.9999

MAPS = """#map = affine_map<(d0, d1) -> (d0, d1)>
#map1 = affine_map<(d0, d1) -> (d1)>
"""

# examples/pytorch/mlp.py's module (up: Linear(256, 512), ReLU, down: Linear(512, 256))
# captured at batch 64 and legalized: arguments are the input, then parameters
# sorted by name (down.bias, down.weight, up.bias, up.weight); both weights are
# pretransposed ([in, out]) and the ReLU is a maximumf with zero.
MLP_LEGAL = MAPS + """module attributes {npu.pretransposed = array<i64: 2, 4>, npu.schema = 1 : i64, npu.stage = "legal"} {
  func.func @main(%arg0: tensor<64x256xf16>, %arg1: tensor<256xf16>, %arg2: tensor<512x256xf16>, %arg3: tensor<512xf16>, %arg4: tensor<256x512xf16>) -> tensor<64x256xf16> {
    %cst = arith.constant 0.000000e+00 : f16
    %0 = tensor.empty() : tensor<64x512xf16>
    %1 = linalg.fill ins(%cst : f16) outs(%0 : tensor<64x512xf16>) -> tensor<64x512xf16>
    %2 = linalg.matmul ins(%arg0, %arg4 : tensor<64x256xf16>, tensor<256x512xf16>) outs(%1 : tensor<64x512xf16>) -> tensor<64x512xf16>
    %3 = linalg.generic {indexing_maps = [#map, #map1, #map], iterator_types = ["parallel", "parallel"]} ins(%2, %arg3 : tensor<64x512xf16>, tensor<512xf16>) outs(%0 : tensor<64x512xf16>) {
    ^bb0(%in: f16, %in_0: f16, %out: f16):
      %10 = arith.addf %in, %in_0 : f16
      linalg.yield %10 : f16
    } -> tensor<64x512xf16>
    %4 = linalg.generic {indexing_maps = [#map, #map], iterator_types = ["parallel", "parallel"]} ins(%3 : tensor<64x512xf16>) outs(%0 : tensor<64x512xf16>) {
    ^bb0(%in: f16, %out: f16):
      %10 = arith.maximumf %in, %cst : f16
      linalg.yield %10 : f16
    } -> tensor<64x512xf16>
    %5 = tensor.empty() : tensor<64x256xf16>
    %6 = linalg.fill ins(%cst : f16) outs(%5 : tensor<64x256xf16>) -> tensor<64x256xf16>
    %7 = linalg.matmul ins(%4, %arg2 : tensor<64x512xf16>, tensor<512x256xf16>) outs(%6 : tensor<64x256xf16>) -> tensor<64x256xf16>
    %8 = linalg.generic {indexing_maps = [#map, #map1, #map], iterator_types = ["parallel", "parallel"]} ins(%7, %arg1 : tensor<64x256xf16>, tensor<256xf16>) outs(%5 : tensor<64x256xf16>) {
    ^bb0(%in: f16, %in_0: f16, %out: f16):
      %10 = arith.addf %in, %in_0 : f16
      linalg.yield %10 : f16
    } -> tensor<64x256xf16>
    return %8 : tensor<64x256xf16>
  }
}
"""

# The same module as imported: each weight transposed in the graph, the ReLU
# as torch-mlir spells it (cmpf ugt + select).
MLP_IMPORTED = MAPS + """#map2 = affine_map<(d0, d1) -> (d1, d0)>
module {
  func.func @main(%arg0: tensor<64x256xf16>, %arg1: tensor<256xf16>, %arg2: tensor<256x512xf16>, %arg3: tensor<512xf16>, %arg4: tensor<512x256xf16>) -> tensor<64x256xf16> {
    %cst = arith.constant 0.000000e+00 : f16
    %0 = tensor.empty() : tensor<256x512xf16>
    %1 = linalg.generic {indexing_maps = [#map2, #map], iterator_types = ["parallel", "parallel"]} ins(%arg4 : tensor<512x256xf16>) outs(%0 : tensor<256x512xf16>) {
    ^bb0(%in: f16, %out: f16):
      linalg.yield %in : f16
    } -> tensor<256x512xf16>
    %2 = tensor.empty() : tensor<64x512xf16>
    %3 = linalg.fill ins(%cst : f16) outs(%2 : tensor<64x512xf16>) -> tensor<64x512xf16>
    %4 = linalg.matmul ins(%arg0, %1 : tensor<64x256xf16>, tensor<256x512xf16>) outs(%3 : tensor<64x512xf16>) -> tensor<64x512xf16>
    %5 = linalg.generic {indexing_maps = [#map, #map1, #map], iterator_types = ["parallel", "parallel"]} ins(%4, %arg3 : tensor<64x512xf16>, tensor<512xf16>) outs(%2 : tensor<64x512xf16>) {
    ^bb0(%in: f16, %in_0: f16, %out: f16):
      %14 = arith.addf %in, %in_0 : f16
      linalg.yield %14 : f16
    } -> tensor<64x512xf16>
    %6 = linalg.generic {indexing_maps = [#map, #map], iterator_types = ["parallel", "parallel"]} ins(%5 : tensor<64x512xf16>) outs(%2 : tensor<64x512xf16>) {
    ^bb0(%in: f16, %out: f16):
      %14 = arith.cmpf ugt, %in, %cst : f16
      %15 = arith.select %14, %in, %cst : f16
      linalg.yield %15 : f16
    } -> tensor<64x512xf16>
    %7 = tensor.empty() : tensor<512x256xf16>
    %8 = linalg.transpose ins(%arg2 : tensor<256x512xf16>) outs(%7 : tensor<512x256xf16>) permutation = [1, 0]
    %9 = tensor.empty() : tensor<64x256xf16>
    %10 = linalg.fill ins(%cst : f16) outs(%9 : tensor<64x256xf16>) -> tensor<64x256xf16>
    %11 = linalg.matmul ins(%6, %8 : tensor<64x512xf16>, tensor<512x256xf16>) outs(%10 : tensor<64x256xf16>) -> tensor<64x256xf16>
    %12 = linalg.generic {indexing_maps = [#map, #map1, #map], iterator_types = ["parallel", "parallel"]} ins(%11, %arg1 : tensor<64x256xf16>, tensor<256xf16>) outs(%9 : tensor<64x256xf16>) {
    ^bb0(%in: f16, %in_0: f16, %out: f16):
      %14 = arith.addf %in, %in_0 : f16
      linalg.yield %14 : f16
    } -> tensor<64x256xf16>
    return %12 : tensor<64x256xf16>
  }
}
"""

# SDPA(q, k, v, is_causal=True, enable_gqa=True), 8 query / 2 key-value heads,
# 128 positions, head size 64, legalized: the key argument is asked for
# transposed (npu.pretransposed), npu.attention carries the group, the scale,
# causal and key_transposed (the LEGAL lines of test/Tools/npu-opt/attention.mlir).
SDPA_LEGAL = """module attributes {npu.pretransposed = array<i64: 1>, npu.schema = 1 : i64, npu.stage = "legal"} {
  func.func @main(%arg0: tensor<1x8x128x64xf16>, %arg1: tensor<1x2x64x128xf16>, %arg2: tensor<1x2x128x64xf16>) -> tensor<1x8x128x64xf16> {
    %cst = arith.constant 0.000000e+00 : f16
    %collapsed = tensor.collapse_shape %arg0 [[0, 1], [2], [3]] : tensor<1x8x128x64xf16> into tensor<8x128x64xf16>
    %collapsed_0 = tensor.collapse_shape %arg1 [[0, 1], [2], [3]] : tensor<1x2x64x128xf16> into tensor<2x64x128xf16>
    %collapsed_1 = tensor.collapse_shape %arg2 [[0, 1], [2], [3]] : tensor<1x2x128x64xf16> into tensor<2x128x64xf16>
    %0 = tensor.empty() : tensor<8x128x64xf16>
    %1 = linalg.fill ins(%cst : f16) outs(%0 : tensor<8x128x64xf16>) -> tensor<8x128x64xf16>
    %2 = "npu.attention"(%collapsed, %collapsed_0, %collapsed_1, %1) <{causal, group = 4 : i64, key_transposed, scale = 1.250000e-01 : f64}> : (tensor<8x128x64xf16>, tensor<2x64x128xf16>, tensor<2x128x64xf16>, tensor<8x128x64xf16>) -> tensor<8x128x64xf16>
    %expanded = tensor.expand_shape %2 [[0, 1], [2], [3]] output_shape [1, 8, 128, 64] : tensor<8x128x64xf16> into tensor<1x8x128x64xf16>
    return %expanded : tensor<1x8x128x64xf16>
  }
}
"""


def _mlp_params(seed=0):
    """The MLP's parameters in the capture's order (index -> tensor, torch layout)."""
    torch.manual_seed(seed)
    up, down = torch.nn.Linear(256, 512), torch.nn.Linear(512, 256)
    return {1: down.bias.half(), 2: down.weight.half(), 3: up.bias.half(), 4: up.weight.half()}


def _capture(tmp: Path, params: dict[int, torch.Tensor], transpose=()):
    """arg<N>.bin files as the capture writes them (export.py:30-40); indices in
    `transpose` hold W^T, the layout of a matmul by a [K, N] parameter."""
    tmp.mkdir(parents=True, exist_ok=True)
    for i, t in params.items():
        data = t.detach().t().contiguous() if i in transpose else t.detach()
        (tmp / f"arg{i}.bin").write_bytes(data.numpy().astype("<f2").tobytes())
    return tmp


def _graph_check(directory):
    from llm_compiler_3_b200 import _native
    out = (ctypes.c_int64 * 6)()
    _native.check(_native.lib().npu_b200_graph_check(str(directory).encode(), out, 6))
    return list(out)


def _write(tmp, name, text):
    path = tmp / name
    path.write_text(text)
    return path


# --------------------------------------------------------------------------- CPU
@pytest.mark.parametrize("text", [MLP_LEGAL, MLP_IMPORTED], ids=["legal", "imported"])
def test_mlp_module_becomes_two_linears(tmp_path, text):
    from llm_compiler_3_b200.graph import GraphPlan
    from llm_compiler_3_b200.legal_ir import write_package
    cap = _capture(tmp_path / "cap", _mlp_params())
    write_package(_write(tmp_path, "m.mlir", text), tmp_path / "pkg", cap)
    plan = GraphPlan.parse((tmp_path / "pkg" / "graph.txt").read_text())
    assert [op[0] for op in plan.ops] == ["linear", "linear"]
    first, second = plan.ops
    assert first[2] == "input0" and first[3] == "arg4" and first[4] == "arg3" and first[5]
    assert second[3] == "arg2" and second[4] == "arg1" and not second[5]
    assert plan.tensors["arg4"] == ("param", (512, 256), 4)   # torch's [out, in]: no flip
    assert plan.outputs == [second[1]]
    inputs, outputs, ops, param_bytes, _, _ = _graph_check(tmp_path / "pkg")
    assert (inputs, outputs, ops) == (1, 1, 2)
    assert param_bytes == 2 * (256 + 512 * 256 + 512 + 256 * 512)


def test_legal_attention_folds_group_scale_and_causal(tmp_path):
    from llm_compiler_3_b200.graph import GraphPlan
    from llm_compiler_3_b200.legal_ir import write_package
    write_package(_write(tmp_path, "a.mlir", SDPA_LEGAL), tmp_path / "pkg")
    plan = GraphPlan.parse((tmp_path / "pkg" / "graph.txt").read_text())
    (op,) = plan.ops
    assert op[0] == "sdpa" and op[5] == 0.125 and op[6] is True
    assert plan.aliases[op[2]][1] == (1, 8, 128, 64)
    assert plan.aliases[op[3]] == ("input1", (1, 2, 128, 64))   # keys read untransposed
    assert plan.inputs == ["input0", "input1", "input2"]
    assert _graph_check(tmp_path / "pkg")[:3] == [3, 1, 1]


def test_matmul_by_a_kn_parameter_is_flipped(tmp_path):
    """x @ B with B a parameter stored [K, N]: the package holds B^T, recorded
    under pretransposed in metadata.json."""
    import json
    from llm_compiler_3_b200.legal_ir import write_package
    text = """func.func @main(%a: tensor<64x128xf16>, %b: tensor<128x192xf16>) -> tensor<64x192xf16> {
  %zero = arith.constant 0.0 : f16
  %empty = tensor.empty() : tensor<64x192xf16>
  %init = linalg.fill ins(%zero : f16) outs(%empty : tensor<64x192xf16>) -> tensor<64x192xf16>
  %out = linalg.matmul ins(%a, %b : tensor<64x128xf16>, tensor<128x192xf16>)
                       outs(%init : tensor<64x192xf16>) -> tensor<64x192xf16>
  return %out : tensor<64x192xf16>
}
"""
    b = seeded((128, 192), 3)
    cap = _capture(tmp_path / "cap", {1: b})
    write_package(_write(tmp_path, "mm.mlir", text), tmp_path / "pkg", cap)
    stored = np.fromfile(tmp_path / "pkg" / "arg1.bin", dtype="<f2").reshape(192, 128)
    assert np.array_equal(stored, b.t().numpy())
    assert json.loads((tmp_path / "pkg" / "metadata.json").read_text())["pretransposed"] == [1]
    assert _graph_check(tmp_path / "pkg")[:3] == [1, 1, 1]


@pytest.mark.parametrize("snippet,reason", [
    ('module attributes {npu.stage = "target"} {\n}', "NPU back-end code"),
    ("""func.func @main(%a: tensor<64x64xf16>, %b: tensor<64x64xf16>) -> tensor<64x64xf16> {
  %zero = arith.constant 0.0 : f16
  %e = tensor.empty() : tensor<64x64xf16>
  %i = linalg.fill ins(%zero : f16) outs(%e : tensor<64x64xf16>) -> tensor<64x64xf16>
  %m = linalg.matmul ins(%a, %b : tensor<64x64xf16>, tensor<64x64xf16>) outs(%i : tensor<64x64xf16>) -> tensor<64x64xf16>
  return %m : tensor<64x64xf16>
}""", "right operand is an activation"),
    ("""func.func @main(%a: tensor<4x64xf16>) -> tensor<4x64xf16> {
  %two = arith.constant dense<2.0> : tensor<4x64xf16>
  return %a : tensor<4x64xf16>
}""", "dense tensor constants"),
    ("""func.func @main(%a: tensor<4x64xf16>) -> tensor<4x64xf16> {
  %e = tensor.empty() : tensor<4x64xf16>
  %r = linalg.generic {indexing_maps = [affine_map<(i, j) -> (i, j)>, affine_map<(i, j) -> (i, j)>], iterator_types = ["parallel", "parallel"]} ins(%a : tensor<4x64xf16>) outs(%e : tensor<4x64xf16>) {
  ^bb0(%x: f16, %o: f16):
    %s = arith.mulf %x, %x : f16
    linalg.yield %s : f16
  } -> tensor<4x64xf16>
  return %r : tensor<4x64xf16>
}""", "arith.mulf"),
])
def test_refusals_name_their_reason(snippet, reason):
    from llm_compiler_3_b200.graph import GraphUnsupported
    from llm_compiler_3_b200.legal_ir import plan_from_mlir
    with pytest.raises(GraphUnsupported, match=reason):
        plan_from_mlir(snippet)


def _reference_fixtures():
    dirs = [REFERENCE / "test" / "Integration", REFERENCE / "test" / "Tools" / "npu-opt"]
    return sorted(p for d in dirs if d.is_dir() for p in d.glob("*.mlir"))


@pytest.mark.skipif(not REFERENCE.is_dir(), reason="the reference tree is not on this machine")
def test_reference_fixtures_accepted_or_refused_by_name(tmp_path):
    """Every MLIR fixture of the reference: a package the loader accepts, or a
    refusal naming the op or stage.  The 2-D matmul graphs are read with their
    right operand as a parameter (a weight), so that those whose K is a multiple
    of 64 become linear layers; the SDPA capture becomes one attention op."""
    from llm_compiler_3_b200.graph import GraphPlan, GraphUnsupported
    from llm_compiler_3_b200.legal_ir import parse_module, write_package
    fixtures = _reference_fixtures()
    assert fixtures, "no fixtures found"
    accepted = {}
    for path in fixtures:
        out = tmp_path / path.stem
        cap = None
        try:
            mod = parse_module(path.read_text())
            if len(mod.args) == 2 and "linalg.matmul" in path.read_text():
                cap = _capture(tmp_path / (path.stem + "_cap"),
                               {1: seeded(mod.args[1][1], 5, 0.1)})
            write_package(path, out, cap)
        except GraphUnsupported as err:
            assert str(err), path.name
            continue
        _graph_check(out)
        accepted[path.name] = GraphPlan.parse((out / "graph.txt").read_text())
    sdpa = accepted["sdpa-gqa-causal-graph.mlir"]
    (op,) = sdpa.ops
    assert op[0] == "sdpa" and op[6] is True and math.isclose(op[5], 0.125)
    assert sdpa.aliases[op[3]][1] == (1, 2, 128, 64)   # group 4: 8 query heads over 2
    for name in ("matmul64-graph.mlir", "pipeline-graph.mlir", "hierarchical-graph.mlir"):
        assert [o[0] for o in accepted[name].ops] == ["linear"], name
    assert "decoder-layer.mlir" not in accepted and "passes.mlir" not in accepted


def test_command_line(tmp_path, capsys):
    from llm_compiler_3_b200.legal_ir import main
    cap = _capture(tmp_path / "cap", _mlp_params())
    assert main([str(_write(tmp_path, "m.mlir", MLP_LEGAL)), "--capture", str(cap),
                 "--out", str(tmp_path / "pkg")]) == 0
    assert "2 ops (linear, linear" in capsys.readouterr().out
    assert main([str(_write(tmp_path, "t.mlir", 'module attributes {npu.stage = "hw"} {\n}')),
                 "--out", str(tmp_path / "pkg2")]) == 1
    assert "unsupported" in capsys.readouterr().out


# --------------------------------------------------------------------------- GPU
def _run(directory, inputs):
    from llm_compiler_3_b200 import _native
    from llm_compiler_3_b200.runtime import GraphRunner
    dev = torch.device("cuda", 0)
    with GraphRunner(directory) as g:
        out = [o.float().cpu() for o in g.run(*[t.to(dev) for t in inputs])]
    assert _native.device_status() == 0
    return out


def _close(got, want):
    err = float((got - want).abs().max())
    assert err <= ATOL and oracle.cosine(got, want) >= COS, f"max-abs {err}"


@pytest.mark.gpu
@pytest.mark.parametrize("text", [MLP_LEGAL, MLP_IMPORTED], ids=["legal", "imported"])
def test_mlp_package_runs(cuda, tmp_path, text):
    """The MLP config (batch 64, 256 -> 512 -> 256) from its MLIR module against
    the oracle's MLP (examples/pytorch/mlp.py:44-51)."""
    from llm_compiler_3_b200.legal_ir import write_package
    params = _mlp_params(3)
    cap = _capture(tmp_path / "cap", params)
    write_package(_write(tmp_path, "m.mlir", text), tmp_path / "pkg", cap)
    x = seeded((64, 256), 4)
    (got,) = _run(tmp_path / "pkg", [x])
    want = oracle.mlp_forward(x, params[4], params[3], params[2], params[1])
    _close(got, want)


@pytest.mark.gpu
def test_legal_attention_package_runs(cuda, tmp_path):
    from llm_compiler_3_b200.legal_ir import write_package
    write_package(_write(tmp_path, "a.mlir", SDPA_LEGAL), tmp_path / "pkg")
    q = seeded((1, 8, 128, 64), 7, 0.5)
    k = seeded((1, 2, 128, 64), 8, 0.5)
    v = seeded((1, 2, 128, 64), 9, 0.5)
    (got,) = _run(tmp_path / "pkg", [q, k, v])
    want = oracle.attention_prefill(q, k, v, 128, 0.125, causal=True)
    _close(got, want)
