"""Graph plans (llm_compiler_3_b200/graph.py, npu_b200_load_graph /
npu_b200_run_graph): a captured module as a sequence of library kernels.

The reference's own runs of these modules are the models: the MLP of
examples/pytorch/mlp.py (Linear -> ReLU -> Linear with biases, checked to 1 % of
the output peak, mlp.py:37-38,88) and the SDPA cases of
test/Integration/attention.py:28-33 (checked to 2e-2 against torch, 99-104,170).
On the CPU: the plan the emitter writes, the host-side checks of the C ABI, and
the oracle's interpretation of the plan against the module itself.  On the GPU:
the library running the plan against the oracle (max-abs 2e-2, cosine 0.9999)."""
import ctypes
import json

import pytest
import torch

import oracle
from conftest import seeded

ATOL = 2e-2
COS = 0.9999


class MLP(torch.nn.Module):
    def __init__(self, hidden, inner):
        super().__init__()
        self.up = torch.nn.Linear(hidden, inner)
        self.down = torch.nn.Linear(inner, hidden)

    def forward(self, x):
        return self.down(torch.relu(self.up(x)))


class SDPA(torch.nn.Module):
    def __init__(self, causal, gqa, scale=None):
        super().__init__()
        self.causal, self.gqa, self.scale = causal, gqa, scale

    def forward(self, q, k, v):
        return torch.nn.functional.scaled_dot_product_attention(
            q, k, v, is_causal=self.causal, enable_gqa=self.gqa, scale=self.scale)


class Flattened(torch.nn.Module):
    """Views on both sides of a linear layer, and no bias."""

    def __init__(self):
        super().__init__()
        self.proj = torch.nn.Linear(128, 96, bias=False)

    def forward(self, x):
        b, t, _ = x.shape
        return self.proj(x.reshape(b * t, 128)).view(b, t, 96)


def _mlp(hidden, inner, seed=0):
    torch.manual_seed(seed)
    return MLP(hidden, inner).to(torch.float16).eval()


# (hidden, inner, rows): the reference example's defaults and config 1 (batch 64)
MLP_CASES = [(64, 128, 32), (256, 512, 64), (256, 512, 300)]
# name, query heads, key/value heads, queries, keys, head size, causal
# (the reference's cases, test/Integration/attention.py:28-33) + a decode query
SDPA_CASES = [
    ("mha", 2, 2, 64, 128, 32, False),
    ("gqa", 8, 2, 64, 256, 64, False),
    ("causal", 4, 1, 128, 128, 64, True),
    ("gqa_causal_d128", 8, 2, 256, 256, 128, True),
    ("decode_gqa_d128", 32, 8, 1, 4096, 128, False),
]


def _sdpa_inputs(heads, kv_heads, queries, keys, dim, seed=1):
    return (seeded((1, heads, queries, dim), seed, 0.5), seeded((1, kv_heads, keys, dim), seed + 1, 0.5),
            seeded((1, kv_heads, keys, dim), seed + 2, 0.5))


def _check_info(directory):
    from llm_compiler_3_b200 import _native
    out = (ctypes.c_int64 * 6)()
    _native.check(_native.lib().npu_b200_graph_check(str(directory).encode(), out, 6))
    return list(out)


@pytest.mark.parametrize("hidden,inner,rows", MLP_CASES)
def test_mlp_plan(tmp_path, hidden, inner, rows):
    from llm_compiler_3_b200.graph import GraphPlan, capture_graph
    model = _mlp(hidden, inner)
    x = seeded((rows, hidden), 3, 0.5)
    path = capture_graph(model, (x,), tmp_path)
    plan = GraphPlan.parse(path.read_text())
    assert [op[0] for op in plan.ops] == ["linear", "linear"]
    assert plan.ops[0][5] is True and plan.ops[1][5] is False  # ReLU fused into the first
    args = (tmp_path / "arguments.txt").read_text().split("\n")
    assert args[0].split()[1] == "input0"
    assert [a.split()[1] for a in args[1:5]] == ["down.bias", "down.weight", "up.bias", "up.weight"]
    params = 2 * (2 * hidden * inner + hidden + inner)
    assert _check_info(tmp_path) == [1, 1, 2, params, 2 * rows * inner, 0]
    meta = json.loads((tmp_path / "metadata.json").read_text())
    assert meta["schema"] == "npu.b200.graph.v1" and meta["numerical_policy"] == "fp16"
    assert [a["index"] for a in meta["arguments"]] == list(range(5))
    assert meta["param_bytes"] == params and meta["outputs"][0]["shape"] == [rows, hidden]
    assert meta["ops"] == ["linear", "linear"]
    got = oracle.run_graph_plan(tmp_path, [x])[0]
    with torch.no_grad():
        want = model.float()(x.float())
    assert float((got - want).abs().max()) <= 0.01 * float(want.abs().max())


@pytest.mark.parametrize("case", SDPA_CASES, ids=[c[0] for c in SDPA_CASES])
def test_sdpa_plan(tmp_path, case):
    from llm_compiler_3_b200.graph import capture_graph
    _, heads, kv_heads, queries, keys, dim, causal = case
    q, k, v = _sdpa_inputs(heads, kv_heads, queries, keys, dim)
    capture_graph(SDPA(causal, heads != kv_heads), (q, k, v), tmp_path)
    decode = 1 if queries == 1 and not causal else 0
    assert _check_info(tmp_path) == [3, 1, 1, 0, 0, decode]
    got = oracle.run_graph_plan(tmp_path, [q, k, v])[0]
    want = torch.nn.functional.scaled_dot_product_attention(
        q.float(), k.float(), v.float(), is_causal=causal, enable_gqa=heads != kv_heads)
    assert float((got - want).abs().max()) <= ATOL


def test_views_and_scale(tmp_path):
    from llm_compiler_3_b200.graph import GraphPlan, capture_graph
    torch.manual_seed(5)
    model = Flattened().to(torch.float16).eval()
    x = seeded((2, 7, 128), 4, 0.5)
    path = capture_graph(model, (x,), tmp_path / "flat")
    plan = GraphPlan.parse(path.read_text())
    assert plan.ops[0][4] is None and plan.aliases  # no bias; x viewed as rows
    got = oracle.run_graph_plan(tmp_path / "flat", [x])[0]
    with torch.no_grad():
        want = model.float()(x.float())
    assert tuple(got.shape) == (14, 96)  # the linear writes the output; the view is free
    assert float((got.reshape(want.shape) - want).abs().max()) <= 2e-2
    q, k, v = _sdpa_inputs(4, 4, 8, 40, 64)
    path = capture_graph(SDPA(False, False, scale=0.05), (q, k, v), tmp_path / "scaled")
    assert GraphPlan.parse(path.read_text()).ops[0][5] == pytest.approx(0.05)


class MatmulParams(torch.nn.Module):
    """x @ W with W [K, N] parameters, one through addmm with a bias."""

    def __init__(self):
        super().__init__()
        g = torch.Generator().manual_seed(9)
        self.w1 = torch.nn.Parameter(torch.randn(64, 128, generator=g) / 8)
        self.w2 = torch.nn.Parameter(torch.randn(128, 64, generator=g) / 11)
        self.b = torch.nn.Parameter(torch.randn(64, generator=g) / 10)

    def forward(self, x):
        return torch.addmm(self.b, torch.relu(x @ self.w1), self.w2)


def test_matmul_weights_are_pretransposed(tmp_path):
    from llm_compiler_3_b200.graph import GraphPlan, capture_graph
    model = MatmulParams().half()
    x = seeded((32, 64), 6, 0.5)
    path = capture_graph(model, (x,), tmp_path)
    plan = GraphPlan.parse(path.read_text())
    assert [(op[0], op[5]) for op in plan.ops] == [("linear", True), ("linear", False)]
    assert plan.tensors["w1"][1] == (128, 64) and plan.tensors["w2"][1] == (64, 128)
    meta = json.loads((tmp_path / "metadata.json").read_text())
    assert meta["pretransposed"] == sorted([plan.tensors["w1"][2], plan.tensors["w2"][2]])
    got = oracle.run_graph_plan(tmp_path, [x])[0]
    with torch.no_grad():
        want = model.float()(x.float())
    assert float((got - want).abs().max()) <= 0.01 * float(want.abs().max())


class TwoHeads(torch.nn.Module):
    """Two outputs, returned in the opposite order of their computation."""

    def __init__(self):
        super().__init__()
        self.a = torch.nn.Linear(64, 32)
        self.b = torch.nn.Linear(64, 48)

    def forward(self, x):
        first = self.a(x)
        second = torch.relu(self.b(x))
        return second, first


class Reshaped(torch.nn.Module):
    """flatten / unsqueeze / squeeze around a linear layer, and eval-mode dropout."""

    def __init__(self):
        super().__init__()
        self.lin = torch.nn.Linear(64, 64)
        self.drop = torch.nn.Dropout(0.1)

    def forward(self, x):
        y = torch.flatten(x, 0, 1).unsqueeze(0).squeeze(0)
        return self.drop(self.lin(y)).unsqueeze(1).squeeze(1)


def test_layout_preserving_ops_are_aliases(tmp_path):
    from llm_compiler_3_b200.graph import GraphPlan, capture_graph
    torch.manual_seed(11)
    model = Reshaped().half().eval()
    x = seeded((2, 8, 64), 12, 0.5)
    path = capture_graph(model, (x,), tmp_path)
    plan = GraphPlan.parse(path.read_text())
    assert [op[0] for op in plan.ops] == ["linear"]
    got = oracle.run_graph_plan(tmp_path, [x])[0]
    with torch.no_grad():
        want = model.float()(x.float())
    assert float((got.reshape(want.shape) - want).abs().max()) <= 0.01 * float(want.abs().max())


def test_outputs_bind_in_return_order(tmp_path):
    from llm_compiler_3_b200.graph import GraphPlan, capture_graph
    torch.manual_seed(8)
    model = TwoHeads().half().eval()
    x = seeded((16, 64), 7, 0.5)
    path = capture_graph(model, (x,), tmp_path)
    plan = GraphPlan.parse(path.read_text())
    assert [plan.tensors[n][1] for n in plan.outputs] == [(16, 48), (16, 32)]
    assert _check_info(tmp_path)[:3] == [1, 2, 2]
    got = oracle.run_graph_plan(tmp_path, [x])
    with torch.no_grad():
        want = model.float()(x.float())
    for g, w in zip(got, want):
        assert float((g - w).abs().max()) <= 0.01 * float(w.abs().max())


def test_unsupported_modules_are_rejected(tmp_path):
    from llm_compiler_3_b200.graph import GraphUnsupported, capture_graph

    class Masked(torch.nn.Module):
        def forward(self, q, k, v, m):
            return torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=m)

    class Matmul(torch.nn.Module):
        def forward(self, a, b):
            return a @ b

    class LoneRelu(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = torch.nn.Linear(64, 64)

        def forward(self, x):
            y = self.lin(x)
            return torch.relu(y) + y

    q, k, v = _sdpa_inputs(2, 2, 4, 8, 64)
    with pytest.raises(GraphUnsupported, match="mask"):
        capture_graph(Masked(), (q, k, v, torch.zeros(4, 8, dtype=torch.float16)), tmp_path / "a")
    with pytest.raises(GraphUnsupported, match="2-D parameter"):
        capture_graph(Matmul(), (seeded((4, 64), 1), seeded((64, 8), 2)), tmp_path / "b")

    class Softmax(torch.nn.Module):
        def forward(self, x):
            return torch.softmax(x, dim=-1)

    with pytest.raises(GraphUnsupported, match="no kernel"):
        capture_graph(Softmax(), (seeded((4, 64), 1),), tmp_path / "d")
    with pytest.raises(GraphUnsupported):
        capture_graph(LoneRelu().half(), (seeded((4, 64), 1),), tmp_path / "c")

    # clone / contiguous become aliases: an output that is only a copy of an
    # input (or of another output) would share its bytes, so it is refused.
    class CloneOut(torch.nn.Module):
        def forward(self, x):
            return x.clone()

    class ContiguousTwice(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.lin = torch.nn.Linear(64, 64)

        def forward(self, x):
            y = self.lin(x)
            return y, y.contiguous()

    with pytest.raises(GraphUnsupported, match="not computed by an op"):
        capture_graph(CloneOut(), (seeded((4, 64), 1),), tmp_path / "e")
    with pytest.raises(GraphUnsupported, match="returned twice"):
        capture_graph(ContiguousTwice().half(), (seeded((4, 64), 1),), tmp_path / "f")


def test_check_command(tmp_path, capsys):
    from llm_compiler_3_b200.graph import capture_graph, main
    capture_graph(_mlp(64, 128), (seeded((8, 64), 3),), tmp_path)
    assert main([str(tmp_path)]) == 0
    assert "1 inputs, 1 outputs, 2 ops (linear, linear; 0 as flash-decoding)" in capsys.readouterr().out
    (tmp_path / "arg1.bin").unlink()
    assert main([str(tmp_path)]) == 1
    assert "invalid" in capsys.readouterr().out


def test_bad_plans_fail_on_the_host(tmp_path):
    from llm_compiler_3_b200 import _native
    from llm_compiler_3_b200.graph import capture_graph
    capture_graph(_mlp(64, 128), (seeded((8, 64), 3),), tmp_path)
    text = (tmp_path / "graph.txt").read_text()

    def check(new_text, match):
        (tmp_path / "graph.txt").write_text(new_text)
        with pytest.raises(_native.NpuError, match=match):
            _check_info(tmp_path)

    check(text.replace("npu.stage cuda-graph", "npu.stage cuda-plan"), "stage")
    check(text.replace("op linear linear_1", "op matmul linear_1"), "unknown op")
    check(text.replace("op linear linear x", "op linear linear linear_1"), "read before")
    check(text.replace("up.bias 1\n", "up.bias 7\n"), "relu 0\\|1")
    check(text.replace("npu.schema 1", "npu.schema 2"), "schema")
    check(text + "alias xv x 9x64\n", "tensors must precede the ops")
    lines = text.splitlines(keepends=True)
    ops_at = next(i for i, ln in enumerate(lines) if ln.startswith("op "))
    check("".join(lines[:ops_at]) + "alias xv x 9x64\n" + "".join(lines[ops_at:]),
          "element count")
    check("".join(lines[:ops_at]) + "tensor spare output f16 4x4\n" + "".join(lines[ops_at:]),
          "never written")
    check(text.replace("tensor linear temp f16 8x128", "tensor linear temp f16 8x64"),
          "not \\[rows, N\\]")
    # Dimensions must fit the kernels' int arguments (2^31 does not).
    check(text.replace("tensor linear temp f16 8x128", "tensor linear temp f16 8x2147483648"),
          "bad dimensions")
    # The projection's row limit (16384 tiles of 128 rows), checked at load:
    # a weight given as an input needs no parameter file of that size.
    head = "npu.stage cuda-graph\nnpu.schema 1\n"
    check(head + "tensor x input f16 8x64\ntensor w input f16 2097280x64\n"
          "tensor y output f16 8x2097280\nop linear y x w - 0\n", "2097152 rows")
    # The prefill grid: query blocks x head subgroups in one grid dimension.
    check(head + "tensor q input f16 1x1x8388736x32\ntensor k input f16 1x1x16x32\n"
          "tensor v input f16 1x1x16x32\ntensor o output f16 1x1x8388736x32\n"
          "op sdpa o q k v 0.17677669 1\n", "query blocks")
    (tmp_path / "graph.txt").unlink()
    with pytest.raises(_native.NpuError, match="cannot read"):
        _check_info(tmp_path)
    (tmp_path / "graph.txt").write_text(text)
    (tmp_path / "arg4.bin").write_bytes(b"\0" * 10)
    with pytest.raises(_native.NpuError, match="arg4.bin"):
        _check_info(tmp_path)


# --------------------------------------------------------------------------- GPU
def _run_twice(directory, inputs):
    from llm_compiler_3_b200 import _native
    from llm_compiler_3_b200.runtime import GraphRunner
    dev = torch.device("cuda", 0)
    with GraphRunner(directory) as g:
        dins = [t.to(dev) for t in inputs]
        first = [o.float().cpu() for o in g.run(*dins)]
        second = [o.float().cpu() for o in g.run(*dins)]
        torch.cuda.synchronize()
    assert _native.device_status() == 0
    for a, b in zip(first, second):
        assert torch.equal(a, b)
    return first


def _close(got, want):
    err = float((got - want).abs().max())
    assert err <= ATOL, f"max-abs {err}"
    assert oracle.cosine(got, want) >= COS


@pytest.mark.gpu
@pytest.mark.parametrize("hidden,inner,rows", MLP_CASES)
def test_mlp_runs(cuda, tmp_path, hidden, inner, rows):
    from llm_compiler_3_b200.graph import capture_graph
    x = seeded((rows, hidden), 3, 0.5)
    capture_graph(_mlp(hidden, inner), (x,), tmp_path)
    got = _run_twice(tmp_path, [x])[0]
    _close(got, oracle.run_graph_plan(tmp_path, [x])[0])


@pytest.mark.gpu
@pytest.mark.parametrize("case", SDPA_CASES, ids=[c[0] for c in SDPA_CASES])
def test_sdpa_runs(cuda, tmp_path, case):
    from llm_compiler_3_b200.graph import capture_graph
    _, heads, kv_heads, queries, keys, dim, causal = case
    q, k, v = _sdpa_inputs(heads, kv_heads, queries, keys, dim)
    capture_graph(SDPA(causal, heads != kv_heads), (q, k, v), tmp_path)
    got = _run_twice(tmp_path, [q, k, v])[0]
    _close(got, oracle.run_graph_plan(tmp_path, [q, k, v])[0])


@pytest.mark.gpu
def test_views_run(cuda, tmp_path):
    from llm_compiler_3_b200.graph import capture_graph
    torch.manual_seed(5)
    x = seeded((2, 7, 128), 4, 0.5)
    capture_graph(Flattened().to(torch.float16).eval(), (x,), tmp_path)
    got = _run_twice(tmp_path, [x])[0]
    _close(got, oracle.run_graph_plan(tmp_path, [x])[0])


@pytest.mark.gpu
def test_matmul_params_run(cuda, tmp_path):
    from llm_compiler_3_b200.graph import capture_graph
    x = seeded((32, 64), 6, 0.5)
    capture_graph(MatmulParams().half(), (x,), tmp_path)
    got = _run_twice(tmp_path, [x])[0]
    _close(got, oracle.run_graph_plan(tmp_path, [x])[0])


@pytest.mark.gpu
def test_layout_preserving_ops_run(cuda, tmp_path):
    from llm_compiler_3_b200.graph import capture_graph
    torch.manual_seed(11)
    x = seeded((2, 8, 64), 12, 0.5)
    capture_graph(Reshaped().half().eval(), (x,), tmp_path)
    got = _run_twice(tmp_path, [x])[0]
    _close(got, oracle.run_graph_plan(tmp_path, [x])[0])
