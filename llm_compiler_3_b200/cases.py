"""Fixed workloads for profiling and timing one kernel or one decode step.

Each case builds seeded synthetic inputs on cuda:0, runs the library's own
entry point `--repeat` times and prints one line with the mean time of the
launches after the first (CUDA events).  Under ncu, capture with `-s 1` or
more to skip the cold first launch.

    python -m llm_compiler_3_b200.cases proj --rows 4096 --k 14336 --batch 1
    python -m llm_compiler_3_b200.cases flash --batch 64 --seq 4096
    python -m llm_compiler_3_b200.cases prefill --queries 4096 --sdpa
    python -m llm_compiler_3_b200.cases step --batch 1 --layers 32 --seq 4096
"""
from __future__ import annotations

import argparse
import sys


def _timed(fn, repeat: int, graph: bool = False) -> float:
    """Mean microseconds per call after a first untimed call; with `graph`,
    the calls are captured once into a CUDA graph and the replay is timed
    (no host launch cost between kernels)."""
    import torch
    fn()
    torch.cuda.synchronize()
    n = max(1, repeat - 1)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if graph:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(n):
                fn()
        g.replay()
        torch.cuda.synchronize()
        start.record()
        g.replay()
        end.record()
    else:
        start.record()
        for _ in range(n):
            fn()
        end.record()
    torch.cuda.synchronize()
    return start.elapsed_time(end) * 1e3 / n


def case_proj(a) -> str:
    """One packed projection (STORE, FP32 out): the GEMV at batch 1-2, the
    tensor-core kernel above."""
    import torch
    from . import _native, ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    ws = [ops.pack_weight((torch.randn(a.rows, a.k, device=dev, generator=g) * 0.02).half())
          for _ in range(max(1, a.copies))]
    x = torch.randn(a.batch, a.k, device=dev, generator=g).half()
    out = torch.empty(a.batch, a.rows, device=dev, dtype=torch.float32)
    e = _native.Epilogue(kind=_native.EPI_STORE, ld_out=a.rows, out_f32=1)
    e.out = out.data_ptr()
    turn = [0]

    def call():  # successive launches read successive weight copies
        ops.projection(x, ws[turn[0] % len(ws)], a.rows, e, packed=True)
        turn[0] += 1

    us = _timed(call, a.repeat, a.graph)
    gbs = a.rows * a.k * 2 / us / 1e3
    return (f"proj rows={a.rows} k={a.k} batch={a.batch} copies={len(ws)}: {us:.1f} us/launch, "
            f"{gbs:.0f} GB/s weights")


def case_flash(a) -> str:
    """Flash-decoding over a full cache of `seq` keys for every sequence."""
    import torch
    from . import ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    q = torch.randn(a.batch, a.q_heads, 128, device=dev, generator=g).half()
    k = torch.randn(a.batch, a.kv_heads, a.seq, 128, device=dev, generator=g).half()
    v = torch.randn(a.batch, a.kv_heads, a.seq, 128, device=dev, generator=g).half()
    lens = torch.full((a.batch,), a.seq, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    us = _timed(lambda: ops.flash_decode(q, k, v, lens, out=out), a.repeat, a.graph)
    gbs = 2 * a.batch * a.kv_heads * a.seq * 128 * 2 / us / 1e3
    return f"flash batch={a.batch} seq={a.seq}: {us:.1f} us/launch, {gbs:.0f} GB/s K+V"


def case_prefill(a) -> str:
    """Causal attention of a `queries`-token prompt appended after `prefix` cached
    tokens (every sequence alike), head size 128; FLOPs count visible keys only.
    With --sdpa (prefix 0) also times torch's SDPA on the same tensors."""
    import torch
    from . import ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    keys = a.prefix + a.queries
    q = torch.randn(a.batch, a.q_heads, a.queries, 128, device=dev, generator=g).half()
    k = torch.randn(a.batch, a.kv_heads, keys, 128, device=dev, generator=g).half()
    v = torch.randn(a.batch, a.kv_heads, keys, 128, device=dev, generator=g).half()
    start = torch.full((a.batch,), a.prefix, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    us = _timed(lambda: ops.prefill_attention(q, k, v, keys=keys, q_start=start, causal=True,
                                              out=out), a.repeat, a.graph)
    visible = sum(min(a.prefix + i + 1, keys) for i in range(a.queries))
    flops = 4.0 * 128 * visible * a.batch * a.q_heads
    line = (f"prefill batch={a.batch} queries={a.queries} prefix={a.prefix}: {us:.1f} us/launch, "
            f"{flops / us / 1e6:.0f} TFLOP/s")
    if a.sdpa and a.prefix == 0:
        f = torch.nn.functional.scaled_dot_product_attention
        ref = _timed(lambda: f(q, k, v, is_causal=True, enable_gqa=True), a.repeat, a.graph)
        line += f"; torch SDPA {ref:.1f} us/launch, {flops / ref / 1e6:.0f} TFLOP/s"
    return line


def case_step(a) -> str:
    """Greedy decode steps of the Llama-3-8B-shaped stack (random weights,
    cache filled to seq - 1, position seq - 1), one CUDA graph per step."""
    import torch
    from . import _native
    from .plan import llama3_8b
    from .runtime import Decoder
    from .plan import DecodePlan
    # --shard N: one tensor-parallel rank's share of a TP=N run (its heads, FFN
    # columns and vocabulary rows) as a one-GPU plan -- the same kernels at the
    # same shapes, without the exchanges.
    n = a.shard
    H, V, F = 4096, -(-128256 // n), 14336 // n
    Q, KV = 32 // n, 8 // n
    dev = torch.device("cuda", 0)
    plan = llama3_8b(layers=a.layers, max_batch=a.batch, max_seq=a.seq) if n == 1 else \
        DecodePlan(arch="llama", hidden=H, heads=Q, kv_heads=KV, head_dim=128, ffn=F,
                   layers=a.layers, vocab=V, rms_eps=1e-5, rope_theta=500000.0,
                   max_batch=a.batch, max_seq=a.seq)
    dec = Decoder(plan, device=0)
    gen = torch.Generator(device=dev)

    def randn(shape, seed, std=0.02):
        gen.manual_seed(seed)
        return (torch.randn(shape, device=dev, generator=gen) * std).half()

    dec.set_weight("model.embed_tokens.weight", randn((V, H), 11))
    dec.set_weight("lm_head.weight", randn((V, H), 12))
    ones = torch.ones(H, dtype=torch.float16, device=dev)
    dec.set_weight("model.norm.weight", ones)
    shapes = {"self_attn.q_proj.weight": (Q * 128, H), "self_attn.k_proj.weight": (KV * 128, H),
              "self_attn.v_proj.weight": (KV * 128, H), "self_attn.o_proj.weight": (H, Q * 128),
              "mlp.gate_proj.weight": (F, H), "mlp.up_proj.weight": (F, H),
              "mlp.down_proj.weight": (H, F)}
    for layer in range(a.layers):
        for j, (name, shape) in enumerate(shapes.items()):
            dec.set_weight(f"model.layers.{layer}.{name}", randn(shape, 1000 + 16 * layer + j))
        dec.set_weight(f"model.layers.{layer}.input_layernorm.weight", ones)
        dec.set_weight(f"model.layers.{layer}.post_attention_layernorm.weight", ones)
        k, v = dec.kv_cache(layer)
        gen.manual_seed(50000 + layer)
        k[:, :, :a.seq - 1].normal_(generator=gen)
        v[:, :, :a.seq - 1].normal_(generator=gen)
    tok = torch.randint(0, V, (a.batch,), device=dev, dtype=torch.int32,
                        generator=torch.Generator(device=dev).manual_seed(7))
    pos = torch.full((a.batch,), a.seq - 1, dtype=torch.int32, device=dev)
    ids = torch.empty(a.batch, dtype=torch.int32, device=dev)
    us = _timed(lambda: dec.step_device(tok, pos, ids), a.repeat)
    status = _native.device_status()
    dec.close()
    return (f"step batch={a.batch} layers={a.layers} seq={a.seq} shard=1/{n}: "
            f"{us / 1e3:.3f} ms/step, device status {status}")


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    sub = ap.add_subparsers(dest="case", required=True)
    p = sub.add_parser("proj")
    p.add_argument("--rows", type=int, default=4096)
    p.add_argument("--k", type=int, default=4096)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--repeat", type=int, default=4)
    p.add_argument("--graph", action="store_true", help="time graph replays of the launches")
    p.add_argument("--copies", type=int, default=1,
                   help="weight copies read in turn (more than L2 holds: cold weights)")
    f = sub.add_parser("flash")
    f.add_argument("--batch", type=int, default=64)
    f.add_argument("--q-heads", type=int, default=32)
    f.add_argument("--kv-heads", type=int, default=8)
    f.add_argument("--seq", type=int, default=4096)
    f.add_argument("--repeat", type=int, default=3)
    f.add_argument("--graph", action="store_true", help="time graph replays of the launches")
    r = sub.add_parser("prefill")
    r.add_argument("--batch", type=int, default=1)
    r.add_argument("--q-heads", type=int, default=32)
    r.add_argument("--kv-heads", type=int, default=8)
    r.add_argument("--queries", type=int, default=4096)
    r.add_argument("--prefix", type=int, default=0)
    r.add_argument("--repeat", type=int, default=5)
    r.add_argument("--graph", action="store_true", help="time graph replays of the launches")
    r.add_argument("--sdpa", action="store_true", help="also time torch SDPA (prefix 0)")
    s = sub.add_parser("step")
    s.add_argument("--batch", type=int, default=1)
    s.add_argument("--layers", type=int, default=32)
    s.add_argument("--seq", type=int, default=4096)
    s.add_argument("--repeat", type=int, default=5)
    s.add_argument("--shard", type=int, default=1, choices=[1, 2, 4, 8],
                   help="one rank's share of tensor parallel over N GPUs, run alone")
    a = ap.parse_args(argv)
    cases = {"proj": case_proj, "flash": case_flash, "prefill": case_prefill, "step": case_step}
    print(cases[a.case](a), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
