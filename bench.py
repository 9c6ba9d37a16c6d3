#!/usr/bin/env python
"""Decode throughput of the Llama-3-8B-shaped FP16 stack on B200 (libnpu_b200).

Workload (N GPUs, tensor parallel): 32 decoder layers (hidden 4096, 32/8 heads of
128, SwiGLU 14336, RMSNorm eps 1e-5, RoPE theta 5e5), final norm, LM head
4096x128256 and greedy argmax; batch 64 sequences, each at position 4095 over a
4095-token FP16 KV cache (4096 keys attended).  Weights are random-init FP16
N(0, 0.02) and the cache N(0, 1), generated on the device (synthetic data of the
config's shapes; nothing is downloaded).  One step reads ~49.4 GB, far more than
the 126 MB L2, so no flush is needed between steps.

    python bench.py [--gpus N --steps K --warmup W]          # libnpu_b200
    python bench.py --impl reference [--steps K --warmup W]  # CPU oracle arm

Multi-GPU: launched by torchrun, one process per GPU; NCCL communicators come
from torch.distributed (unique id broadcast) and the library's own all-reduces.
Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "decode tokens/s (Llama-3-8B shape, FP16) & % of HBM roofline"
HIDDEN, HEADS, KV_HEADS, HEAD_DIM, FFN, VOCAB = 4096, 32, 8, 128, 14336, 128256
FALLBACK_HBM_GBS = 6650.0


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--seq", type=int, default=4096, help="keys attended (position + 1)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the single-GPU attention and layer configs")
    a = ap.parse_args(argv)
    if a.warmup < 3:
        ap.error("--warmup must be >= 3")
    return a


def step_bytes(batch, layers, seq, tp=1):
    """Algorithmic HBM bytes of one decode step, whole job (FP16 weights and
    every valid KV entry read once; the new K/V entries and outputs written once)."""
    per_layer_w = (HEADS + 2 * KV_HEADS) * HEAD_DIM * HIDDEN + HIDDEN * HEADS * HEAD_DIM \
        + 3 * FFN * HIDDEN + 2 * HIDDEN
    kv = 2 * batch * KV_HEADS * (seq - 1) * HEAD_DIM
    kv_new = 2 * batch * KV_HEADS * HEAD_DIM
    acts = 2 * batch * HIDDEN  # layer input read / output written (FP16 equivalent)
    top = VOCAB * HIDDEN + HIDDEN + batch * HIDDEN  # LM head, final norm, embedding rows
    return 2 * (layers * (per_layer_w + kv + kv_new + acts) + top)


def attention_bytes(batch, kv_heads, q_heads, seq):
    """Algorithmic bytes of one flash-decoding launch: K and V of every attended
    key, the queries read and the outputs written (FP16)."""
    return 2 * (2 * batch * kv_heads * seq * HEAD_DIM + 2 * batch * q_heads * HEAD_DIM)


def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic():
    """DRAM bytes per flash-decoding launch from the committed ncu summary, if any."""
    path = ROOT / "profiles" / "flash_decode_b64_kv4096.md"
    try:
        for line in path.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":")[1].strip())
    except Exception:
        pass
    return None


class ClockSampler:
    """nvidia-smi samples of this GPU's clocks and throttle reasons while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.file = None

    def start(self):
        if not self.uuid:
            return
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.uuid}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "20"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.file.flush()
        rows = [r.split(",") for r in Path(self.file.name).read_text().splitlines() if r.strip()]
        os.unlink(self.file.name)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[0]))
                mx.append(float(r[1]))
                for name, flag in zip(names, r[4:8]):
                    if flag.strip().lower() == "active":
                        reasons.add(name)
            except (ValueError, IndexError):
                continue
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "samples": len(sm),
                "reasons": sorted(reasons)}


def host_cpu_model() -> str:
    """The host CPU's model name (first entry of /proc/cpuinfo), or the platform's."""
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or platform.machine()


class CpuOracleStep:
    """The oracle (PyTorch on the host CPU, FP16 storage, FP32 compute) running
    whole decode steps of the stack: the embedding rows, every one of the
    `layers` decoder layers with its K/V append at the position, the final norm,
    the LM head and the greedy argmax.  One layer's weights and cache are built
    once and serve every layer (each layer reads ~1.5 GB, far more than the
    host's caches hold, so reuse saves memory, not time); the embedding rows are
    read from the LM-head table (tied embeddings)."""

    def __init__(self, batch, layers, seq):
        import torch
        import oracle
        self.torch, self.oracle = torch, oracle
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.batch, self.layers, self.seq = batch, layers, seq
        self.shape = oracle.LLAMA3_8B
        g = torch.Generator().manual_seed(5)

        def h(*s, std=0.02):
            return (torch.randn(*s, generator=g) * std).half()

        def norm_w():
            return (1.0 + 0.1 * torch.randn(HIDDEN, generator=g)).half()

        self.w = {"self_attn.q_proj.weight": h(HEADS * HEAD_DIM, HIDDEN),
                  "self_attn.k_proj.weight": h(KV_HEADS * HEAD_DIM, HIDDEN),
                  "self_attn.v_proj.weight": h(KV_HEADS * HEAD_DIM, HIDDEN),
                  "self_attn.o_proj.weight": h(HIDDEN, HEADS * HEAD_DIM),
                  "mlp.gate_proj.weight": h(FFN, HIDDEN), "mlp.up_proj.weight": h(FFN, HIDDEN),
                  "mlp.down_proj.weight": h(HIDDEN, FFN),
                  "input_layernorm.weight": norm_w(),
                  "post_attention_layernorm.weight": norm_w()}
        self.final_norm = norm_w()
        self.k = h(batch, KV_HEADS, seq, HEAD_DIM, std=1.0)
        self.v = h(batch, KV_HEADS, seq, HEAD_DIM, std=1.0)
        self.lm = h(VOCAB, HIDDEN)
        self.tokens = torch.randint(0, VOCAB, (batch,), generator=g)
        self.pos = torch.full((batch,), seq - 1, dtype=torch.int32)
        self.inv_freq = oracle.rope_inv_freq(self.shape.rope_theta, HEAD_DIM)
        self.sample = (f"oracle: whole decode steps ({layers} layers with K/V append, final "
                       f"norm, LM head, argmax) at batch {batch}, {seq} keys")

    def step(self):
        o, torch = self.oracle, self.torch
        x = self.lm[self.tokens].float()
        for _ in range(self.layers):
            x, _, _ = o.decoder_layer_decode(self.w, x, self.pos, self.k, self.v, self.shape,
                                             inv_freq=self.inv_freq, write_cache=True)
        logits = o.linear(o.rms_norm(x, self.final_norm, self.shape.eps), self.lm)
        return o.greedy_argmax(logits)

    def seconds_per_step(self):
        t0 = time.perf_counter()
        self.step()
        return time.perf_counter() - t0


def cpu_baseline(batch, layers, seq, samples=3):
    """Bounded sample of the CPU oracle: one untimed step, then the median of
    `samples` whole steps (~4 s each for the 32-layer batch-64 stack on 16 cores)."""
    step = CpuOracleStep(batch, layers, seq)
    step.seconds_per_step()
    t_step = statistics.median(step.seconds_per_step() for _ in range(samples))
    return {"value": batch / t_step, "unit": "tokens/s", "cores": step.threads, "kind": "port",
            "sample": f"{step.sample}, median of {samples} after 1 untimed",
            "cpu_model": host_cpu_model(), "seconds_per_step": t_step}


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    t_begin = time.perf_counter()
    step = CpuOracleStep(a.batch, a.layers, a.seq)
    times = [step.seconds_per_step() for _ in range(a.warmup + a.steps)][a.warmup:]
    t = statistics.median(times)
    value = a.batch / t
    line = {"metric": METRIC, "impl": "reference", "value": value, "unit": "tokens/s",
            "n_gpus": a.gpus, "steps": a.steps, "warmup": a.warmup, "ms_per_step": t * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
            "data": "synthetic", "config": workload_config(a),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": step.threads,
                             "kind": "port", "cpu_model": host_cpu_model(),
                             "sample": f"{step.sample}, median of {a.steps} timed steps after "
                                       f"{a.warmup} untimed"},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "timed_s": sum(times), "run_s": time.perf_counter() - t_begin}
    print(json.dumps(line), flush=True)
    return 0


def layer_bytes(hidden, heads, kv_heads, ffn, batch, cached, attended, qk_norm=False):
    """Algorithmic HBM bytes of one decoder-layer decode step (FP16): every weight,
    `attended` keys of K and V per sequence and KV head, the new K/V entries when
    `cached` < `attended` counts them apart (cached + 1 = attended), the norms and
    the layer's input and output rows."""
    d = HEAD_DIM
    w = ((heads + 2 * kv_heads) * d * hidden + hidden * heads * d + 3 * ffn * hidden) * 2
    kv = 2 * batch * kv_heads * cached * d * 2
    kv_new = 2 * batch * kv_heads * d * 2 if cached < attended else 0
    norms = 2 * hidden * 2 + (2 * d * 2 if qk_norm else 0)
    acts = 2 * batch * hidden * 2
    return w + kv + kv_new + norms + acts


def _time_replays(fn, reps, warmup, stream):
    """Mean seconds per call of `fn` (CUDA events on `stream`, after `warmup` calls)."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(stream)
    for _ in range(reps):
        fn()
    e.record(stream)
    torch.cuda.synchronize()
    return s.elapsed_time(e) / 1e3 / reps


def measure_configs(dev, peak, warmup, reps=20):
    """The contract's single-GPU configs 2-4, each through the library's own entry
    point with inputs resident in HBM, timed with CUDA events; bytes are the
    configs' algorithmic bytes (FP16, every weight and attended key read once)."""
    import torch
    from llm_compiler_3_b200 import ops
    from llm_compiler_3_b200.plan import llama3_8b, qwen3_8b
    from llm_compiler_3_b200.runtime import Decoder
    stream = torch.cuda.current_stream()
    gen = torch.Generator(device=dev)
    res = {}

    def randn(shape, seed, std):
        gen.manual_seed(seed)
        return (torch.randn(shape, device=dev, generator=gen) * std).half()

    # Config 2: flash-decoding, batch 1, 32 query / 8 KV heads, 4096 keys.  One
    # launch reads 16.8 MB, less than L2: ten caches are read in turn (168 MB).
    copies = 10
    q = randn((1, HEADS, HEAD_DIM), 21, 1.0)
    kvs = [(randn((1, KV_HEADS, 4096, HEAD_DIM), 22 + 2 * i, 1.0),
            randn((1, KV_HEADS, 4096, HEAD_DIM), 23 + 2 * i, 1.0)) for i in range(copies)]
    lens = torch.full((1,), 4096, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    for kc, vc in kvs:
        ops.flash_decode(q, kc, vc, lens, out=out)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for kc, vc in kvs:
            ops.flash_decode(q, kc, vc, lens, out=out)
    t = _time_replays(graph.replay, reps, warmup, stream) / copies
    b = attention_bytes(1, KV_HEADS, HEADS, 4096)
    res["attention_b1_kv4096"] = {"us": t * 1e6, "algorithmic_bytes": b,
                                  "achieved_GBps": b / t / 1e9, "frac": b / t / 1e9 / peak,
                                  "l2": f"{copies} caches read in turn ({copies * b >> 20} MiB)"}
    del graph, kvs

    def layer_case(plan, name_shapes, batch, position, qk_norm, seed):
        with Decoder(plan, device=dev.index) as dec:
            ones = torch.ones(HIDDEN, dtype=torch.float16, device=dev)
            for j, (name, shape) in enumerate(name_shapes.items()):
                dec.set_weight(f"model.layers.0.{name}", randn(shape, seed + j, 0.02))
            dec.set_weight("model.layers.0.input_layernorm.weight", ones)
            dec.set_weight("model.layers.0.post_attention_layernorm.weight", ones)
            if qk_norm:
                hd = torch.ones(HEAD_DIM, dtype=torch.float16, device=dev)
                dec.set_weight("model.layers.0.self_attn.q_norm.weight", hd)
                dec.set_weight("model.layers.0.self_attn.k_norm.weight", hd)
            k, v = dec.kv_cache(0)
            gen.manual_seed(seed + 50)
            k[:batch, :, :position].normal_(generator=gen)
            v[:batch, :, :position].normal_(generator=gen)
            x = randn((batch, HIDDEN), seed + 60, 1.0)
            pos = torch.full((batch,), position, dtype=torch.int32, device=dev)
            y = torch.empty_like(x)
            return _time_replays(lambda: dec.forward_hidden_device(x, pos, y), reps, warmup, stream)

    def shapes(ffn):
        return {"self_attn.q_proj.weight": (HEADS * HEAD_DIM, HIDDEN),
                "self_attn.k_proj.weight": (KV_HEADS * HEAD_DIM, HIDDEN),
                "self_attn.v_proj.weight": (KV_HEADS * HEAD_DIM, HIDDEN),
                "self_attn.o_proj.weight": (HIDDEN, HEADS * HEAD_DIM),
                "mlp.gate_proj.weight": (ffn, HIDDEN), "mlp.up_proj.weight": (ffn, HIDDEN),
                "mlp.down_proj.weight": (HIDDEN, ffn)}

    # Config 3: one Llama-3-8B-shaped layer, batch 1, position 2047 (2047 cached keys).
    t = layer_case(llama3_8b(layers=1, vocab=0, max_batch=1, max_seq=2048), shapes(FFN), 1, 2047,
                   False, 3000)
    b = layer_bytes(HIDDEN, HEADS, KV_HEADS, FFN, 1, 2047, 2048)
    res["llama_layer_b1_pos2047"] = {"us": t * 1e6, "tokens_per_s": 1 / t,
                                     "algorithmic_bytes": b, "achieved_GBps": b / t / 1e9,
                                     "frac": b / t / 1e9 / peak}
    # Config 4: one Qwen3-8B-shaped layer (QK-norm, theta 1e6), batch 16, 8192
    # keys attended per sequence (8191 cached + the new one).
    t = layer_case(qwen3_8b(layers=1, vocab=0, max_batch=16, max_seq=8192), shapes(12288), 16,
                   8191, True, 4000)
    b = layer_bytes(HIDDEN, HEADS, KV_HEADS, 12288, 16, 8192, 8192, qk_norm=True)
    res["qwen3_layer_b16_kv8192"] = {"us": t * 1e6, "tokens_per_s": 16 / t,
                                     "algorithmic_bytes": b, "achieved_GBps": b / t / 1e9,
                                     "frac": b / t / 1e9 / peak}
    return res


def workload_config(a):
    return {"workload": f"llama3-8b-shaped {a.layers}-layer FP16 decode stack + LM head "
                        f"4096x{VOCAB} + greedy argmax",
            "global_batch": a.batch, "kv_len": a.seq, "position": a.seq - 1,
            "layers": a.layers, "parallelism": f"tp{a.gpus}",
            "l2": "inputs larger than L2 (~49 GB read per step), no flush"}


def run_b200(a):
    import torch
    import torch.distributed as dist
    from llm_compiler_3_b200 import _native, ops
    from llm_compiler_3_b200.plan import llama3_8b
    from llm_compiler_3_b200.runtime import Decoder, nccl_unique_id

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    nid = None
    if world > 1:
        box = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        nid = box[0]

    plan = llama3_8b(layers=a.layers, max_batch=a.batch, max_seq=a.seq)
    dec = Decoder(plan, device=local, tp_rank=rank, tp_size=world, nccl_id=nid)
    info = dec.info
    gen = torch.Generator(device=dev)

    def randn(shape, seed, std):
        gen.manual_seed(seed)
        return (torch.randn(shape, device=dev, generator=gen) * std).half()

    dec.set_weight("model.embed_tokens.weight", randn((VOCAB, HIDDEN), 11, 0.02))
    dec.set_weight("lm_head.weight", randn((VOCAB, HIDDEN), 12, 0.02))
    ones = torch.ones(HIDDEN, dtype=torch.float16, device=dev)
    dec.set_weight("model.norm.weight", ones)
    shapes = {"self_attn.q_proj.weight": (HEADS * HEAD_DIM, HIDDEN),
              "self_attn.k_proj.weight": (KV_HEADS * HEAD_DIM, HIDDEN),
              "self_attn.v_proj.weight": (KV_HEADS * HEAD_DIM, HIDDEN),
              "self_attn.o_proj.weight": (HIDDEN, HEADS * HEAD_DIM),
              "mlp.gate_proj.weight": (FFN, HIDDEN), "mlp.up_proj.weight": (FFN, HIDDEN),
              "mlp.down_proj.weight": (HIDDEN, FFN)}
    for layer in range(a.layers):
        for j, (name, shape) in enumerate(shapes.items()):
            dec.set_weight(f"model.layers.{layer}.{name}", randn(shape, 1000 + 16 * layer + j, 0.02))
        dec.set_weight(f"model.layers.{layer}.input_layernorm.weight", ones)
        dec.set_weight(f"model.layers.{layer}.post_attention_layernorm.weight", ones)
        k, v = dec.kv_cache(layer)
        gen.manual_seed(50000 + 2 * layer + 1000 * rank)
        k[:, :, : a.seq - 1].normal_(generator=gen)
        gen.manual_seed(50001 + 2 * layer + 1000 * rank)
        v[:, :, : a.seq - 1].normal_(generator=gen)
    torch.cuda.synchronize()

    gen.manual_seed(7)
    tokens = torch.randint(0, VOCAB, (a.batch,), device=dev, generator=gen, dtype=torch.int32)
    positions = torch.full((a.batch,), a.seq - 1, dtype=torch.int32, device=dev)
    ids = torch.empty(a.batch, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(a.warmup):
        dec.step_device(tokens, positions, ids)
    torch.cuda.synchronize()
    _native.device_status()

    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(local).uuid)
        uuid = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
    except Exception:
        uuid = None
    clocks = ClockSampler(uuid)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(a.steps):
        dec.step_device(tokens, positions, ids)
    end.record(stream)
    torch.cuda.synchronize()
    barrier()
    clock_info = clocks.stop()
    elapsed = max_over_ranks(start.elapsed_time(end) / 1e3)
    status = _native.device_status()

    # End to end through the public API with host buffers: H2D of tokens and
    # positions, the step, D2H of the ids, every step.
    tok_h = tokens.cpu().numpy()
    pos_h = positions.cpu().numpy()
    barrier()
    torch.cuda.synchronize()
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(stream)
    t0 = time.perf_counter()
    for _ in range(a.steps):
        dec.step(tok_h, pos_h)
    e2.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    e2e_elapsed = max_over_ranks(max(s2.elapsed_time(e2) / 1e3, wall))

    # The latency case: the same stack and cache at batch 1 (one sequence,
    # position 4095), through its own captured graph in the same context.
    tok1, pos1, ids1 = tokens[:1].clone(), positions[:1].clone(), ids[:1].clone()
    for _ in range(a.warmup):
        dec.step_device(tok1, pos1, ids1)
    barrier()
    torch.cuda.synchronize()
    s1, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s1.record(stream)
    for _ in range(a.steps):
        dec.step_device(tok1, pos1, ids1)
    e1.record(stream)
    torch.cuda.synchronize()
    b1_elapsed = max_over_ranks(s1.elapsed_time(e1) / 1e3)

    # Dominant kernel (flash-decoding: ~70% of the step's bytes), timed alone on
    # this rank's shard shape with CUDA events around graph replays that
    # alternate between two layers' caches.
    kv0 = dec.kv_cache(0)
    kv1 = dec.kv_cache(1 if a.layers > 1 else 0)
    q = torch.randn(a.batch, info["q_heads"], HEAD_DIM, device=dev).half()
    out = torch.empty_like(q)
    lens = torch.full((a.batch,), a.seq, dtype=torch.int32, device=dev)
    ops.flash_decode(q, kv0[0], kv0[1], lens, out=out)
    ops.flash_decode(q, kv1[0], kv1[1], lens, out=out)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    reps = 10
    with torch.cuda.graph(graph):
        for i in range(reps):
            kv = kv0 if i % 2 == 0 else kv1
            ops.flash_decode(q, kv[0], kv[1], lens, out=out)
    graph.replay()
    torch.cuda.synchronize()
    s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s3.record(stream)
    graph.replay()
    e3.record(stream)
    torch.cuda.synchronize()
    fd_launch_s = s3.elapsed_time(e3) / 1e3 / reps
    del graph

    if rank != 0:
        dec.close()
        if world > 1:
            dist.destroy_process_group()
        return 0

    peak, peak_kind = measured_peak()
    fd_bytes = attention_bytes(a.batch, info["kv_heads"], info["q_heads"], a.seq)
    fd_achieved = fd_bytes / fd_launch_s / 1e9
    traffic = ncu_traffic()
    if traffic is not None and world > 1:
        traffic = traffic // world
    t_step = elapsed / a.steps
    value = a.batch * a.steps / elapsed
    sb = step_bytes(a.batch, a.layers, a.seq)
    per_step_launches = 1 + a.layers * (5 + (2 if world > 1 else 0)) + 2 + (1 if world > 1 else 0)
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": t_step * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16",
        "data": "synthetic (random-init weights N(0,0.02), KV cache N(0,1), seeded on device)",
        "config": dict(workload_config(a), **({"tp_exchange": "nvlink peer memory"
                                                 if info.get("peer_exchange") else "nccl"}
                                                if world > 1 else {})),
        "roofline": {"bound": "hbm", "kernel": "flash_decode", "achieved": fd_achieved,
                     "peak": peak, "unit": "GB/s", "frac": fd_achieved / peak,
                     "peak_source": peak_kind, "traffic": traffic,
                     "algorithmic_bytes_per_launch": fd_bytes,
                     "launch_us": fd_launch_s * 1e6},
        "step_roofline": {"algorithmic_bytes": sb, "achieved_GBps": sb / t_step / 1e9,
                          "frac": sb / t_step / 1e9 / (peak * world), "peak_GBps": peak * world},
        "e2e": {"value": a.batch * a.steps / e2e_elapsed, "unit": "tokens/s",
                "h2d_bytes_per_step": 2 * 4 * a.batch, "d2h_bytes_per_step": 4 * a.batch},
        "batch1_stack": {
            "tokens_per_s": a.steps / b1_elapsed, "ms_per_token": b1_elapsed / a.steps * 1e3,
            "algorithmic_bytes": step_bytes(1, a.layers, a.seq),
            "step_roofline_frac": step_bytes(1, a.layers, a.seq) / (b1_elapsed / a.steps) / 1e9
            / (peak * world)},
        "gpu_launches": per_step_launches * a.steps,
        "device_error_bits": status,
    }
    if clock_info:
        line["clocks"] = clock_info
    dec.close()
    if world == 1 and not a.no_configs:
        line["configs"] = measure_configs(dev, peak, a.warmup)
    if world == 1 and not a.no_cpu_baseline:
        base = cpu_baseline(a.batch, a.layers, a.seq)
        line["cpu_baseline"] = {k: base[k] for k in ("value", "unit", "cores", "kind", "sample",
                                                     "cpu_model")}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()
    return 0


def main(argv=None):
    a = parse_args(argv)
    if a.impl == "reference":
        return run_reference(a)
    return run_b200(a)


if __name__ == "__main__":
    sys.exit(main())
