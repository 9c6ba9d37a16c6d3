"""Tensor parallelism on the CPU: two gloo ranks, no GPU.

Each rank asks the library which share of the model it holds
(npu_b200_shard_info -- the split the runtime applies when weights are set),
takes exactly those rows and columns of the weights and the KV cache, and runs
a decode step of a 2-layer stack with the oracle's arithmetic: column-sharded
q/k/v and gate/up, row-sharded o_proj and down_proj each followed by an
all-reduce, the LM head sharded by vocabulary rows with the per-rank argmaxes
all-gathered (ties to the lowest id, like torch.argmax).  The ranks' greedy ids
must equal the single-process oracle's, and every logit must agree -- the
decomposition the B200 runtime uses is exact up to summation order."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle

SHAPE = oracle.DecoderShape(hidden=256, heads=4, kv_heads=2, head_dim=128, ffn=512, eps=1e-5,
                            rope_theta=500000.0, vocab=1001, layers=2)
BATCH, MAX_SEQ = 3, 32
POSITIONS = [0, 5, 31]
TOKENS = [7, 1000, 512]


def _half(shape, seed, std):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * std).half()


def _model():
    s, H, D = SHAPE, SHAPE.hidden, SHAPE.head_dim
    top = {"embed": _half((s.vocab, H), 1, 0.5), "norm": (1 + 0.1 * _half((H,), 2, 1.0).float()).half(),
           "lm_head": _half((s.vocab, H), 3, 0.05)}
    layers = []
    for i in range(s.layers):
        b = 100 * (i + 1)
        layers.append({
            "self_attn.q_proj.weight": _half((s.heads * D, H), b + 1, 0.05),
            "self_attn.k_proj.weight": _half((s.kv_heads * D, H), b + 2, 0.05),
            "self_attn.v_proj.weight": _half((s.kv_heads * D, H), b + 3, 0.05),
            "self_attn.o_proj.weight": _half((H, s.heads * D), b + 4, 0.05),
            "mlp.gate_proj.weight": _half((s.ffn, H), b + 5, 0.05),
            "mlp.up_proj.weight": _half((s.ffn, H), b + 6, 0.05),
            "mlp.down_proj.weight": _half((H, s.ffn), b + 7, 0.05),
            "input_layernorm.weight": (1 + 0.1 * _half((H,), b + 8, 1.0).float()).half(),
            "post_attention_layernorm.weight": (1 + 0.1 * _half((H,), b + 9, 1.0).float()).half(),
        })
    caches = [(_half((BATCH, s.kv_heads, MAX_SEQ, D), 500 + i, 1.0),
               _half((BATCH, s.kv_heads, MAX_SEQ, D), 600 + i, 1.0)) for i in range(s.layers)]
    return top, layers, caches


def _plan(path):
    from llm_compiler_3_b200.plan import DecodePlan
    s = SHAPE
    return DecodePlan(arch="llama", hidden=s.hidden, heads=s.heads, kv_heads=s.kv_heads,
                      head_dim=s.head_dim, ffn=s.ffn, layers=s.layers, vocab=s.vocab,
                      rms_eps=s.eps, rope_theta=s.rope_theta, max_batch=BATCH,
                      max_seq=MAX_SEQ).write(path)


def _shard_info(plan_path, rank, world):
    import ctypes
    from llm_compiler_3_b200 import _native
    out = (ctypes.c_int64 * 5)()
    _native.check(_native.lib().npu_b200_shard_info(str(plan_path).encode(), rank, world, out, 5))
    return list(out)


def _rank_main(rank, world, port, plan_path, out_dir):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    s, D = SHAPE, SHAPE.head_dim
    q_loc, kv_loc, ffn_loc, vocab_loc, vocab_off = _shard_info(plan_path, rank, world)
    top, layers, caches = _model()
    qs, ks, fs = slice(rank * q_loc * D, (rank + 1) * q_loc * D), \
        slice(rank * kv_loc * D, (rank + 1) * kv_loc * D), slice(rank * ffn_loc, (rank + 1) * ffn_loc)
    positions = torch.tensor(POSITIONS)
    inv_freq = oracle.rope_inv_freq(s.rope_theta, D)
    cos, sin = oracle.rope_cos_sin(inv_freq, positions)
    x = top["embed"][torch.tensor(TOKENS)].float()
    for i, w in enumerate(layers):
        k_cache = caches[i][0][:, rank * kv_loc:(rank + 1) * kv_loc].clone()
        v_cache = caches[i][1][:, rank * kv_loc:(rank + 1) * kv_loc].clone()
        h = oracle.rms_norm(x, w["input_layernorm.weight"], s.eps)
        q = oracle.linear(h, w["self_attn.q_proj.weight"][qs]).view(BATCH, q_loc, D)
        k = oracle.linear(h, w["self_attn.k_proj.weight"][ks]).view(BATCH, kv_loc, D)
        v = oracle.linear(h, w["self_attn.v_proj.weight"][ks]).view(BATCH, kv_loc, D)
        q, k = oracle.apply_rope(q, cos, sin), oracle.apply_rope(k, cos, sin)
        attn = torch.zeros(BATCH, q_loc, D)
        for b, p in enumerate(POSITIONS):
            kb = torch.cat([k_cache[b, :, :p].float(), k[b][:, None]], dim=1)
            vb = torch.cat([v_cache[b, :, :p].float(), v[b][:, None]], dim=1)
            attn[b] = oracle.attention_decode(q[b:b + 1], kb[None], vb[None], [p + 1], D ** -0.5)[0]
        part = oracle.linear(attn.reshape(BATCH, -1), w["self_attn.o_proj.weight"][:, qs])
        dist.all_reduce(part)  # the exchange after o_proj
        y = x + part
        h = oracle.rms_norm(y, w["post_attention_layernorm.weight"], s.eps)
        act = oracle.silu_mul(oracle.linear(h, w["mlp.gate_proj.weight"][fs]),
                              oracle.linear(h, w["mlp.up_proj.weight"][fs]))
        part = oracle.linear(act, w["mlp.down_proj.weight"][:, fs])
        dist.all_reduce(part)  # the exchange after down_proj
        x = y + part
    h = oracle.rms_norm(x, top["norm"], s.eps)
    logits = oracle.linear(h, top["lm_head"][vocab_off:vocab_off + vocab_loc])
    best = oracle.greedy_argmax(logits)
    pair = torch.stack([logits.gather(1, best[:, None])[:, 0], (best + vocab_off).float()], dim=1)
    pairs = [torch.zeros_like(pair) for _ in range(world)]
    dist.all_gather(pairs, pair)  # per-rank (value, id) of the best logit
    value = torch.stack([p[:, 0] for p in pairs], dim=1)
    ids = torch.stack([p[:, 1] for p in pairs], dim=1).long()
    top_v = value.max(dim=1, keepdim=True).values
    winner = torch.where(value == top_v, ids, s.vocab).min(dim=1).values
    np.save(os.path.join(out_dir, f"ids_r{rank}.npy"), winner.numpy())
    np.save(os.path.join(out_dir, f"logits_r{rank}.npy"), logits.numpy())
    np.save(os.path.join(out_dir, f"shard_r{rank}.npy"), np.array([q_loc, kv_loc, ffn_loc, vocab_loc,
                                                                   vocab_off]))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as sock:
        sock.bind(("127.0.0.1", 0))
        return sock.getsockname()[1]


def test_shard_info_partitions_the_model(tmp_path):
    plan = _plan(tmp_path / "plan.txt")
    for world in (1, 2):
        infos = [_shard_info(plan, r, world) for r in range(world)]
        assert sum(i[0] for i in infos) == SHAPE.heads and sum(i[1] for i in infos) == SHAPE.kv_heads
        assert sum(i[2] for i in infos) == SHAPE.ffn
        assert [i[4] for i in infos] == [sum(j[3] for j in infos[:r]) for r in range(world)]
        assert sum(i[3] for i in infos) == SHAPE.vocab
    from llm_compiler_3_b200 import _native
    with pytest.raises(_native.NpuError, match="kv_heads 2 not divisible"):
        _shard_info(plan, 0, 4)


def test_two_gloo_ranks_match_the_oracle(tmp_path):
    plan = _plan(tmp_path / "plan.txt")
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), str(plan), str(tmp_path)),
                       nprocs=world, start_method="spawn", join=True)
    top, layers, caches = _model()
    ids, logits = oracle.stack_decode(lambda i: layers[i], SHAPE.layers, top["embed"], top["norm"],
                                      top["lm_head"], torch.tensor(TOKENS), torch.tensor(POSITIONS),
                                      lambda i: (caches[i][0].clone(), caches[i][1].clone()), SHAPE,
                                      return_logits=True)
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"ids_r{r}.npy"), ids.numpy())
    parts = []
    for r in range(world):
        _, _, _, vocab_loc, vocab_off = np.load(tmp_path / f"shard_r{r}.npy")
        part = np.load(tmp_path / f"logits_r{r}.npy")
        assert part.shape == (BATCH, vocab_loc)
        parts.append(part)
    np.testing.assert_allclose(np.concatenate(parts, axis=1), logits.numpy(), atol=1e-4, rtol=0)
