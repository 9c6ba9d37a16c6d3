"""Tensor-parallel decode (2 or 4 ranks, one process per GPU) against the oracle.

q/k/v and gate/up are column-sharded, o_proj/down_proj row-sharded with one
NCCL all-reduce each, the LM head vocabulary-sharded with an all-gather of
per-rank argmaxes.  Every rank must return the oracle's greedy ids and hidden
states; ranks learn each other's NCCL id through torch.distributed (gloo)."""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import oracle

pytestmark = pytest.mark.gpu

SHAPE = oracle.DecoderShape(hidden=1024, heads=8, kv_heads=4, head_dim=128, ffn=2048, eps=1e-5,
                            rope_theta=500000.0, vocab=8192, layers=2)
BATCH, MAX_SEQ = 4, 256
POSITIONS = [0, 77, 200, 255]


def _half(shape, seed, std):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g) * std).half()


def _weights():
    s, H, D = SHAPE, SHAPE.hidden, SHAPE.head_dim
    top = {"model.embed_tokens.weight": _half((s.vocab, H), 1, 0.02),
           "model.norm.weight": (1 + 0.1 * _half((H,), 2, 1.0).float()).half(),
           "lm_head.weight": _half((s.vocab, H), 3, 0.02)}
    layers = []
    for i in range(s.layers):
        b = 100 * (i + 1)
        layers.append({
            "self_attn.q_proj.weight": _half((s.heads * D, H), b + 1, 0.03),
            "self_attn.k_proj.weight": _half((s.kv_heads * D, H), b + 2, 0.03),
            "self_attn.v_proj.weight": _half((s.kv_heads * D, H), b + 3, 0.03),
            "self_attn.o_proj.weight": _half((H, s.heads * D), b + 4, 0.03),
            "mlp.gate_proj.weight": _half((s.ffn, H), b + 5, 0.03),
            "mlp.up_proj.weight": _half((s.ffn, H), b + 6, 0.03),
            "mlp.down_proj.weight": _half((H, s.ffn), b + 7, 0.03),
            "input_layernorm.weight": (1 + 0.1 * _half((H,), b + 8, 1.0).float()).half(),
            "post_attention_layernorm.weight": (1 + 0.1 * _half((H,), b + 9, 1.0).float()).half(),
        })
    caches = [(_half((BATCH, s.kv_heads, MAX_SEQ, 128), 500 + i, 1.0),
               _half((BATCH, s.kv_heads, MAX_SEQ, 128), 600 + i, 1.0)) for i in range(s.layers)]
    tokens = torch.tensor([5, 4000, 8191, 123], dtype=torch.int32)
    return top, layers, caches, tokens


def _rank_main(rank, world, port, out_dir, batch, exchange):
    os.environ["NPU_B200_TP_EXCHANGE"] = exchange
    import torch.distributed as dist
    from llm_compiler_3_b200.plan import DecodePlan
    from llm_compiler_3_b200.runtime import Decoder, nccl_unique_id
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    box = [nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    s = SHAPE
    plan = DecodePlan(arch="llama", hidden=s.hidden, heads=s.heads, kv_heads=s.kv_heads,
                      head_dim=s.head_dim, ffn=s.ffn, layers=s.layers, vocab=s.vocab,
                      rms_eps=s.eps, rope_theta=s.rope_theta, max_batch=BATCH, max_seq=MAX_SEQ)
    top, layers, caches, tokens = _weights()
    kv_loc = s.kv_heads // world
    with Decoder(plan, device=rank, tp_rank=rank, tp_size=world, nccl_id=box[0]) as dec:
        np.save(os.path.join(out_dir, f"peer_r{rank}.npy"), np.array(dec.info["peer_exchange"]))
        for name, t in top.items():
            dec.set_weight(name, t)
        for i, w in enumerate(layers):
            for name, t in w.items():
                dec.set_weight(f"model.layers.{i}.{name}", t)
        for step in range(2):  # the second step re-uses the captured graph
            for i, (kc, vc) in enumerate(caches):
                k, v = dec.kv_cache(i)
                k.copy_(kc[:, rank * kv_loc:(rank + 1) * kv_loc].cuda())
                v.copy_(vc[:, rank * kv_loc:(rank + 1) * kv_loc].cuda())
            ids = dec.step(tokens[:batch].numpy(), POSITIONS[:batch])
            np.save(os.path.join(out_dir, f"ids_r{rank}_s{step}.npy"), ids)
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
@pytest.mark.parametrize("batch", [1, 4])
@pytest.mark.parametrize("exchange", ["peer", "nccl"])
def test_tensor_parallel_matches_oracle(world, batch, exchange):
    """Batch 1 runs the GEMV projections, batch 4 the tensor-core ones; the
    all-reduces go over NVLink peer memory (or NCCL when asked)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"tensor parallel over {world} ranks needs {world} GPUs")
    with tempfile.TemporaryDirectory() as out:
        mp.start_processes(_rank_main, args=(world, _free_port(), out, batch, exchange),
                           nprocs=world, start_method="spawn", join=True)
        got = [[np.load(os.path.join(out, f"ids_r{r}_s{s}.npy")) for r in range(world)]
               for s in range(2)]
        peer = [int(np.load(os.path.join(out, f"peer_r{r}.npy"))) for r in range(world)]
    assert peer == [1 if exchange == "peer" else 0] * world
    top, layers, caches, tokens = _weights()
    ref_ids, logits = oracle.stack_decode(
        lambda i: layers[i], SHAPE.layers, top["model.embed_tokens.weight"],
        top["model.norm.weight"], top["lm_head.weight"], tokens[:batch],
        torch.tensor(POSITIONS[:batch], dtype=torch.int32),
        lambda i: (caches[i][0][:batch].clone(), caches[i][1][:batch].clone()), SHAPE,
        return_logits=True)
    from test_decode import _check_ids
    for per_step in got:
        for ids in per_step:
            assert np.array_equal(ids, per_step[0]), "ranks disagree"
        _check_ids(per_step[0], ref_ids, logits)
