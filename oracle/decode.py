"""FP32 CPU restatement of the decode computation (test infrastructure only).

Every tensor that the B200 path stores in FP16 (weights, KV cache, activations
handed between kernels) is taken as FP16 here too, then widened; all arithmetic
is FP32.  This is the "FP32-accumulated result" the parity tolerances refer to:
max-abs 2e-2 and cosine >= 0.9999 for FP16 outputs, exact for KV indexing,
positions and argmax ids.

Reference anchors (paths inside LLM_Compiler_3 unless marked transformers):
  * matmul: FP16 operands, FP32 accumulation from zero, one FP16 rounding at the
    write-out -- lib/Transforms/Normalize.cpp:123-192 (foldAccumulateAndRound),
    lib/Transforms/Legalize.cpp:136-161 (zero-filled accumulator),
    lib/Transforms/Emit.cpp:348-378 (matrix write-out).
  * attention: npu.attention with group / scale / key_transposed,
    include/npu/Dialect/NPUDialect.td:31-61 and the online-softmax row ops
    147-189; expansion lib/Transforms/Attention.cpp:296-374 (CS-4);
    default scale 1/sqrt(d) canonicalizeAttention Attention.cpp:384-419.
  * row reductions in FP32 -- lib/Transforms/Pipeline.cpp:149-185 (reductionOf),
    lib/Transforms/Normalize.cpp:74-104 (widenRowChain).
  * the decoder layer itself is the module the reference captures
    (examples/llama/capture.py:15-58): transformers 5.5
    models/llama/modeling_llama.py LlamaRMSNorm / rotate_half /
    apply_rotary_pos_emb / LlamaAttention / LlamaMLP / LlamaDecoderLayer, and
    models/qwen3/modeling_qwen3.py Qwen3Attention (q_norm / k_norm on the head
    dim before RoPE).
  * the MLP plumbing config follows examples/pytorch/mlp.py:44-51.
  * decode-step semantics (flat cache in, new entry written at `position`,
    attention over positions [0, position]) follow docs/DESIGN.md:365-392.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable, Mapping

import torch

__all__ = [
    "DecoderShape", "grid_values", "linear", "rms_norm", "norm_for_projection", "rope_inv_freq",
    "rope_cos_sin",
    "apply_rope", "attention_decode", "attention_prefill", "attention_online", "silu_mul", "decoder_layer_decode",
    "stack_decode", "mlp_forward", "greedy_argmax", "cosine", "LLAMA3_8B", "QWEN3_8B",
]


@dataclass(frozen=True)
class DecoderShape:
    """Architecture numbers of one decoder family."""

    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    eps: float
    rope_theta: float
    qk_norm: bool = False
    vocab: int = 0
    layers: int = 1

    @property
    def group(self) -> int:
        return self.heads // self.kv_heads


LLAMA3_8B = DecoderShape(hidden=4096, heads=32, kv_heads=8, head_dim=128, ffn=14336, eps=1e-5,
                         rope_theta=500000.0, vocab=128256, layers=32)
QWEN3_8B = DecoderShape(hidden=4096, heads=32, kv_heads=8, head_dim=128, ffn=12288, eps=1e-6,
                        rope_theta=1000000.0, qk_norm=True, vocab=151936, layers=36)


def _f32(t: torch.Tensor) -> torch.Tensor:
    """FP16 storage widened to FP32 (what every kernel reads)."""
    return t.to(torch.float16).to(torch.float32) if t.dtype != torch.float32 else t


def grid_values(count: int, seed: int) -> torch.Tensor:
    """Known-answer operands: |x| <= 1/2 on the 1/16 grid, so with K <= 512 every
    FP32 partial sum is exact and an FP16 result can be checked bit for bit
    (test/Integration/matmul.py:18-21, docs/DESIGN.md:407-410)."""
    return ((torch.arange(count) * seed % 17 - 8).float() / 16).half()


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """y[B, N] = x[B, K] . W[N, K]^T (+ b) with FP16 operands and FP32 accumulation
    (Normalize.cpp:123-192; W is torch's [out, in] layout, capture arg<N>.bin)."""
    y = _f32(x) @ _f32(weight).t()
    if bias is not None:
        y = y + _f32(bias)
    return y


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """transformers LlamaRMSNorm / Qwen3RMSNorm in FP32: x * rsqrt(mean(x^2) + eps) * w."""
    x = x.to(torch.float32)
    variance = x.pow(2).mean(-1, keepdim=True)
    return _f32(weight) * (x * torch.rsqrt(variance + eps))


def rope_inv_freq(theta: float, head_dim: int) -> torch.Tensor:
    """transformers compute_default_rope_parameters: 1 / theta^(2i/d), FP32."""
    exponent = torch.arange(0, head_dim, 2, dtype=torch.int64).to(torch.float32) / head_dim
    return 1.0 / (theta ** exponent)


def rope_cos_sin(inv_freq: torch.Tensor, positions: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """LlamaRotaryEmbedding.forward: freqs = pos * inv_freq in FP32, emb = cat(freqs, freqs)."""
    freqs = positions.to(torch.float32)[:, None] * inv_freq.to(torch.float32)[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos(), emb.sin()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """apply_rotary_pos_emb: x * cos + rotate_half(x) * sin, x [B, H, D], cos/sin [B, D]."""
    half = x.shape[-1] // 2
    rotated = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos[:, None, :] + rotated * sin[:, None, :]


def attention_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     seq_lens, scale: float) -> torch.Tensor:
    """One query per sequence against its cache: softmax(scale q K^T) V over keys
    [0, seq_lens[b]).  GQA: query head h reads KV head h // group
    (Attention.cpp:42-68 unrepeat -> npu.attention group).  A sequence with no
    keys yields zeros (the B200 kernel's documented convention).

    q [B, Hq, D]; k_cache, v_cache [B, Hkv, S, D]; returns FP32 [B, Hq, D]."""
    batch, heads, dim = q.shape
    kv_heads = k_cache.shape[1]
    group = heads // kv_heads
    out = torch.zeros(batch, heads, dim, dtype=torch.float32)
    for b in range(batch):
        n = int(seq_lens[b])
        if n <= 0:
            continue
        k = _f32(k_cache[b, :, :n])                      # [Hkv, n, D]
        v = _f32(v_cache[b, :, :n])
        qg = _f32(q[b]).view(kv_heads, group, dim)        # head h -> KV head h // group
        scores = torch.einsum("kgd,knd->kgn", qg, k) * scale
        probs = torch.softmax(scores, dim=-1)
        out[b] = torch.einsum("kgn,knd->kgd", probs, v).reshape(heads, dim)
    return out


def attention_prefill(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      keys: int, scale: float, causal: bool, q_start=None) -> torch.Tensor:
    """M queries per head against keys [0, keys) of the cache: npu.attention with
    M >= 1 rows (NPUDialect.td:31-61).  Causal: query i of sequence b sees key j
    iff j <= q_start[b] + i; q_start 0 is the mask the frontend builds for
    is_causal (0 where the key index is at most the query index, -inf elsewhere,
    Attention.cpp:70-92).  A row with no visible key yields zeros.

    q [B, Hq, M, D]; k_cache, v_cache [B, Hkv, S, D]; returns FP32 [B, Hq, M, D]."""
    batch, heads, queries, dim = q.shape
    kv_heads = k_cache.shape[1]
    group = heads // kv_heads
    out = torch.zeros(batch, heads, queries, dim, dtype=torch.float32)
    if keys <= 0:
        return out
    for b in range(batch):
        k = _f32(k_cache[b, :, :keys]).repeat_interleave(group, dim=0)   # [Hq, n, D]
        v = _f32(v_cache[b, :, :keys]).repeat_interleave(group, dim=0)
        scores = torch.einsum("hmd,hnd->hmn", _f32(q[b]), k) * scale
        if causal:
            start = 0 if q_start is None else int(q_start[b])
            rows = torch.arange(queries)[:, None] + start
            visible = torch.arange(keys)[None, :] <= rows
            scores = scores.masked_fill(~visible, float("-inf"))
            seen = visible.any(dim=1)
        else:
            seen = torch.ones(queries, dtype=torch.bool)
        probs = torch.softmax(scores, dim=-1).nan_to_num(0.0) * seen[None, :, None]
        out[b] = torch.einsum("hmn,hnd->hmd", probs, v)
    return out


def attention_online(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     seq_lens, scale: float, block: int = 32) -> torch.Tensor:
    """The same attention as the block-wise online softmax the reference expands
    (Attention.cpp:296-374; NPUDialect.td:150-154): per key block j,
    m = max(m, rowmax(t)), p = exp(t - m), alpha = exp(m_prev - m),
    l = alpha l + sum p, O = alpha O + P V, and out = O / l at the end."""
    batch, heads, dim = q.shape
    kv_heads = k_cache.shape[1]
    group = heads // kv_heads
    out = torch.zeros(batch, heads, dim, dtype=torch.float32)
    for b in range(batch):
        n = int(seq_lens[b])
        if n <= 0:
            continue
        qb = _f32(q[b])
        m = torch.full((heads,), -math.inf)
        l = torch.zeros(heads)
        acc = torch.zeros(heads, dim)
        for start in range(0, n, block):
            stop = min(n, start + block)
            k = _f32(k_cache[b, :, start:stop]).repeat_interleave(group, dim=0)
            v = _f32(v_cache[b, :, start:stop]).repeat_interleave(group, dim=0)
            t = torch.einsum("hd,hnd->hn", qb, k) * scale
            m_new = torch.maximum(m, t.max(dim=-1).values)
            p = torch.exp(t - m_new[:, None])
            alpha = torch.exp(m - m_new)
            l = alpha * l + p.sum(dim=-1)
            acc = alpha[:, None] * acc + torch.einsum("hn,hnd->hd", p, v)
            m = m_new
        out[b] = acc / l[:, None]
    return out


def silu_mul(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """LlamaMLP activation: silu(gate) * up (hidden_act = "silu")."""
    return torch.nn.functional.silu(gate) * up


def _handoff(t: torch.Tensor, fp16: bool) -> torch.Tensor:
    """A tensor handed from one kernel to the next: stored in FP16 when `fp16`."""
    return t.to(torch.float16).to(torch.float32) if fp16 else t


def norm_for_projection(x: torch.Tensor, weight: torch.Tensor, eps: float,
                        fp16: bool = False) -> torch.Tensor:
    """RMSNorm of a projection's input.  With fp16, as the B200 kernels hand it
    over: the producer stores xw = fp16(x * w) and the consumer multiplies its
    FP32 dot products by rsqrt(mean(x^2) + eps) (linear in the row, so the scale
    is applied here before the product)."""
    if not fp16:
        return rms_norm(x, weight, eps)
    x = x.to(torch.float32)
    scale = torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps)
    return scale * _handoff(x * _f32(weight), True)


def decoder_layer_decode(weights: Mapping[str, torch.Tensor], x: torch.Tensor,
                         positions: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                         shape: DecoderShape, inv_freq: torch.Tensor | None = None,
                         write_cache: bool = True, fp16_handoff: bool = False
                         ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """One decode step of LlamaDecoderLayer / Qwen3DecoderLayer for B sequences.

    weights: transformers names relative to the layer ("self_attn.q_proj.weight", ...).
    x [B, hidden] (any float dtype), positions [B] (int), caches [B, Hkv, S, D] FP16.
    Sequence b writes its new K/V at positions[b] and attends keys [0, positions[b]].
    Returns (y FP32 [B, hidden], k_new FP32 [B, Hkv, D], v_new FP32 [B, Hkv, D]); with
    write_cache the FP16-rounded new entries are stored into the caches in place.

    fp16_handoff rounds to FP16 where the B200 path stores a tensor between
    kernels -- the normed projection inputs (norm_for_projection), q / k / v
    after RoPE (k and v are attended from the FP16 cache), the attention output
    and the SwiGLU output -- so that only accumulation order differs; the
    residual stream stays FP32 as there.  Off, every intermediate is FP32 (the
    FP32-accumulated result the tolerances refer to).
    """
    batch = x.shape[0]
    hd = shape.head_dim
    if inv_freq is None:
        inv_freq = rope_inv_freq(shape.rope_theta, hd)
    x = x.to(torch.float32)
    residual = x
    h = norm_for_projection(x, weights["input_layernorm.weight"], shape.eps, fp16_handoff)
    q = linear(h, weights["self_attn.q_proj.weight"]).view(batch, shape.heads, hd)
    k = linear(h, weights["self_attn.k_proj.weight"]).view(batch, shape.kv_heads, hd)
    v = linear(h, weights["self_attn.v_proj.weight"]).view(batch, shape.kv_heads, hd)
    if shape.qk_norm:
        q = rms_norm(q, weights["self_attn.q_norm.weight"], shape.eps)
        k = rms_norm(k, weights["self_attn.k_norm.weight"], shape.eps)
    cos, sin = rope_cos_sin(inv_freq, positions)
    q = _handoff(apply_rope(q, cos, sin), fp16_handoff)
    k = _handoff(apply_rope(k, cos, sin), fp16_handoff)
    v = _handoff(v, fp16_handoff)

    attn = torch.zeros(batch, shape.heads, hd)
    scale = hd ** -0.5
    for b in range(batch):
        p = int(positions[b])
        kb = torch.cat([_f32(k_cache[b, :, :p]), k[b][:, None, :]], dim=1)
        vb = torch.cat([_f32(v_cache[b, :, :p]), v[b][:, None, :]], dim=1)
        attn[b] = attention_decode(q[b:b + 1], kb[None], vb[None], [p + 1], scale)[0]
    if write_cache:
        for b in range(batch):
            p = int(positions[b])
            k_cache[b, :, p] = k[b].to(k_cache.dtype)
            v_cache[b, :, p] = v[b].to(v_cache.dtype)

    attn = _handoff(attn, fp16_handoff)
    y = residual + linear(attn.reshape(batch, -1), weights["self_attn.o_proj.weight"])
    residual = y
    h = norm_for_projection(y, weights["post_attention_layernorm.weight"], shape.eps,
                            fp16_handoff)
    gate = linear(h, weights["mlp.gate_proj.weight"])
    up = linear(h, weights["mlp.up_proj.weight"])
    act = _handoff(silu_mul(gate, up), fp16_handoff)
    y = residual + linear(act, weights["mlp.down_proj.weight"])
    return y, k, v


def stack_decode(layer_weights: Callable[[int], Mapping[str, torch.Tensor]], num_layers: int,
                 embed: torch.Tensor, final_norm: torch.Tensor, lm_head: torch.Tensor,
                 tokens: torch.Tensor, positions: torch.Tensor,
                 caches: Callable[[int], tuple[torch.Tensor, torch.Tensor]],
                 shape: DecoderShape, return_logits: bool = False, fp16_handoff: bool = False):
    """LlamaForCausalLM decode step followed by greedy argmax.

    layer_weights(i) / caches(i) produce layer i's tensors on demand, so a 32-layer
    8B-shaped stack is checked one layer at a time.  Returns argmax ids [B]
    (ties to the lowest id, like torch.argmax) and, if asked, FP32 logits.
    fp16_handoff as in decoder_layer_decode (the LM head's input included)."""
    inv_freq = rope_inv_freq(shape.rope_theta, shape.head_dim)
    x = _f32(embed[tokens.long()])
    for i in range(num_layers):
        k_cache, v_cache = caches(i)
        x, _, _ = decoder_layer_decode(layer_weights(i), x, positions, k_cache, v_cache, shape,
                                       inv_freq=inv_freq, fp16_handoff=fp16_handoff)
    h = norm_for_projection(x, final_norm, shape.eps, fp16_handoff)
    logits = linear(h, lm_head)
    ids = greedy_argmax(logits)
    return (ids, logits) if return_logits else ids


def greedy_argmax(logits: torch.Tensor) -> torch.Tensor:
    """argmax over the vocabulary, ties to the lowest index."""
    best = logits.max(dim=-1, keepdim=True).values
    idx = torch.arange(logits.shape[-1]).expand_as(logits)
    return torch.where(logits == best, idx, logits.shape[-1]).min(dim=-1).values


def mlp_forward(x: torch.Tensor, w1: torch.Tensor, b1: torch.Tensor, w2: torch.Tensor,
                b2: torch.Tensor, round_hidden: bool = True) -> torch.Tensor:
    """examples/pytorch/mlp.py:44-51: down(relu(up(x))) with biases.  The hidden
    activation is handed between the two matmuls in FP16 when round_hidden."""
    hidden = torch.relu(linear(x, w1, b1))
    if round_hidden:
        hidden = hidden.half().float()
    return linear(hidden, w2, b2)


def cosine(a: torch.Tensor, b: torch.Tensor) -> float:
    """Cosine similarity of two tensors, flattened, in float64."""
    a = a.double().flatten()
    b = b.double().flatten()
    denom = a.norm() * b.norm()
    return float((a @ b) / denom) if denom > 0 else float(a.norm() == b.norm())
