"""Fused projection epilogues (npu_b200_projection) against the CPU oracle.

Each epilogue is the arithmetic of one piece of the decoder layer the reference
captures (examples/llama/capture.py:15-58), fused behind the FP32-accumulated
matmul (lib/Transforms/Normalize.cpp:123-192): RMSNorm scale, RoPE, QK-norm,
KV append, SwiGLU, residual add + next norm, greedy-argmax partials."""
import ctypes

import pytest
import torch

import oracle
from conftest import seeded

pytestmark = pytest.mark.gpu
ATOL = 2e-2


def _p(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _close(got, ref, atol=ATOL):
    err = float((got.float().cpu() - ref).abs().max())
    assert err <= atol, f"max-abs {err}"
    assert oracle.cosine(got.float().cpu(), ref) >= 0.9999


def _norm_input(x32, batch, parts=4):
    """The producer side of the fused RMSNorm: partial sums of squares of the
    FP32 hidden state over `parts` row chunks (what the residual epilogue writes)."""
    chunks = x32.view(batch, parts, -1)
    return (chunks * chunks).sum(-1).t().contiguous()      # [parts, batch]


def _pair_order(w, heads):
    """Rows of each 128-row head in rotary pair order: row 2i holds dim i,
    row 2i + 1 dim i + 64 (NPU_B200_PACK_HEAD_PAIRS)."""
    i = torch.arange(64)
    perm = torch.stack([i, i + 64], 1).reshape(-1)
    return w.view(heads, 128, -1)[:, perm].reshape(w.shape)


def _interleave(gate, up):
    """gate_j at row 2j, up_j at row 2j + 1 (NPU_B200_PACK_INTERLEAVE)."""
    return torch.stack([gate, up], 1).reshape(2 * gate.shape[0], -1)


@pytest.mark.parametrize("batch", [1, 2, 16, 64])
@pytest.mark.parametrize("packed", [False, True])
@pytest.mark.parametrize("rows", [6144 + 64, 768])
def test_packed_weights(cuda, batch, packed, rows):
    """Panels give the bit-identical tensor-core result; at batch 1-2 packed
    weights run the GEMV (768 rows: K split over clusters of 8), checked
    against the oracle."""
    from llm_compiler_3_b200 import _native, ops
    x = seeded((batch, 4096), 1)
    w = seeded((rows, 4096), 2, 0.02)          # 6208: partial last tile
    ref = ops.linear(x.cuda(), w.cuda(), out_dtype=torch.float32)
    e = _native.Epilogue(kind=_native.EPI_STORE, ld_out=w.shape[0], out_f32=1)
    out = torch.empty(batch, w.shape[0], dtype=torch.float32, device="cuda")
    e.out = _p(out)
    wd = w.cuda()
    ops.projection(x.cuda(), ops.pack_weight(wd) if packed else wd, w.shape[0], e, packed=packed)
    if packed and batch <= 2:
        _close(out, oracle.linear(x, w), atol=1e-3)
    else:
        assert torch.equal(out, ref)


@pytest.mark.parametrize("batch", [1, 2, 16, 64])
@pytest.mark.parametrize("qk_norm", [False, True])
@pytest.mark.parametrize("packed", [False, True])
def test_qkv_rope_append(cuda, batch, qk_norm, packed):
    """QKV projection with the input RMSNorm scale, optional per-head QK-norm,
    RoPE at per-sequence positions and the KV append (exact slot)."""
    from llm_compiler_3_b200 import _native, ops
    H, qh, kvh, max_seq = 512, 4, 2, 64
    h32 = seeded((batch, H), 3).float()
    norm_w = (1 + 0.1 * seeded((H,), 4).float()).half()
    xw = (h32 * norm_w.float()).half()
    wq = seeded((qh * 128, H), 5, 0.05)
    wk = seeded((kvh * 128, H), 9, 0.05)
    wv = seeded((kvh * 128, H), 10, 0.05)
    w = torch.cat([wq, wk, wv])
    qn = (1 + 0.1 * seeded((128,), 6).float()).half() if qk_norm else None
    kn = (1 + 0.1 * seeded((128,), 7).float()).half() if qk_norm else None
    positions = torch.randint(0, max_seq, (batch,), generator=torch.Generator().manual_seed(8),
                              dtype=torch.int32)
    eps = 1e-6
    ssq = _norm_input(h32, batch)
    inv_freq = oracle.rope_inv_freq(1e6, 128)
    dev = "cuda"
    q = torch.empty(batch, qh * 128, dtype=torch.float16, device=dev)
    kc = torch.full((batch, kvh, max_seq, 128), 7.0, dtype=torch.float16, device=dev)
    vc = torch.full((batch, kvh, max_seq, 128), 7.0, dtype=torch.float16, device=dev)
    t = {n: v.to(dev) for n, v in dict(ssq=ssq, pos=positions, inv=inv_freq, qn=qn, kn=kn).items()
         if v is not None}
    e = _native.Epilogue(kind=_native.EPI_QKV, ssq_parts=4, ssq_ld=batch, hidden=H, ssq_eps=eps,
                         ld_out=qh * 128, q_heads=qh, kv_heads=kvh, max_seq=max_seq, qk_eps=eps)
    e.ssq_in, e.out, e.positions, e.inv_freq = _p(t["ssq"]), _p(q), _p(t["pos"]), _p(t["inv"])
    e.k_cache, e.v_cache = _p(kc), _p(vc)
    if qk_norm:
        e.q_norm_w, e.k_norm_w = _p(t["qn"]), _p(t["kn"])
    rows = w.shape[0]
    if packed:
        pairs = _native.PACK_HEAD_PAIRS
        wd = ops.pack_weight_rows([(wq.to(dev), pairs, 0), (wk.to(dev), pairs, qh * 128),
                                   (wv.to(dev), pairs, (qh + kvh) * 128)], rows)
    else:
        wd = _pair_order(w, qh + 2 * kvh).to(dev)
    ops.projection(xw.to(dev), wd, rows, e, packed=packed)
    # Oracle: RMSNorm(h) with norm_w, linear, QK-norm, RoPE.
    hn = oracle.rms_norm(h32, norm_w, eps)
    proj = oracle.linear(hn, w)
    qr = proj[:, :qh * 128].view(batch, qh, 128)
    kr = proj[:, qh * 128:(qh + kvh) * 128].view(batch, kvh, 128)
    vr = proj[:, (qh + kvh) * 128:].view(batch, kvh, 128)
    if qk_norm:
        qr = oracle.rms_norm(qr, qn, eps)
        kr = oracle.rms_norm(kr, kn, eps)
    cos, sin = oracle.rope_cos_sin(inv_freq, positions)
    qr, kr = oracle.apply_rope(qr, cos, sin), oracle.apply_rope(kr, cos, sin)
    _close(q.view(batch, qh, 128), qr)
    kcpu, vcpu = kc.cpu(), vc.cpu()
    for b in range(batch):
        p = int(positions[b])
        _close(kcpu[b, :, p], kr[b])
        _close(vcpu[b, :, p], vr[b])
        keep = torch.ones(max_seq, dtype=torch.bool)
        keep[p] = False
        assert bool((kcpu[b][:, keep] == 7.0).all()) and bool((vcpu[b][:, keep] == 7.0).all())


@pytest.mark.parametrize("batch", [1, 2, 16, 64])
@pytest.mark.parametrize("rows", [128, 16])
@pytest.mark.parametrize("packed", [False, True])
@pytest.mark.parametrize("K", [512, 384, 1280])
def test_residual_and_next_norm(cuda, batch, rows, packed, K):
    """K 384 / 1280 split unevenly over the GEMV's cluster members (a partial
    last stage; 1-2 stages per member)."""
    from llm_compiler_3_b200 import _native, ops
    H = 1024
    x = seeded((batch, K), 11)
    w = seeded((H, K), 12, 0.05)
    resid = seeded((batch, H), 13).float()
    norm_w = (1 + 0.1 * seeded((H,), 14).float()).half()
    dev = "cuda"
    r_d = resid.clone().to(dev)
    xw = torch.empty(batch, H, dtype=torch.float16, device=dev)
    ssq = torch.zeros(H // rows, batch, dtype=torch.float32, device=dev)
    nw = norm_w.to(dev)
    e = _native.Epilogue(kind=_native.EPI_RESID, ld_resid=H, ld_xw=H, ssq_out_ld=batch,
                         ssq_out_rows=rows)
    e.resid, e.norm_w, e.xw, e.ssq_out = _p(r_d), _p(nw), _p(xw), _p(ssq)
    wd = ops.pack_weight(w.to(dev)) if packed else w.to(dev)
    ops.projection(x.to(dev), wd, H, e, packed=packed)
    h = resid + oracle.linear(x, w)
    _close(r_d, h, atol=1e-3)
    _close(xw, h * norm_w.float())
    ref_ssq = (h * h).view(batch, H // rows, rows).sum(-1).t()
    torch.testing.assert_close(ssq.cpu(), ref_ssq, rtol=1e-4, atol=1e-3)


@pytest.mark.parametrize("batch", [1, 2, 16, 64])
@pytest.mark.parametrize("packed", [False, True])
def test_swiglu(cuda, batch, packed):
    from llm_compiler_3_b200 import _native, ops
    H, F = 512, 384
    h32 = seeded((batch, H), 21).float()
    xw = h32.half()
    gate = seeded((F, H), 22, 0.05)
    up = seeded((F, H), 23, 0.05)
    ssq = _norm_input(h32, batch)
    dev = "cuda"
    act = torch.empty(batch, F, dtype=torch.float16, device=dev)
    s_d = ssq.to(dev)
    e = _native.Epilogue(kind=_native.EPI_SWIGLU, ssq_parts=4, ssq_ld=batch, hidden=H,
                         ssq_eps=1e-5, ld_out=F)
    e.ssq_in, e.out = _p(s_d), _p(act)
    if packed:
        il = _native.PACK_INTERLEAVE
        wd = ops.pack_weight_rows([(gate.to(dev), il, 0), (up.to(dev), il, 1)], 2 * F)
    else:
        wd = _interleave(gate, up).to(dev)
    ops.projection(xw.to(dev), wd, 2 * F, e, packed=packed)
    hn = oracle.rms_norm(h32, torch.ones(H), 1e-5)
    ref = oracle.silu_mul(oracle.linear(hn, gate), oracle.linear(hn, up))
    _close(act, ref)


@pytest.mark.parametrize("batch", [1, 2, 16, 64])
@pytest.mark.parametrize("rows", [128, 16])
@pytest.mark.parametrize("vocab", [1000, 1008])
@pytest.mark.parametrize("packed", [False, True])
def test_argmax_partials(cuda, batch, rows, vocab, packed):
    """Per-`rows` partial (max, argmax); 1008 rows at batch 1-2 with 16-row
    partials and packed weights take the GEMV, 1000 the tensor cores."""
    from llm_compiler_3_b200 import _native, ops
    V, H = vocab, 256
    x = seeded((batch, H), 31)
    w = seeded((V, H), 32, 0.05)
    parts = (V + rows - 1) // rows
    dev = "cuda"
    val = torch.full((parts, batch), float("nan"), dtype=torch.float32, device=dev)
    idx = torch.full((parts, batch), -1, dtype=torch.int32, device=dev)
    e = _native.Epilogue(kind=_native.EPI_ARGMAX, am_ld=batch, am_rows=rows)
    e.am_val, e.am_idx = _p(val), _p(idx)
    wd = ops.pack_weight(w.to(dev)) if packed else w.to(dev)
    ops.projection(x.to(dev), wd, V, e, packed=packed)
    logits = oracle.linear(x, w)
    val_c, idx_c = val.cpu(), idx.cpu()
    for p in range(parts):      # every partial is its rows' argmax
        lo, hi = p * rows, min(V, (p + 1) * rows)
        ref_v, ref_i = logits[:, lo:hi].max(1)
        torch.testing.assert_close(val_c[p], ref_v, rtol=0, atol=1e-3)
        close = (idx_c[p].long() == ref_i + lo) | \
            ((logits[:, lo:hi].gather(1, (idx_c[p].long() - lo).clamp(0, hi - lo - 1)[:, None])[:, 0]
              - ref_v).abs() <= 1e-3)
        assert bool(close.all()) and bool(((idx_c[p] >= lo) & (idx_c[p] < hi)).all())
    best = val_c.max(0)
    got_ids = idx_c.gather(0, best.indices[None])[0]
    assert torch.equal(got_ids.long(), oracle.greedy_argmax(logits))
