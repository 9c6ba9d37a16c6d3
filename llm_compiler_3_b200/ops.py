"""Kernel-level operators over torch CUDA tensors, calling the C ABI.

torch is used for device memory and the current stream only; every operator
here runs a libnpu_b200 kernel and nothing else.  Inputs must be CUDA, FP16
(unless stated), contiguous; violations raise before anything is launched.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native

_workspaces: dict[tuple[int, int], torch.Tensor] = {}


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _require(t: torch.Tensor, name: str, dtype=torch.float16, ndim: int | None = None) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if ndim is not None and t.dim() != ndim:
        raise ValueError(f"{name} must have {ndim} dims, got {tuple(t.shape)}")


def workspace(nbytes: int, device: torch.device, slot: int = 0) -> torch.Tensor:
    """A zero-filled, 256-byte aligned scratch buffer of at least nbytes, cached
    per (device, slot).  Kernels that use one leave it zero-filled again."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), slot)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


def flash_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 seq_lens: torch.Tensor, scale: float | None = None, num_splits: int = 0,
                 out: torch.Tensor | None = None, workspace_buf: torch.Tensor | None = None
                 ) -> torch.Tensor:
    """Split-KV flash-decoding: q [B, Hq, D], caches [B, Hkv, S, D], seq_lens [B] int32.

    Returns out [B, Hq, D] FP16 = softmax(scale q K^T) V over keys [0, seq_lens[b])."""
    _require(q, "q", ndim=3)
    _require(k_cache, "k_cache", ndim=4)
    _require(v_cache, "v_cache", ndim=4)
    _require(seq_lens, "seq_lens", dtype=torch.int32, ndim=1)
    batch, q_heads, head_dim = q.shape
    _, kv_heads, max_seq, d2 = k_cache.shape
    if v_cache.shape != k_cache.shape or d2 != head_dim or k_cache.shape[0] != batch:
        raise ValueError("k_cache / v_cache / q shapes disagree")
    if seq_lens.shape[0] != batch:
        raise ValueError("seq_lens must have one entry per sequence")
    if scale is None:
        scale = head_dim ** -0.5
    if out is None:
        out = torch.empty_like(q)
    else:
        _require(out, "out", ndim=3)
    lib = _native.lib()
    need = lib.npu_b200_flash_decode_workspace_size(batch, kv_heads, head_dim, max_seq, num_splits)
    ws = workspace_buf if workspace_buf is not None else (
        workspace(need, q.device) if need else None)
    _native.check(lib.npu_b200_flash_decode(
        _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(seq_lens), _ptr(out), batch, q_heads,
        kv_heads, head_dim, max_seq, float(scale), int(num_splits), _ptr(ws),
        ws.numel() if ws is not None else 0, _stream()))
    return out


def prefill_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                      keys: int | None = None, q_start: torch.Tensor | None = None,
                      causal: bool = False, scale: float | None = None,
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """Multi-query attention on tcgen05: q [B, Hq, M, D], caches [B, Hkv, S, D].

    out[b, h, i] = softmax(scale q K^T) V over keys j < keys (default S) and, when
    causal, j <= q_start[b] + i (q_start [B] int32, default 0: torch's is_causal).
    Returns out [B, Hq, M, D] FP16; a row that sees no key is zero."""
    _require(q, "q", ndim=4)
    _require(k_cache, "k_cache", ndim=4)
    _require(v_cache, "v_cache", ndim=4)
    batch, q_heads, queries, head_dim = q.shape
    _, kv_heads, max_seq, d2 = k_cache.shape
    if v_cache.shape != k_cache.shape or d2 != head_dim or k_cache.shape[0] != batch:
        raise ValueError("k_cache / v_cache / q shapes disagree")
    if q_start is not None:
        _require(q_start, "q_start", dtype=torch.int32, ndim=1)
        if q_start.shape[0] != batch:
            raise ValueError("q_start must have one entry per sequence")
    if keys is None:
        keys = max_seq
    if scale is None:
        scale = head_dim ** -0.5
    if out is None:
        out = torch.empty_like(q)
    else:
        _require(out, "out", ndim=4)
        if out.shape != q.shape:
            raise ValueError("out must have q's shape")
    _native.check(_native.lib().npu_b200_prefill_attention(
        _ptr(q), _ptr(k_cache), _ptr(v_cache), _ptr(q_start), _ptr(out), batch, q_heads,
        kv_heads, head_dim, queries, int(keys), max_seq, float(scale), 1 if causal else 0,
        _stream()))
    return out


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
           relu: bool = False, out_dtype: torch.dtype = torch.float16,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """out[b, n] = act(x[b, :] . weight[n, :] + bias[n]) on tcgen05 tensor cores.

    x [B, K] FP16 (B <= 128), weight [N, K] FP16 (torch Linear layout, K % 64 == 0),
    bias [N] FP16 or None; FP32 accumulation; out FP16 or FP32 [B, N]."""
    _require(x, "x", ndim=2)
    _require(weight, "weight", ndim=2)
    batch, k = x.shape
    n_rows = weight.shape[0]
    if weight.shape[1] != k:
        raise ValueError(f"x is [{batch}, {k}] but weight is {tuple(weight.shape)}")
    if bias is not None:
        _require(bias, "bias", ndim=1)
    if out_dtype not in (torch.float16, torch.float32):
        raise ValueError("out_dtype must be float16 or float32")
    if out is None:
        out = torch.empty(batch, n_rows, dtype=out_dtype, device=x.device)
    else:
        _require(out, "out", dtype=out_dtype, ndim=2)
    flags = (_native.LINEAR_RELU if relu else 0) | (
        _native.LINEAR_OUT_F32 if out_dtype == torch.float32 else 0)
    lib = _native.lib()
    need = lib.npu_b200_linear_workspace_size(n_rows, k, batch)
    ws = workspace(need, x.device, slot=1)
    _native.check(lib.npu_b200_linear(_ptr(x), _ptr(weight), _ptr(bias), _ptr(out), batch,
                                      n_rows, k, flags, _ptr(ws), ws.numel(), _stream()))
    return out


def pack_weight(weight: torch.Tensor) -> torch.Tensor:
    """Weight panels of weight [N, K] (see npu_b200_pack_weight): a flat uint8
    tensor of 16 KB blocks streamed by one bulk copy each."""
    _require(weight, "weight", ndim=2)
    n, k = weight.shape
    lib = _native.lib()
    out = torch.empty(lib.npu_b200_packed_weight_bytes(n, k), dtype=torch.uint8,
                      device=weight.device)
    _native.check(lib.npu_b200_pack_weight(_ptr(weight), n, k, _ptr(out), _stream()))
    return out


def pack_weight_rows(parts, rows: int) -> torch.Tensor:
    """Panels of `rows` rows assembled from (weight [n_i, K], order, row_offset)
    parts (see npu_b200_pack_weight_rows), e.g. [(gate, PACK_INTERLEAVE, 0),
    (up, PACK_INTERLEAVE, 1)] for the SwiGLU epilogue."""
    k = parts[0][0].shape[1]
    lib = _native.lib()
    out = torch.zeros(lib.npu_b200_packed_weight_bytes(rows, k), dtype=torch.uint8,
                      device=parts[0][0].device)
    for weight, order, offset in parts:
        _require(weight, "weight", ndim=2)
        if weight.shape[1] != k:
            raise ValueError("pack_weight_rows: parts differ in K")
        _native.check(lib.npu_b200_pack_weight_rows(_ptr(weight), weight.shape[0], k, _ptr(out),
                                                    rows, order, offset, _stream()))
    return out


def projection(x: torch.Tensor, weight: torch.Tensor, n_rows: int, epilogue,
               packed: bool = False) -> None:
    """Run npu_b200_projection with a filled _native.Epilogue (pointers set by the
    caller).  x [B, K] FP16; weight [n_rows, K] FP16 or its packed panels."""
    _require(x, "x", ndim=2)
    batch, k = x.shape
    lib = _native.lib()
    need = lib.npu_b200_linear_workspace_size(n_rows, k, batch)
    ws = workspace(need, x.device, slot=1)
    _native.check(lib.npu_b200_projection(_ptr(x), _ptr(weight), 1 if packed else 0, batch,
                                          n_rows, k, ctypes.byref(epilogue), _ptr(ws),
                                          ws.numel(), _stream()))
