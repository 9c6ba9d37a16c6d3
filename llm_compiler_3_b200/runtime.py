"""Host-side mirror of the decode runtime (libnpu_b200 contexts) for Python callers.

This plays, for the B200 path, the role the reference's driver scripts play for
the NPU path (examples/llama/verify.py:84-92: capture, compile, run, read the
output back): a plan plus the captured weights go in, decode steps come out.
torch provides device memory, streams and torch.distributed plumbing only.
"""
from __future__ import annotations

import ctypes
import tempfile
from pathlib import Path
from typing import Iterable, Mapping

import numpy as np
import torch

from . import _native
from .plan import DecodePlan

INFO_FIELDS = ("layers", "hidden", "q_heads", "kv_heads", "ffn", "vocab", "vocab_offset",
               "max_batch", "max_seq", "head_dim", "fingerprint", "tp_size", "peer_exchange")


class _DeviceArray:
    """Zero-copy view of library-owned device memory for torch.as_tensor."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str = "<f2"):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    _native.check(_native.lib().npu_b200_nccl_unique_id(buf))
    return buf.raw


class Decoder:
    """One libnpu_b200 context: a plan, this rank's weights and KV cache."""

    def __init__(self, plan: DecodePlan | str | Path, device: int = 0, tp_rank: int = 0,
                 tp_size: int = 1, nccl_id: bytes | None = None):
        self.lib = _native.lib()
        self.device = device
        self._ctx = ctypes.c_void_p()
        idbuf = ctypes.create_string_buffer(nccl_id, 128) if nccl_id is not None else None
        _native.check(self.lib.npu_b200_create(device, tp_rank, tp_size, idbuf,
                                               ctypes.byref(self._ctx)))
        if isinstance(plan, DecodePlan):
            self._tmp = tempfile.TemporaryDirectory(prefix="npu_b200_plan_")
            path = plan.write(Path(self._tmp.name) / "plan.txt")
        else:
            path = Path(plan)
        _native.check(self.lib.npu_b200_load_plan(self._ctx, str(path).encode()))
        self.info = self._info()

    def _info(self) -> dict:
        out = (ctypes.c_int64 * len(INFO_FIELDS))()
        _native.check(self.lib.npu_b200_plan_info(self._ctx, out, len(INFO_FIELDS)))
        return dict(zip(INFO_FIELDS, list(out)))

    # -- weights -----------------------------------------------------------
    def set_weight(self, name: str, tensor: torch.Tensor) -> None:
        """Copy one whole FP16 parameter (CPU or CUDA tensor) into this rank's layout."""
        if tensor.dtype != torch.float16:
            raise ValueError(f"{name}: weights must be float16, got {tensor.dtype}")
        t = tensor.contiguous()
        _native.check(self.lib.npu_b200_set_weight(self._ctx, name.encode(),
                                                   ctypes.c_void_p(t.data_ptr()),
                                                   t.numel() * 2))

    def set_weights(self, weights: Mapping[str, torch.Tensor] | Iterable) -> None:
        items = weights.items() if isinstance(weights, Mapping) else weights
        for name, t in items:
            self.set_weight(name, t)

    def save_image(self, directory: str | Path) -> None:
        """This rank's weights as a per-rank image under directory/rank<r>-of-<N>/."""
        _native.check(self.lib.npu_b200_save_image(self._ctx, str(directory).encode()))

    def load_image(self, directory: str | Path) -> None:
        """Every weight from a per-rank image written by save_image for this plan and rank."""
        _native.check(self.lib.npu_b200_load_image(self._ctx, str(directory).encode()))

    def load_capture(self, directory: str | Path) -> None:
        """Every weight of a capture directory (arguments.txt + arg<N>.bin)."""
        _native.check(self.lib.npu_b200_load_capture(self._ctx, str(directory).encode()))

    def kv_cache(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Views [max_batch, local kv heads, max_seq, head_dim] FP16 of one layer's cache."""
        k = ctypes.c_void_p()
        v = ctypes.c_void_p()
        _native.check(self.lib.npu_b200_kv_cache(self._ctx, layer, ctypes.byref(k),
                                                  ctypes.byref(v)))
        i = self.info
        shape = (i["max_batch"], i["kv_heads"], i["max_seq"], i["head_dim"])
        dev = torch.device("cuda", self.device)
        return (torch.as_tensor(_DeviceArray(k.value, shape), device=dev),
                torch.as_tensor(_DeviceArray(v.value, shape), device=dev))

    # -- decode --------------------------------------------------------------
    @staticmethod
    def _stream():
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def step(self, tokens, positions) -> np.ndarray:
        """One greedy decode step through host buffers; returns the next token ids."""
        tok = np.ascontiguousarray(np.asarray(tokens, dtype=np.int32))
        pos = np.ascontiguousarray(np.asarray(positions, dtype=np.int32))
        if tok.shape != pos.shape or tok.ndim != 1:
            raise ValueError("tokens and positions must be equal-length 1-D sequences")
        out = np.empty_like(tok)
        _native.check(self.lib.npu_b200_decode_step(
            self._ctx, tok.ctypes.data_as(ctypes.c_void_p), pos.ctypes.data_as(ctypes.c_void_p),
            len(tok), out.ctypes.data_as(ctypes.c_void_p), self._stream()))
        return out

    def step_device(self, tokens: torch.Tensor, positions: torch.Tensor,
                    out: torch.Tensor) -> torch.Tensor:
        """Asynchronous decode step on device int32 buffers (current stream)."""
        for t in (tokens, positions, out):
            if t.dtype != torch.int32 or not t.is_cuda or not t.is_contiguous():
                raise ValueError("device decode buffers must be contiguous CUDA int32")
        _native.check(self.lib.npu_b200_decode_step_device(
            self._ctx, ctypes.c_void_p(tokens.data_ptr()), ctypes.c_void_p(positions.data_ptr()),
            tokens.numel(), ctypes.c_void_p(out.data_ptr()), self._stream()))
        return out

    def forward_hidden(self, x: torch.Tensor, positions) -> torch.Tensor:
        """Layers only: x [B, hidden] FP16 (CPU) -> y [B, hidden] FP16 (CPU)."""
        x = x.to(torch.float16).contiguous().cpu()
        pos = np.ascontiguousarray(np.asarray(positions, dtype=np.int32))
        y = torch.empty_like(x)
        _native.check(self.lib.npu_b200_forward_hidden(
            self._ctx, ctypes.c_void_p(x.data_ptr()), pos.ctypes.data_as(ctypes.c_void_p),
            x.shape[0], ctypes.c_void_p(y.data_ptr()), self._stream()))
        return y

    def forward_hidden_device(self, x: torch.Tensor, positions: torch.Tensor,
                              out: torch.Tensor) -> torch.Tensor:
        _native.check(self.lib.npu_b200_forward_hidden_device(
            self._ctx, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(positions.data_ptr()),
            x.shape[0], ctypes.c_void_p(out.data_ptr()), self._stream()))
        return out

    def close(self) -> None:
        if self._ctx:
            _native.check(self.lib.npu_b200_destroy(self._ctx))
            self._ctx = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass


class GraphRunner:
    """A graph plan (``graph.capture_graph``) loaded into its own libnpu_b200
    context: the B200 counterpart of compiling a capture and running the
    program with the captured arguments (examples/pytorch/mlp.py)."""

    def __init__(self, directory: str | Path, device: int = 0):
        from .graph import GraphPlan
        self.lib = _native.lib()
        self.device = device
        self.directory = Path(directory)
        self.plan = GraphPlan.parse((self.directory / "graph.txt").read_text())
        self._ctx = ctypes.c_void_p()
        _native.check(self.lib.npu_b200_create(device, 0, 1, None, ctypes.byref(self._ctx)))
        try:
            _native.check(self.lib.npu_b200_load_graph(self._ctx, str(self.directory).encode()))
        except Exception:
            self.close()
            raise

    def run(self, *inputs: torch.Tensor, outs: Iterable[torch.Tensor] | None = None
            ) -> list[torch.Tensor]:
        """Run the graph on CUDA FP16 inputs (graph.txt order) on the current
        stream; returns the outputs (allocated unless `outs` is given)."""
        dev = torch.device("cuda", self.device)
        if len(inputs) != len(self.plan.inputs):
            raise ValueError(f"graph takes {len(self.plan.inputs)} inputs, got {len(inputs)}")
        for name, t in zip(self.plan.inputs, inputs):
            want = self.plan.tensors[name][1]
            if t.dtype != torch.float16 or not t.is_cuda or not t.is_contiguous() or \
                    t.numel() != int(np.prod(want)):
                raise ValueError(f"input {name}: need a contiguous CUDA float16 tensor of {want}")
        if outs is None:
            outs = [torch.empty(self.plan.tensors[n][1], dtype=torch.float16, device=dev)
                    for n in self.plan.outputs]
        outs = list(outs)
        args = (ctypes.c_void_p * max(1, len(inputs)))(*[t.data_ptr() for t in inputs])
        res = (ctypes.c_void_p * max(1, len(outs)))(*[t.data_ptr() for t in outs])
        _native.check(self.lib.npu_b200_run_graph(
            self._ctx, args, res, ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)))
        return outs

    def close(self) -> None:
        if self._ctx:
            _native.check(self.lib.npu_b200_destroy(self._ctx))
            self._ctx = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass
