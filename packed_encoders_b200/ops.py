"""Torch-facing entry points of the B200 packed attention backend.

Each function validates shapes on the host (no device syncs, no reads of ``cu_seqlens``
values), fills the C ABI parameter block and enqueues the sm_100a kernels on
``torch.cuda.current_stream()``. Nothing here computes attention itself: a missing or
unloadable ``libpe_b200.so`` raises ``PackedEncodersError``.

Reference interfaces mirrored (packed-encoders 0.3.0):
  packed_short_attention(q, k, v, cu_seqlens, max_seqlen, *, half_window, softmax_scale)
      packed_encoders/_kernels/triton_packed_attention.py:175-196
  attention_bshd(q, k, v, *, window, scaling, cu_seqlens, max_seqlen, backend)
      packed_encoders/ops.py:502-538
  flash_attention_varlen(q, k, v, cu_seqlens, max_seqlen, window, scaling)
      packed_encoders/ops.py:432-461
"""

from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass

import torch
from torch import Tensor

from packed_encoders_b200 import _lib
from packed_encoders_b200.errors import PackedEncodersError, UnsupportedTargetError

SUPPORTED_HEAD_DIMS = (64, 128, 256)
_WORKSPACES: dict[tuple[int, int], Tensor] = {}


def _ptr(t: Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _workspace(device: torch.device, stream: torch.cuda.Stream, nbytes: int) -> Tensor:
    """One growing workspace per (device, stream): calls on a stream run in order, so the
    schedule of one call is never overwritten while a kernel still reads it."""
    key = (device.index, stream.cuda_stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws


def _check_qkv(q: Tensor, k: Tensor, v: Tensor) -> None:
    if q.ndim != 3 or k.ndim != 3 or v.ndim != 3:
        raise UnsupportedTargetError("b200 attention takes [tokens, heads, head_dim] q/k/v")
    if k.shape != v.shape or q.shape[2] != k.shape[2] or q.shape[1] % k.shape[1]:
        raise UnsupportedTargetError("b200 attention requires matching head_dim, k.shape == v.shape and an "
                                     "integer GQA ratio")
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16:
        raise UnsupportedTargetError("b200 attention is bf16 (fp32 accumulation)")
    if not (q.is_cuda and k.is_cuda and v.is_cuda) or not (q.device == k.device == v.device):
        raise UnsupportedTargetError("b200 attention needs q/k/v on one CUDA device")
    if q.shape[2] not in SUPPORTED_HEAD_DIMS:
        raise UnsupportedTargetError(f"b200 attention supports head_dim {SUPPORTED_HEAD_DIMS}, got {q.shape[2]}")
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.stride(2) != 1:
            raise UnsupportedTargetError(f"{name} must have a contiguous head_dim")
        if (t.stride(0) * 2) % 16 or (t.stride(1) * 2) % 16 or t.data_ptr() % 16:
            raise UnsupportedTargetError(f"{name} strides / base must be 16-byte aligned (TMA)")


@dataclass(frozen=True)
class LaunchShape:
    """Host-visible shape of one call (never derived from device values)."""

    n_seq: int
    total_q: int
    total_k: int
    max_seqlen_q: int
    max_seqlen_k: int


LAUNCHES = {"kernels": 0}  # kernels enqueued by this module (bench / test bookkeeping)


def _count(n: int) -> None:
    LAUNCHES["kernels"] += n


def _extra_passes(rope, gate) -> int:
    """Kernels a call launches besides the schedule build and the attention kernel: the RoPE pass,
    and the output-gate pass unless the gate is fused into the epilogue (PE_B200_GATE=fused, which
    the library reads once per process)."""
    gate_pass = gate is not None and os.environ.get("PE_B200_GATE") != "fused"
    return (1 if rope is not None else 0) + (1 if gate_pass else 0)


class AttentionPlan:
    """A device tile schedule built once for one set of segment boundaries and one attention
    kind (window / causal / head_dim), reusable by every layer of a forward that shares them
    (e.g. all global layers of a packed ModernBERT forward). Building enqueues two small
    kernels on the current stream and reads no device values on the host, so it can be
    captured in a CUDA graph. Calls that use the plan must run on the same stream (or after
    it) and must not overlap with a rebuild of it."""

    def __init__(self, cu_seqlens: Tensor, max_seqlen: int, *, total_q: int, total_k: int | None = None,
                 head_dim: int, window: tuple[int, int] = (-1, -1), causal: bool = False,
                 cu_seqlens_k: Tensor | None = None, max_seqlen_k: int | None = None):
        if head_dim not in SUPPORTED_HEAD_DIMS:
            raise UnsupportedTargetError(f"b200 attention supports head_dim {SUPPORTED_HEAD_DIMS}, got {head_dim}")
        self.cu_q = cu_seqlens
        self.cu_k = cu_seqlens if cu_seqlens_k is None else cu_seqlens_k
        self.max_q = int(max_seqlen)
        self.max_k = int(max_seqlen if max_seqlen_k is None else max_seqlen_k)
        self.total_q = int(total_q)
        self.total_k = int(total_q if total_k is None else total_k)
        self.head_dim = int(head_dim)
        self.window = tuple(int(w) for w in window)
        self.causal = bool(causal)
        self.workspace: Tensor | None = None
        self.build()

    def key(self):
        return (self.cu_q.data_ptr(), self.cu_k.data_ptr(), self.total_q, self.total_k, self.head_dim, self.window,
                self.causal)

    def _params(self) -> _lib.PeB200AttnParams:
        return _lib.PeB200AttnParams(
            cu_seqlens_q=_ptr(self.cu_q), cu_seqlens_k=_ptr(self.cu_k), n_seq=self.cu_q.numel() - 1,
            total_q=self.total_q, total_k=self.total_k, max_seqlen_q=self.max_q, max_seqlen_k=self.max_k,
            heads=1, kv_heads=1, head_dim=self.head_dim, window_left=self.window[0], window_right=self.window[1],
            causal=int(self.causal), q_stride_token=8, q_stride_head=8, k_stride_token=8, k_stride_head=8,
            v_stride_token=8, v_stride_head=8, o_stride_token=8, o_stride_head=8, scale=1.0)

    def build(self) -> None:
        params = self._params()
        so = _lib.lib()
        nbytes = ctypes.c_size_t(0)
        _lib.check(so.pe_b200_attn_workspace_size(ctypes.byref(params), ctypes.byref(nbytes)), "workspace size")
        device = self.cu_q.device
        if self.workspace is None or self.workspace.numel() < nbytes.value:
            self.workspace = torch.empty(max(nbytes.value, 1 << 12), dtype=torch.uint8, device=device)
        params.workspace = self.workspace.data_ptr()
        params.workspace_bytes = self.workspace.numel()
        with torch.cuda.device(device):
            stream = torch.cuda.current_stream(device)
            _lib.check(so.pe_b200_build_schedule(ctypes.byref(params), ctypes.c_void_p(stream.cuda_stream)),
                       "pe_b200_build_schedule")
        _count(1)

    def error_word(self) -> int:
        """Synchronising read of the device error word of the last build / run on this plan."""
        return int(self.workspace[4:8].view(torch.int32).item())


def plan_attention(q: Tensor, k: Tensor, cu_seqlens: Tensor, max_seqlen: int, *, window=(-1, -1), causal=False,
                   cu_seqlens_k: Tensor | None = None, max_seqlen_k: int | None = None) -> AttentionPlan:
    """Build the tile schedule for ``packed_attention(q, k, v, cu_seqlens, ..., plan=...)``."""
    return AttentionPlan(cu_seqlens, max_seqlen, total_q=q.shape[0], total_k=k.shape[0], head_dim=q.shape[2],
                         window=window, causal=causal, cu_seqlens_k=cu_seqlens_k, max_seqlen_k=max_seqlen_k)


def packed_attention(
    q: Tensor,
    k: Tensor,
    v: Tensor,
    cu_seqlens: Tensor,
    max_seqlen: int,
    *,
    scale: float | None = None,
    window: tuple[int, int] = (-1, -1),
    causal: bool = False,
    cu_seqlens_k: Tensor | None = None,
    max_seqlen_k: int | None = None,
    out: Tensor | None = None,
    return_lse: bool = False,
    plan: AttentionPlan | None = None,
    gate: Tensor | None = None,
    rope: tuple[Tensor, Tensor] | None = None,
):
    """Packed variable-length attention on B200.

    q ``[Tq, H, D]``, k/v ``[Tk, KV, D]`` bf16 (any token/head strides, D contiguous);
    ``cu_seqlens`` int32 ``[N + 1]`` on the same device. ``cu_seqlens_k`` (default: the same)
    gives key segments; a query segment shorter than its key segment is aligned to the end of
    it (the reference's prefixed form, runtime/attention.py:242-261). ``window`` is
    ``(left, right)`` with -1 unbounded (runtime/attention.py:157-170). Returns ``out``
    ``[Tq, H, D]`` bf16, and with ``return_lse`` also the fp32 natural-log LSE ``[H, Tq]``.
    ``plan`` (from ``plan_attention``) reuses an already built tile schedule.
    ``gate`` ``[Tq, H, D]`` bf16 (D contiguous) applies the Qwen3.5 output gate in the same call:
    ``out = bf16(o * bf16(sigmoid(gate)))`` with ``o`` the bf16 attention output, the roundings
    of the reference's ``sigmoid_gate`` (_kernels/hybrid.py:196-205); the LSE is not gated.
    ``rope`` ``(cos, sin)``, each ``[Tq, D]`` bf16 per-token tables (D contiguous, one row
    stride): q and k are given un-rotated (e.g. views of the fused qkv projection); the call
    rotates them (the reference's rotate-half rule of ``apply_rope_bshd``, _kernels/rope.py:140-200,
    used at forward.py:199-205) into its workspace with this library's rope pass, then attends.
    head_dim 64, self-attention (no ``cu_seqlens_k``), no ``plan``.
    """
    _check_qkv(q, k, v)
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad or v.requires_grad):
        if (q.shape[2] != 64 or k.shape[1] != q.shape[1] or cu_seqlens_k is not None or gate is not None
                or rope is not None or plan is not None or out is not None or return_lse):
            raise UnsupportedTargetError("b200 attention with autograd: head_dim 64 self-attention with heads == "
                                         "kv_heads, no gate / rope / plan / out / return_lse")
        scale_ = float(q.shape[2] ** -0.5 if scale is None else scale)
        return _PackedAttentionFn.apply(q, k, v, cu_seqlens, int(max_seqlen), scale_,
                                        tuple(int(w) for w in window), bool(causal))
    cu_k = cu_seqlens if cu_seqlens_k is None else cu_seqlens_k
    for name, cu in (("cu_seqlens", cu_seqlens), ("cu_seqlens_k", cu_k)):
        if cu.dtype != torch.int32 or cu.ndim != 1 or cu.numel() < 1 or cu.device != q.device:
            raise UnsupportedTargetError(f"{name} must be a 1-D int32 tensor on {q.device}")
        if not cu.is_contiguous():
            raise UnsupportedTargetError(f"{name} must be contiguous")
    if cu_k.numel() != cu_seqlens.numel():
        raise UnsupportedTargetError("cu_seqlens and cu_seqlens_k must describe the same number of segments")
    left, right = (int(w) for w in window)
    if left < -1 or right < -1:
        raise UnsupportedTargetError("window entries must be >= -1")
    tq, heads, dim = q.shape
    tk, kv_heads, _ = k.shape
    if out is None:
        out = torch.empty((tq, heads, dim), dtype=q.dtype, device=q.device)
    elif out.shape != q.shape or out.dtype != q.dtype or out.stride(2) != 1 or out.device != q.device:
        raise UnsupportedTargetError("out must match q's shape/dtype with a contiguous head_dim")
    if rope is not None:
        cos, sin = rope
        if (cos.shape != (tq, dim) or sin.shape != cos.shape or cos.dtype != torch.bfloat16
                or sin.dtype != torch.bfloat16 or cos.stride(1) != 1 or sin.stride(1) != 1
                or cos.stride(0) != sin.stride(0) or cos.device != q.device or sin.device != q.device):
            raise UnsupportedTargetError("rope tables must be bf16 [Tq, D] with a contiguous D and one row stride")
        if dim != 64 or cu_seqlens_k is not None or tk != tq:
            raise UnsupportedTargetError("rope: head_dim 64 self-attention only")
        if plan is not None:
            raise UnsupportedTargetError("rope calls keep the rotated q/k in their own workspace: omit plan")
    if gate is not None and (gate.shape != q.shape or gate.dtype != torch.bfloat16 or gate.stride(2) != 1
                             or gate.device != q.device):
        raise UnsupportedTargetError("gate must be bf16 with q's shape and a contiguous head_dim")
    lse = torch.empty((heads, tq), dtype=torch.float32, device=q.device) if return_lse else None
    n_seq = cu_seqlens.numel() - 1
    if tq == 0 or n_seq == 0:
        if lse is not None:
            lse.fill_(float("-inf"))
        return (out, lse) if return_lse else out
    if tk == 0:
        raise UnsupportedTargetError("queries without keys")
    params = _lib.PeB200AttnParams(
        q=_ptr(q), k=_ptr(k), v=_ptr(v), out=_ptr(out), lse=_ptr(lse),
        cu_seqlens_q=_ptr(cu_seqlens), cu_seqlens_k=_ptr(cu_k),
        n_seq=n_seq, total_q=tq, total_k=tk,
        max_seqlen_q=int(max_seqlen), max_seqlen_k=int(max_seqlen_k if max_seqlen_k is not None else max_seqlen),
        heads=heads, kv_heads=kv_heads, head_dim=dim,
        q_stride_token=q.stride(0), q_stride_head=q.stride(1),
        k_stride_token=k.stride(0), k_stride_head=k.stride(1),
        v_stride_token=v.stride(0), v_stride_head=v.stride(1),
        o_stride_token=out.stride(0), o_stride_head=out.stride(1),
        scale=float(dim ** -0.5 if scale is None else scale),
        window_left=left, window_right=right, causal=int(bool(causal)),
    )
    if gate is not None:
        params.gate = _ptr(gate)
        params.g_stride_token, params.g_stride_head = gate.stride(0), gate.stride(1)
    if rope is not None:
        params.rope_cos, params.rope_sin = _ptr(rope[0]), _ptr(rope[1])
        params.rope_stride_token = rope[0].stride(0)
    so = _lib.lib()
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device)
        if plan is not None:
            if plan.key() != (cu_seqlens.data_ptr(), cu_k.data_ptr(), tq, tk, dim, (left, right), bool(causal)):
                raise UnsupportedTargetError("plan was built for other segments / window / causal / head_dim")
            params.workspace = plan.workspace.data_ptr()
            params.workspace_bytes = plan.workspace.numel()
            _lib.check(so.pe_b200_attn_run(ctypes.byref(params), ctypes.c_void_p(stream.cuda_stream)),
                       "pe_b200_attn_run")
            _count(1 + _extra_passes(rope, gate))
        else:
            nbytes = ctypes.c_size_t(0)
            _lib.check(so.pe_b200_attn_workspace_size(ctypes.byref(params), ctypes.byref(nbytes)), "workspace size")
            ws = _workspace(q.device, stream, nbytes.value)
            params.workspace = ws.data_ptr()
            params.workspace_bytes = ws.numel()
            _lib.check(so.pe_b200_attn_fwd(ctypes.byref(params), ctypes.c_void_p(stream.cuda_stream)),
                       "pe_b200_attn_fwd")
            _count(2 + _extra_passes(rope, gate))  # schedule build + attention
    return (out, lse) if return_lse else out


def packed_attention_backward(dout: Tensor, q: Tensor, k: Tensor, v: Tensor, out: Tensor, lse: Tensor,
                              cu_seqlens: Tensor, max_seqlen: int, *, scale: float, window=(-1, -1),
                              causal: bool = False) -> tuple[Tensor, Tensor, Tensor]:
    """Gradients (dq, dk, dv) of ``out = packed_attention(q, k, v, cu_seqlens, max_seqlen, scale=scale,
    window=window, causal=causal)`` given ``dout``, ``out`` and the forward's ``lse`` ([H, T] fp32,
    ``return_lse=True``): the tcgen05 backward kernel of this library (head_dim 64, heads == kv_heads,
    one ``cu_seqlens``). The reference has no counterpart: its training path keeps SDPA's backward
    (packed_encoders/pack.py:231-235)."""
    for name, t in (("dout", dout), ("out", out)):
        if t.shape != q.shape or t.dtype != torch.bfloat16 or t.stride(2) != 1 or t.device != q.device:
            raise UnsupportedTargetError(f"{name} must be bf16 with q's shape and a contiguous head_dim")
    _check_qkv(q, k, v)
    tq, heads, dim = q.shape
    if dim != 64 or k.shape[1] != heads or k.shape[0] != tq:
        raise UnsupportedTargetError("b200 backward: head_dim 64 self-attention with heads == kv_heads")
    if lse.shape != (heads, tq) or lse.dtype != torch.float32 or not lse.is_contiguous():
        raise UnsupportedTargetError("lse must be the forward's contiguous fp32 [H, T]")
    if cu_seqlens.dtype != torch.int32 or cu_seqlens.ndim != 1 or not cu_seqlens.is_contiguous():
        raise UnsupportedTargetError("cu_seqlens must be a contiguous 1-D int32 tensor")
    dq, dk, dv = (torch.empty_like(t, memory_format=torch.contiguous_format) for t in (q, k, v))
    n_seq = cu_seqlens.numel() - 1
    if tq == 0 or n_seq == 0:
        return dq.zero_(), dk.zero_(), dv.zero_()
    params = _lib.PeB200AttnBwdParams(
        q=_ptr(q), k=_ptr(k), v=_ptr(v), out=_ptr(out), dout=_ptr(dout), lse=_ptr(lse), dq=_ptr(dq), dk=_ptr(dk),
        dv=_ptr(dv), cu_seqlens=_ptr(cu_seqlens), n_seq=n_seq, total=tq, max_seqlen=int(max_seqlen), heads=heads,
        head_dim=dim, q_stride_token=q.stride(0), q_stride_head=q.stride(1), k_stride_token=k.stride(0),
        k_stride_head=k.stride(1), v_stride_token=v.stride(0), v_stride_head=v.stride(1),
        o_stride_token=out.stride(0), o_stride_head=out.stride(1), do_stride_token=dout.stride(0),
        do_stride_head=dout.stride(1), dq_stride_token=dq.stride(0), dq_stride_head=dq.stride(1),
        dk_stride_token=dk.stride(0), dk_stride_head=dk.stride(1), dv_stride_token=dv.stride(0),
        dv_stride_head=dv.stride(1), scale=float(scale), window_left=int(window[0]), window_right=int(window[1]),
        causal=int(bool(causal)))
    so = _lib.lib()
    nbytes = ctypes.c_size_t(0)
    _lib.check(so.pe_b200_attn_bwd_workspace_size(ctypes.byref(params), ctypes.byref(nbytes)), "bwd workspace size")
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=q.device)
    params.workspace, params.workspace_bytes = ws.data_ptr(), ws.numel()
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device)
        _lib.check(so.pe_b200_attn_bwd(ctypes.byref(params), ctypes.c_void_p(stream.cuda_stream)), "pe_b200_attn_bwd")
    _count(4)  # per-row prep, schedule build, backward, dq conversion
    return dq, dk, dv  # the workspace returns to torch's stream-ordered allocator


class _PackedAttentionFn(torch.autograd.Function):
    """packed_attention with a backward on this library's kernels (head_dim 64 self-attention)."""

    @staticmethod
    def forward(ctx, q, k, v, cu_seqlens, max_seqlen, scale, window, causal):
        with torch.no_grad():
            out, lse = packed_attention(q, k, v, cu_seqlens, max_seqlen, scale=scale, window=window, causal=causal,
                                        return_lse=True)
        ctx.save_for_backward(q, k, v, out, lse, cu_seqlens)
        ctx.cfg = (max_seqlen, scale, window, causal)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse, cu = ctx.saved_tensors
        max_seqlen, scale, window, causal = ctx.cfg
        dq, dk, dv = packed_attention_backward(dout.contiguous(), q, k, v, out, lse, cu, max_seqlen, scale=scale,
                                               window=window, causal=causal)
        return dq, dk, dv, None, None, None, None, None


def device_error_word(device: torch.device | int | None = None) -> int:
    """Read (synchronising) the device error word of the current stream's workspace: 0 when
    the last call saw no bounded-wait timeout, schedule overflow or malformed cu_seqlens."""
    device = torch.device("cuda", torch.cuda.current_device() if device is None else
                          (device if isinstance(device, int) else device.index))
    stream = torch.cuda.current_stream(device)
    ws = _WORKSPACES.get((device.index, stream.cuda_stream))
    if ws is None:
        return 0
    return int(ws[4:8].view(torch.int32).item())


def packed_short_attention(q, k, v, cu_seqlens, max_seqlen, *, half_window, softmax_scale):
    """Drop-in for triton_packed_attention.packed_short_attention (same arguments and return:
    contiguous ``[M, H, D]``). The envelope is wider: any H, D in (64, 128, 256), any length."""
    window = (-1, -1) if half_window is None else (int(half_window), int(half_window))
    return packed_attention(q, k, v, cu_seqlens, max_seqlen, scale=softmax_scale, window=window)


def packed_short_attention_supported(q, k, v, cu_seqlens, max_seqlen, *, half_window) -> bool:
    """Capability predicate with the reference's signature (triton_packed_attention.py:146-172)."""
    try:
        _check_qkv(q, k, v)
    except PackedEncodersError:
        return False
    return (cu_seqlens.is_cuda and cu_seqlens.dtype == torch.int32 and cu_seqlens.ndim == 1
            and cu_seqlens.numel() >= 2 and int(max_seqlen) > 0
            and (half_window is None or int(half_window) >= 0)
            and not torch.is_grad_enabled())


def _row_segments(batch: int, seq: int, device: torch.device) -> Tensor:
    """cu_seqlens of a rectangular batch read as ``batch`` sequences of ``seq`` tokens each; built on
    the device with no host synchronisation, so a CUDA-graph capture can contain it."""
    return torch.arange(0, (batch + 1) * seq, seq, dtype=torch.int32, device=device)


def _rectangular(q: Tensor, k: Tensor, v: Tensor, window, scaling) -> Tensor:
    """``[B, S, H, D]`` q/k/v of an unpadded batch: every row is one sequence of S tokens (the
    reference's dense flash call makes the same assumption, ops.py:404-409). Returns ``[B, S, H*D]``."""
    b, s, h, d = q.shape
    if k.shape[:2] != (b, s) or v.shape[:2] != (b, s):
        raise UnsupportedTargetError("rectangular b200 attention needs q, k and v with the same [B, S]")
    flat = [t.reshape(b * s, t.shape[2], d) for t in (q, k, v)]  # a view when the rows are evenly strided
    out = packed_attention(*flat, _row_segments(b, s, q.device), s, scale=scaling, window=tuple(window))
    return out.reshape(b, s, h * d)


def attention_bshd(q, k, v, *, window, scaling, cu_seqlens=None, max_seqlen=None, backend="b200"):
    """Drop-in for packed_encoders.ops.attention_bshd (ops.py:502-538): ``[1, T, H, D]`` views and
    ``cu_seqlens`` in, ``[1, T, H*D]`` out; without ``cu_seqlens`` a ``[B, S, H, D]`` unpadded batch
    (each row one sequence, like the reference's dense flash call) in, ``[B, S, H*D]`` out."""
    if backend != "b200":
        raise UnsupportedTargetError(f"packed_encoders_b200.attention_bshd serves backend 'b200', not {backend!r}")
    if cu_seqlens is None:
        if q.ndim != 4:
            raise UnsupportedTargetError("rectangular b200 attention_bshd takes [B, S, H, D] q/k/v")
        return _rectangular(q, k, v, window, scaling)
    qf, kf, vf = q.squeeze(0), k.squeeze(0), v.squeeze(0)
    out = packed_attention(qf, kf, vf, cu_seqlens, int(max_seqlen), scale=scaling, window=tuple(window))
    return out.reshape(1, out.shape[0], -1)


def flash_attention(q, k, v, window, scaling):
    """Drop-in for packed_encoders.ops.flash_attention (ops.py:404-430): ``[B, H, S, D]`` views of an
    unpadded batch in (every row one sequence of S tokens; the window as given per layer),
    ``[B, S, H*D]`` out. Differentiable (head_dim 64), so the reference's rectangular training graph
    (train_graph.py:170-181) can run on these kernels."""
    if q.ndim != 4:
        raise UnsupportedTargetError("b200 flash_attention takes [B, H, S, D] q/k/v")
    return _rectangular(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), window, scaling)


def flash_attention_varlen(q, k, v, cu_seqlens, max_seqlen, window, scaling):
    """Drop-in for packed_encoders.ops.flash_attention_varlen (ops.py:432-461): ``[1, H, T, D]``
    views in, ``[1, T, H*D]`` out."""
    qt, kt, vt = (t.squeeze(0).transpose(0, 1) for t in (q, k, v))
    out = packed_attention(qt, kt, vt, cu_seqlens, int(max_seqlen), scale=scaling, window=tuple(window))
    return out.reshape(1, out.shape[0], -1)


def debug_qk(q: Tensor, k: Tensor) -> Tensor:
    """Layout probe: fp32 ``q[:128] @ k[:128].T`` of one head through TMA + tcgen05 (rows past the
    inputs read as zero). q, k: ``[rows, D]`` bf16 CUDA, D contiguous."""
    s = torch.empty(128, 128, dtype=torch.float32, device=q.device)
    stream = torch.cuda.current_stream(q.device)
    _lib.check(_lib.lib().pe_b200_debug_qk(q.data_ptr(), k.data_ptr(), q.stride(0), k.stride(0), q.shape[0],
                                           k.shape[0], q.shape[1], s.data_ptr(), stream.cuda_stream), "debug_qk")
    return s


def debug_pv(p: Tensor, v: Tensor) -> Tensor:
    """Layout probe: fp32 ``bf16(p) @ v[:128]`` through TMEM P and a TMA'd V. p: ``[128, 128]`` fp32."""
    p = p.contiguous()
    o = torch.empty(128, v.shape[1], dtype=torch.float32, device=v.device)
    stream = torch.cuda.current_stream(v.device)
    _lib.check(_lib.lib().pe_b200_debug_pv(p.data_ptr(), v.data_ptr(), v.stride(0), v.shape[0], v.shape[1],
                                           o.data_ptr(), stream.cuda_stream), "debug_pv")
    return o


def apply_rope_bshd(qkv: Tensor, h: int, d: int, cos: Tensor, sin: Tensor) -> tuple[Tensor, Tensor]:
    """RoPE'd q, k from the packed qkv ``[..., 3*H*D]`` (the fused Wqkv output), contiguous
    ``[..., H, D]``: the reference's ``apply_rope_bshd`` (_kernels/rope.py:302-345, same arguments
    and rotate-half rule, fp32 rounded to bf16) on this library's rope pass. ``cos``/``sin`` are
    ``[S, D]`` (or ``[1, S, D]``) position tables of a dense ``[B, S]`` batch (row ``t % S``) or the
    per-token gathered ``[total, D]`` tables of a packed batch. head_dim 64."""
    if qkv.dtype != torch.bfloat16 or not qkv.is_cuda or qkv.shape[-1] != 3 * h * d or qkv.stride(-1) != 1:
        raise UnsupportedTargetError("rope: qkv must be CUDA bf16 [..., 3*H*D] with a contiguous last dim")
    if d != 64:
        raise UnsupportedTargetError("rope: head_dim 64 only")
    if cos.ndim == 3:
        cos, sin = cos[0], sin[0]
    if (cos.shape != sin.shape or cos.ndim != 2 or cos.shape[1] != d or cos.dtype != torch.bfloat16
            or sin.dtype != torch.bfloat16 or cos.stride(1) != 1 or sin.stride(1) != 1 or cos.stride(0) != sin.stride(0)
            or cos.device != qkv.device or sin.device != qkv.device):
        raise UnsupportedTargetError("rope: cos/sin must be bf16 [S, D] tables on qkv's device with one row stride")
    rows = qkv.reshape(-1, 3 * h * d)
    n = rows.shape[0]
    view = rows.view(n, 3, h, d)
    q_out = torch.empty(n, h, d, dtype=qkv.dtype, device=qkv.device)
    k_out = torch.empty(n, h, d, dtype=qkv.dtype, device=qkv.device)
    if n:
        with torch.cuda.device(qkv.device):
            stream = torch.cuda.current_stream(qkv.device)
            q, k = view[:, 0], view[:, 1]
            _lib.check(_lib.lib().pe_b200_rope_qk(
                _ptr(q), _ptr(k), q.stride(0), q.stride(1), k.stride(0), k.stride(1), _ptr(cos), _ptr(sin),
                cos.stride(0), cos.shape[0], n, h, h, d, _ptr(q_out), _ptr(k_out), ctypes.c_void_p(stream.cuda_stream)),
                "pe_b200_rope_qk")
        _count(1)
    shape = tuple(qkv.shape[:-1]) + (h, d)
    return q_out.view(shape), k_out.view(shape)

