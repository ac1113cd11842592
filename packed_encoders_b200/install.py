"""Register the single ``"b200"`` attention backend into an imported ``packed_encoders``.

After ``install()``, the reference's own entry points run on the B200 kernels unchanged:

* ``pe.pack(model, attention_backend="b200", pieces=b200_pieces())`` prepares ModernBERT
  (the backend-name check of packed_encoders/pack.py:111-115 accepts ``"b200"``);
* the patched HF forward and ``forward.packed_forward`` take the packed (varlen) path for
  ``"b200"`` (padded batches are unpadded first, forward.py:634-657, like the Triton backend);
* inside ``forward._encoder_layer`` the BSHD RoPE + attention path is used
  (``ops.use_bshd_rope_flash``, ops.py:464-482) and ``execution.attention_bshd`` is the
  b200 piece (pieces/attention.py:70-73; swapped with ``dataclasses.replace`` as
  docs/architectures.md:139-149 describes);
* ``ops.attention_bshd`` / ``ops.attention`` (ops.py:502-555) route ``backend="b200"`` to
  the kernels;
* ``runtime.attention`` gains a ``"b200"`` candidate (runtime/attention.py:187-196) with
  packed / padded / prefixed forms, first in the default order on sm_100, and the Qwen3.5
  engine accepts ``attention_backend="b200"`` (arch/qwen3_5/__init__.py:49).

* on an sm_100 GPU (B200 / GB200), the default and ``"auto"`` backends resolve to ``"b200"``:
  ``pack._default_backend`` (pack.py:147-158), ``pack._resolve_attention_backend``
  (pack.py:161-192) and ``forward._resolve_eager_backend`` (forward.py:301-331, the branch that
  consults the calibrated Triton-vs-FA policy of attention_dispatch.py:129-205, eager and
  ``for_cuda_graph`` alike) stop there, so ``pe.pack(model)`` with no backend argument runs on
  these kernels. A leaf-level ``"auto"`` resolved while grad is enabled keeps the reference's own
  resolution.
* training: with grad enabled the ModernBERT layer takes its BHSD path (RoPE outside the
  attention call, ``ops.use_bshd_rope_flash`` is False), and ``ops.attention`` with ``"b200"``
  runs this library's forward and backward kernels (head_dim 64): packed batches through
  ``flash_attention_varlen`` (the eager packed training forward, forward.py:634-657), unpadded
  rectangular batches through ``flash_attention`` (the training graph of train_graph.py:170-181,
  which ``pe.pack(..., train_cuda_graph=True)`` builds with the pack's backend, pack.py:216-238).

There is no policy and no fallback: ``"b200"`` always means these kernels; anything they do
not implement raises ``UnsupportedTargetError``.
"""

from __future__ import annotations

import dataclasses
import functools

import torch

from packed_encoders_b200 import ops as b200_ops
from packed_encoders_b200.errors import UnsupportedTargetError

BACKEND = "b200"
_INSTALLED = {"done": False}


# --------------------------------------------------------------------------- pieces
def _reference_bshd(q, k, v, *, window, scaling, backend="flash", cu_seqlens=None, max_seqlen=None):
    from packed_encoders.pieces.attention import reference_bshd

    return reference_bshd(q, k, v, window=window, scaling=scaling, backend="flash", cu_seqlens=cu_seqlens,
                          max_seqlen=max_seqlen)


def _check_bshd(q, k, v, *, window, scaling, backend="flash", cu_seqlens=None, max_seqlen=None):
    if q.ndim != 4 or q.shape != k.shape or q.shape != v.shape:
        raise UnsupportedTargetError("attention piece requires equal Q/K/V shapes")
    if cu_seqlens is not None and (q.shape[0] != 1 or cu_seqlens.dtype != torch.int32 or max_seqlen is None):
        raise UnsupportedTargetError("packed b200 BSHD attention: B=1, int32 cu_seqlens, max_seqlen")
    if scaling <= 0:
        raise UnsupportedTargetError("unsupported attention scale")


def _execute_bshd(q, k, v, *, window, scaling, backend=BACKEND, cu_seqlens=None, max_seqlen=None):
    """The piece always runs the B200 kernels, whatever backend name the caller probes with."""
    return b200_ops.attention_bshd(q, k, v, window=window, scaling=scaling, cu_seqlens=cu_seqlens,
                                   max_seqlen=max_seqlen, backend=BACKEND)


def b200_attention_bshd_piece():
    """The BSHD attention piece (contract pieces/attention.py:11-12) executed by the B200 kernels,
    validated against the reference's own independent oracle."""
    from packed_encoders.pieces.attention import BSHD
    from packed_encoders.pieces.base import Piece

    return Piece("attention-bshd-b200", BSHD, _execute_bshd, _reference_bshd, _check_bshd)


def _execute_rope_qkv(qkv, h, d, cos, sin):
    return b200_ops.apply_rope_bshd(qkv, h, d, cos, sin)


def b200_rope_qkv_piece():
    """The QKV-BSHD RoPE piece (contract pieces/rope.py:97-99) executed by this library's rope
    pass, with the reference's own oracle and argument checks (pieces/rope.py:73-80)."""
    from packed_encoders.pieces.rope import QKV_BSHD, RoPEPiece, check_qkv, reference_qkv

    return RoPEPiece("split-half-rope-qkv-bshd-b200", QKV_BSHD, _execute_rope_qkv, reference_qkv, check_qkv)


def b200_pieces(base=None):
    """ModernBERT pieces with the BSHD attention and QKV RoPE slots replaced
    (docs/architectures.md:139-149)."""
    if base is None:
        from packed_encoders.arch.modernbert_pieces import default_pieces

        base = default_pieces()
    return dataclasses.replace(base, attention_bshd=b200_attention_bshd_piece(), rope_qkv=b200_rope_qkv_piece())


# --------------------------------------------------------------------------- runtime candidate
def b200_candidate(window, scale):
    """``runtime.attention`` candidate: ``(packed, padded, prefixed)`` on the B200 kernels."""

    def packed(q, k, v, cu32, max_len, lengths, causal):
        return b200_ops.packed_attention(q, k, v, cu32, int(max_len), scale=scale, window=window, causal=causal)

    def padded(q, k, v, static, causal):
        # [real | pad] segments (runtime/graphs.py:65-72) are ordinary segments of the packed form.
        return b200_ops.packed_attention(q, k, v, static.seg_cu32, int(static.seq), scale=scale, window=window,
                                         causal=causal)

    def prefixed(q, k, v, cu_q, cu_k, max_q, max_k, lengths_q, lengths_k, causal):
        return b200_ops.packed_attention(q, k, v, cu_q, int(max_q), scale=scale, window=window, causal=causal,
                                         cu_seqlens_k=cu_k, max_seqlen_k=int(max_k))

    return packed, padded, prefixed


# --------------------------------------------------------------------------- device policy
def on_b200() -> bool:
    """True when the current CUDA device is an sm_100 part these kernels run on. Uses the
    reference's own capability probe (attention_dispatch.py:148-154), so a test can fake it."""
    from packed_encoders import attention_dispatch

    return attention_dispatch.current_compute_capability() == (10, 0)


def resolve_backend(backend: str | None) -> str | None:
    """The single policy that replaces the calibrated Triton-vs-FA dispatch on sm_100: an unset
    or ``"auto"`` backend, in inference, is ``"b200"``. Anything else is returned unchanged."""
    if backend in (None, "auto") and not torch.is_grad_enabled() and on_b200():
        return BACKEND
    return backend


# --------------------------------------------------------------------------- install
def install() -> None:
    """Patch the imported reference package in place (idempotent)."""
    if _INSTALLED["done"]:
        return
    import importlib

    forward = importlib.import_module("packed_encoders.forward")
    ops = importlib.import_module("packed_encoders.ops")
    pack = importlib.import_module("packed_encoders.pack")  # the package re-exports a function of this name
    graph = importlib.import_module("packed_encoders.graph")
    rt_attention = importlib.import_module("packed_encoders.runtime.attention")

    orig_use_bshd = ops.use_bshd_rope_flash

    @functools.wraps(orig_use_bshd)
    def use_bshd_rope_flash(backend, h, d, cu_seqlens):
        if backend == BACKEND:
            return not torch.is_grad_enabled() and ops._bshd_applicable(h, d)
        return orig_use_bshd(backend, h, d, cu_seqlens)

    orig_attention_bshd = ops.attention_bshd

    @functools.wraps(orig_attention_bshd)
    def attention_bshd(q, k, v, *, window, scaling, cu_seqlens=None, max_seqlen=None, backend="flash"):
        if backend == BACKEND:
            return b200_ops.attention_bshd(q, k, v, window=window, scaling=scaling, cu_seqlens=cu_seqlens,
                                           max_seqlen=max_seqlen, backend=BACKEND)
        return orig_attention_bshd(q, k, v, window=window, scaling=scaling, cu_seqlens=cu_seqlens,
                                   max_seqlen=max_seqlen, backend=backend)

    orig_attention = ops.attention

    @functools.wraps(orig_attention)
    def attention(q, k, v, *, mask, window, scaling, backend, cu_seqlens=None, max_seqlen=None):
        if backend == BACKEND:
            if cu_seqlens is None:  # the rectangular (unpadded) form, e.g. the training graph's forward
                return b200_ops.flash_attention(q, k, v, window, scaling)
            return b200_ops.flash_attention_varlen(q, k, v, cu_seqlens, max_seqlen, window, scaling)
        return orig_attention(q, k, v, mask=mask, window=window, scaling=scaling, backend=backend,
                              cu_seqlens=cu_seqlens, max_seqlen=max_seqlen)

    orig_fused = forward.fused_forward

    @functools.wraps(orig_fused)
    def fused_forward(model, params, input_ids, attention_mask, *, execution=None, backend="sdpa"):
        backend = resolve_backend(backend) if backend == "auto" else backend
        if backend == BACKEND:  # always the packed path, like the Triton backend (forward.py:696-703)
            if attention_mask is None:
                attention_mask = torch.ones_like(input_ids)
            return forward._varlen_forward(model, params, input_ids, attention_mask, backend=BACKEND,
                                           execution=execution)
        return orig_fused(model, params, input_ids, attention_mask, execution=execution, backend=backend)

    orig_resolve_eager = forward._resolve_eager_backend

    @functools.wraps(orig_resolve_eager)
    def _resolve_eager_backend(backend, workload=None, *, triton_supported=False, flash_available=None,
                               for_cuda_graph=False):
        if backend == BACKEND:
            return BACKEND
        if backend == "auto" and resolve_backend(backend) == BACKEND:
            return BACKEND  # the calibrated Triton-vs-FA policy is not consulted on sm_100
        return orig_resolve_eager(backend, workload, triton_supported=triton_supported,
                                  flash_available=flash_available, for_cuda_graph=for_cuda_graph)

    orig_default = pack._default_backend

    @functools.wraps(orig_default)
    def _default_backend():
        return BACKEND if on_b200() else orig_default()

    orig_resolve_attention = pack._resolve_attention_backend

    @functools.wraps(orig_resolve_attention)
    def _resolve_attention_backend(backend):
        if backend == BACKEND or (backend == "auto" and on_b200()):
            return BACKEND
        return orig_resolve_attention(backend)

    orig_rect = graph.rectangular_graph_backend

    @functools.wraps(orig_rect)
    def rectangular_graph_backend(backend):
        # b200 serves the packed path only: padded batches reach it through the packed runner.
        return None if backend == BACKEND else orig_rect(backend)

    orig_prepare = pack._prepare_modernbert

    @functools.wraps(orig_prepare)
    def _prepare_modernbert(encoder, *, attention_backend=None, cuda_graph=None, cuda_graph_seq_cutoff=64,
                            **kwargs):
        if attention_backend is None:
            attention_backend = pack._default_backend()
        if attention_backend == "auto" and on_b200():
            attention_backend = BACKEND
        if attention_backend != BACKEND:
            return orig_prepare(encoder, attention_backend=attention_backend, cuda_graph=cuda_graph,
                                cuda_graph_seq_cutoff=cuda_graph_seq_cutoff, **kwargs)
        # "sdpa" passes the name check with no optional dependency; the state is then switched
        # to b200 before any runner is built, so the inference graphs and the training graph
        # (pack.py:216-238 builds it with the state's backend) run on these kernels.
        train_cuda_graph = kwargs.pop("train_cuda_graph", False)
        state = orig_prepare(encoder, attention_backend="sdpa", cuda_graph=False, train_cuda_graph=False,
                             cuda_graph_seq_cutoff=cuda_graph_seq_cutoff, **kwargs)
        state.attention_backend = BACKEND
        if cuda_graph:
            pack._enable_graphs(encoder, state, cuda_graph, cuda_graph_seq_cutoff)
        if train_cuda_graph:
            pack._enable_train_graphs(encoder, state, train_cuda_graph, cuda_graph_seq_cutoff)
        return state

    ops.use_bshd_rope_flash = use_bshd_rope_flash
    ops.attention_bshd = attention_bshd
    ops.attention = attention
    forward.fused_forward = fused_forward
    forward._resolve_eager_backend = _resolve_eager_backend
    pack._default_backend = _default_backend
    pack._resolve_attention_backend = _resolve_attention_backend
    pack._prepare_modernbert = _prepare_modernbert
    graph.rectangular_graph_backend = rectangular_graph_backend

    rt_attention._CANDIDATES[BACKEND] = b200_candidate
    orig_order = rt_attention.default_order

    @functools.wraps(orig_order)
    def default_order(device):
        order = tuple(n for n in orig_order(device) if n != BACKEND)
        if torch.cuda.get_device_capability(device) == (10, 0):
            return (BACKEND, *order)
        return order

    rt_attention.default_order = default_order
    try:
        from packed_encoders.arch import qwen3_5

        qwen3_5._BACKENDS[BACKEND] = (BACKEND,)
    except ImportError:  # the Qwen engine needs fla; ModernBERT does not
        pass
    try:  # pieces are bound at first use; drop any cached default so rebinding sees the patch
        from packed_encoders.arch import modernbert_pieces

        modernbert_pieces.default_pieces.cache_clear()
        modernbert_pieces.default_execution.cache_clear()
    except (ImportError, AttributeError):
        pass
    _INSTALLED["done"] = True


__all__ = ["BACKEND", "b200_attention_bshd_piece", "b200_candidate", "b200_pieces", "b200_rope_qkv_piece", "install",
           "on_b200", "resolve_backend"]
