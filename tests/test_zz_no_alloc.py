"""pe_b200_attn_fwd_noalloc: the entry point for callers that cannot give the library any
device memory (a plugin host that hands over only a stream and the tensors, a language
binding without CUDA allocation calls, a server that allocates nothing per request).

It keeps the tile schedule in a fixed 1 MiB array inside the library instead of a caller
workspace. This file is named to be collected last, so a run that stops at the first failure
has already run every other test. It calls the entry point through the C ABI and compares
it with the regular entry point (pe_b200_attn_fwd, through packed_attention) on two calls in a
row with different shapes, so stale schedule contents from the first call would show up in the
second.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import packed_inputs

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2  # the parity bar the other GPU tests use


def _noalloc_fn():
    from packed_encoders_b200 import _lib

    fn = _lib.lib().pe_b200_attn_fwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(_lib.PeB200AttnParams), ctypes.c_void_p]
    return fn


def _params(q, k, v, out, cu, max_len, *, scale, window, causal):
    from packed_encoders_b200 import _lib

    return _lib.PeB200AttnParams(
        q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), out=out.data_ptr(), lse=None,
        cu_seqlens_q=cu.data_ptr(), cu_seqlens_k=cu.data_ptr(), n_seq=cu.numel() - 1,
        total_q=q.shape[0], total_k=k.shape[0], max_seqlen_q=max_len, max_seqlen_k=max_len,
        heads=q.shape[1], kv_heads=k.shape[1], head_dim=q.shape[2],
        q_stride_token=q.stride(0), q_stride_head=q.stride(1), k_stride_token=k.stride(0),
        k_stride_head=k.stride(1), v_stride_token=v.stride(0), v_stride_head=v.stride(1),
        o_stride_token=out.stride(0), o_stride_head=out.stride(1), scale=scale,
        window_left=window[0], window_right=window[1], causal=int(causal),
        workspace=None, workspace_bytes=0)


CALLS = [
    # (lengths, heads, kv_heads, dim, window, causal)
    ([1, 2, 31, 300, 33, 64, 65, 127, 128, 700], 12, 12, 64, (-1, -1), False),
    ([5, 640, 0, 37, 129], 8, 2, 256, (-1, -1), True),
]


def test_noalloc_matches_regular_entry_point_twice():
    import packed_encoders_b200 as pe

    fn = _noalloc_fn()
    for i, (lengths, heads, kv_heads, dim, window, causal) in enumerate(CALLS):
        q, k, v, cu = packed_inputs(lengths, heads, dim, kv_heads=kv_heads, seed=40 + i, device="cuda")
        scale = dim ** -0.5
        expected = pe.packed_attention(q, k, v, cu, max(lengths), scale=scale, window=window, causal=causal)
        got = torch.full_like(q, float("nan"))
        params = _params(q, k, v, got, cu, max(lengths), scale=scale, window=window, causal=causal)
        stream = torch.cuda.current_stream()
        status = fn(ctypes.byref(params), ctypes.c_void_p(stream.cuda_stream))
        assert status == 0, f"call {i}: status {status}"
        torch.cuda.synchronize()
        assert torch.isfinite(got).all(), f"call {i}: output not fully written"
        err = (got.float() - expected.float()).abs().max().item()
        assert err <= MAX_ABS, f"call {i}: max abs difference {err}"


def test_noalloc_rejects_calls_beyond_its_scratch():
    fn = _noalloc_fn()
    from packed_encoders_b200 import _lib

    # 70,000 segments need more work-item slots than the fixed 1 MiB holds; rejected before
    # anything is enqueued (no pointer is dereferenced).
    params = _lib.PeB200AttnParams(n_seq=70_000, total_q=70_000, total_k=70_000, max_seqlen_q=1, max_seqlen_k=1,
                                   heads=1, kv_heads=1, head_dim=64, scale=0.125, window_left=-1,
                                   window_right=-1, causal=0)
    assert fn(ctypes.byref(params), None) == -9  # PE_B200_ERR_SCRATCH_LIMIT
    assert "no-allocation scratch" in _lib.status_string(-9)
