"""pe_b200_attn_fwd_noalloc: the entry point for callers that cannot give the library any
device memory (a plugin host that hands over only a stream and the tensors, a language
binding without CUDA allocation calls, a server that allocates nothing per request).

It keeps the tile schedule and the device error word in a fixed 1 MiB array inside the library
instead of a caller workspace. This file is named to be collected last, so a run that stops at
the first failure has already run every other test. It calls the entry point through the C ABI
and compares it with the regular entry point (pe_b200_attn_fwd, through packed_attention) on
two calls in a row with different shapes, so stale schedule contents from the first call would
show up in the second; both run the same kernels on the same schedule, so the outputs must be
bit-identical. It also reads the device error word back through pe_b200_noalloc_error_word
after a call with malformed cu_seqlens.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from conftest import packed_inputs, rope_tables

pytestmark = pytest.mark.gpu

PE_B200_ERR_SCRATCH_LIMIT = -9
PE_B200_DEVERR_BAD_SEGMENTS = 4


def _so():
    from packed_encoders_b200 import _lib

    return _lib.lib()


def _params(q, k, v, out, cu, max_len, *, scale, window, causal, rope=None):
    from packed_encoders_b200 import _lib

    p = _lib.PeB200AttnParams(
        q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), out=out.data_ptr(), lse=None,
        cu_seqlens_q=cu.data_ptr(), cu_seqlens_k=cu.data_ptr(), n_seq=cu.numel() - 1,
        total_q=q.shape[0], total_k=k.shape[0], max_seqlen_q=max_len, max_seqlen_k=max_len,
        heads=q.shape[1], kv_heads=k.shape[1], head_dim=q.shape[2],
        q_stride_token=q.stride(0), q_stride_head=q.stride(1), k_stride_token=k.stride(0),
        k_stride_head=k.stride(1), v_stride_token=v.stride(0), v_stride_head=v.stride(1),
        o_stride_token=out.stride(0), o_stride_head=out.stride(1), scale=scale,
        window_left=window[0], window_right=window[1], causal=int(causal),
        workspace=None, workspace_bytes=0)
    if rope is not None:
        p.rope_cos, p.rope_sin = rope[0].data_ptr(), rope[1].data_ptr()
        p.rope_stride_token = rope[0].stride(0)
    return p


def _noalloc(params):
    stream = torch.cuda.current_stream()
    return _so().pe_b200_attn_fwd_noalloc(ctypes.byref(params), ctypes.c_void_p(stream.cuda_stream))


def _error_word():
    word = ctypes.c_int(-1)
    stream = torch.cuda.current_stream()
    status = _so().pe_b200_noalloc_error_word(ctypes.byref(word), ctypes.c_void_p(stream.cuda_stream))
    assert status == 0, f"pe_b200_noalloc_error_word status {status}"
    return word.value


CALLS = [
    # (lengths, heads, kv_heads, dim, window, causal)
    ([1, 2, 31, 300, 33, 64, 65, 127, 128, 700], 12, 12, 64, (-1, -1), False),
    ([5, 640, 0, 37, 129], 8, 2, 256, (-1, -1), True),
]


def test_noalloc_matches_regular_entry_point_twice():
    import packed_encoders_b200 as pe

    for i, (lengths, heads, kv_heads, dim, window, causal) in enumerate(CALLS):
        q, k, v, cu = packed_inputs(lengths, heads, dim, kv_heads=kv_heads, seed=40 + i, device="cuda")
        scale = dim ** -0.5
        expected = pe.packed_attention(q, k, v, cu, max(lengths), scale=scale, window=window, causal=causal)
        got = torch.full_like(q, float("nan"))
        status = _noalloc(_params(q, k, v, got, cu, max(lengths), scale=scale, window=window, causal=causal))
        assert status == 0, f"call {i}: status {status}"
        torch.cuda.synchronize()
        assert torch.equal(got, expected), f"call {i}: differs from pe_b200_attn_fwd"
        assert _error_word() == 0


def test_noalloc_rotary_call_matches_regular_entry_point():
    """A small call with rotary tables (its rotated q and k also live in the fixed scratch)."""
    import packed_encoders_b200 as pe

    lengths = [100, 7, 300, 93]
    q, k, v, cu = packed_inputs(lengths, 2, 64, seed=44, device="cuda")
    cos, sin = (t.cuda() for t in rope_tables(lengths))
    expected = pe.packed_attention(q, k, v, cu, max(lengths), scale=0.125, window=(64, 64), rope=(cos, sin))
    got = torch.full_like(q, float("nan"))
    status = _noalloc(_params(q, k, v, got, cu, max(lengths), scale=0.125, window=(64, 64), causal=False,
                              rope=(cos, sin)))
    assert status == 0
    torch.cuda.synchronize()
    assert torch.equal(got, expected)
    assert _error_word() == 0


def test_noalloc_error_word_reports_malformed_segments():
    """Decreasing cu_seqlens: the device schedule builder refuses the batch (schedules nothing, sets
    PE_B200_DEVERR_BAD_SEGMENTS); the getter reads it back, and the next good call clears it."""
    q, k, v, cu = packed_inputs([50, 30, 20], 2, 64, seed=45, device="cuda")
    bad = torch.tensor([0, 50, 30, 100], dtype=torch.int32, device="cuda")
    out = torch.zeros_like(q)
    assert _noalloc(_params(q, k, v, out, bad, 50, scale=0.125, window=(-1, -1), causal=False)) == 0
    torch.cuda.synchronize()
    assert _error_word() & PE_B200_DEVERR_BAD_SEGMENTS
    assert torch.count_nonzero(out) == 0  # nothing was scheduled
    assert _noalloc(_params(q, k, v, out, cu, 50, scale=0.125, window=(-1, -1), causal=False)) == 0
    torch.cuda.synchronize()
    assert _error_word() == 0


def test_noalloc_rejects_calls_beyond_its_scratch():
    from packed_encoders_b200 import _lib

    # 70,000 segments need more work-item slots than the fixed 1 MiB holds; rejected before
    # anything is enqueued (no pointer is dereferenced).
    params = _lib.PeB200AttnParams(n_seq=70_000, total_q=70_000, total_k=70_000, max_seqlen_q=1, max_seqlen_k=1,
                                   heads=1, kv_heads=1, head_dim=64, scale=0.125, window_left=-1,
                                   window_right=-1, causal=0)
    assert _so().pe_b200_attn_fwd_noalloc(ctypes.byref(params), None) == PE_B200_ERR_SCRATCH_LIMIT
    assert "no-allocation scratch" in _lib.status_string(PE_B200_ERR_SCRATCH_LIMIT)
