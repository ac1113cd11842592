"""Parity at the configurations' full sizes (GPU), through properties that do not need a CPU
reference for the whole batch:

* a long sequence's rows of the packed batch equal a call on that sequence alone, bit for bit
  (its key tiles start at the sequence's first key either way, so the arithmetic is the same),
  for global, windowed and causal GQA layers, including the longest sequence of the batch;
* sampled sequences of the batch match the CPU oracle run on those sequences alone (parity bars
  of the north star: max-abs 2e-2, per-token cosine 0.9999, LSE 1e-3);
* the device error word stays clear.

Inputs are the bench's seeded synthetic batches (packed_encoders_b200.workloads).
"""

from __future__ import annotations

import pytest
import torch

import oracle
from packed_encoders_b200 import workloads as wl

pytestmark = pytest.mark.gpu


def _parity(got, ref, what):
    got, ref = got.float().cpu(), ref.float().cpu()
    assert torch.isfinite(got).all(), what
    err = (got - ref).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(got.flatten(1), ref.flatten(1), dim=1).min().item()
    print(f"PARITY {what}: max_abs={err:.5f} min_cos={cos:.7f}")
    assert err <= 2e-2, what
    assert cos >= 0.9999, what


def _lse(got, ref, what):
    err = (got.float().cpu() - ref.float().cpu()).abs().max().item()
    print(f"PARITY {what}: lse_max_abs={err:.6f}")
    assert err <= 1e-3, what


def _batch(w):
    q, k, v = wl.make_qkv(w.lengths, w.heads, w.kv_heads, w.head_dim, seed=1)
    cu = w.cu_seqlens()
    return q, k, v, cu


def _long_sample(lengths, n=6):
    """Indices of the longest sequence and of a spread of other sequences longer than one tile."""
    order = sorted(range(len(lengths)), key=lambda i: -lengths[i])
    longs = [i for i in order if lengths[i] > 128]
    step = max(1, len(longs) // n)
    return sorted(set([order[0]] + longs[::step][:n]))


@pytest.mark.parametrize("kind", ["global", "local"])
def test_config1_full_batch_matches_oracle_and_reference_kernel(kind):
    """Config 1 (the north-star parity configuration) at full size: 32 x U[8,512] from seed 0,
    12 heads x 64, scale 1/8, global and +-64, q/k/v ~ N(0,1) bf16 from seed 1. The whole batch is
    checked against the fp32 oracle (output and LSE) and against the reference's own CPU kernel
    pe_local_attention (packed_encoders/cpu/local_attention_x86.c:192-235, compiled from the
    reference source into oracle/_ref; global = half-window >= the longest sequence)."""
    import packed_encoders_b200 as pe

    w = wl.config1(kind)
    (window, causal), = set(w.layers)
    q, k, v, cu = _batch(w)
    out, lse = pe.packed_attention(q, k, v, cu.cuda(), max(w.lengths), scale=w.scale, window=window,
                                   causal=causal, return_lse=True)
    torch.cuda.synchronize()
    assert pe.device_error_word() == 0
    qc, kc, vc = q.cpu(), k.cpu(), v.cpu()
    ref, ref_lse = oracle.attention(qc, kc, vc, cu, scale=w.scale, window=window, causal=causal)
    _parity(out, ref, f"config1 {kind} vs oracle")
    _lse(lse, ref_lse, f"config1 {kind} vs oracle")
    if oracle.available_reference() is None:
        pytest.skip("reference CPU kernel not built for this host's ISA (oracle/_ref)")
    half = max(w.lengths) if window == (-1, -1) else window[0]
    ref_native = oracle.reference_local_attention(qc.permute(1, 0, 2), kc.permute(1, 0, 2), vc.permute(1, 0, 2),
                                                  w.lengths, half)
    _parity(out, ref_native.permute(1, 0, 2), f"config1 {kind} vs reference pe_local_attention")


@pytest.mark.parametrize("kind", ["global", "local"])
def test_config3_rows_equal_standalone_calls(kind):
    import packed_encoders_b200 as pe

    w = wl.config3(kind)
    (window, causal), = set(w.layers)
    q, k, v, cu = _batch(w)
    out, lse = pe.packed_attention(q, k, v, cu.cuda(), max(w.lengths), scale=w.scale, window=window,
                                   causal=causal, return_lse=True)
    torch.cuda.synchronize()
    assert pe.device_error_word() == 0
    assert max(w.lengths) == max(w.lengths[i] for i in _long_sample(w.lengths))
    for i in _long_sample(w.lengths):
        a, b = int(cu[i]), int(cu[i + 1])
        one = torch.tensor([0, b - a], dtype=torch.int32, device="cuda")
        o1, l1 = pe.packed_attention(q[a:b].contiguous(), k[a:b].contiguous(), v[a:b].contiguous(), one, b - a,
                                     scale=w.scale, window=window, causal=causal, return_lse=True)
        assert torch.equal(out[a:b], o1), (kind, i, b - a)
        assert torch.equal(lse[:, a:b], l1), (kind, i, b - a)


@pytest.mark.parametrize("kind", ["global", "local"])
def test_config3_sampled_sequences_match_oracle(kind):
    import packed_encoders_b200 as pe

    w = wl.config3(kind)
    (window, causal), = set(w.layers)
    q, k, v, cu = _batch(w)
    out, lse = pe.packed_attention(q, k, v, cu.cuda(), max(w.lengths), scale=w.scale, window=window,
                                   causal=causal, return_lse=True)
    torch.cuda.synchronize()
    # short, median and ~1.5k-token sequences (the oracle is fp32 CPU)
    by_len = sorted(range(len(w.lengths)), key=lambda i: w.lengths[i])
    picks = [by_len[0], by_len[len(by_len) // 2], next(i for i in by_len if w.lengths[i] >= 1500)]
    for i in picks:
        a, b = int(cu[i]), int(cu[i + 1])
        one = torch.tensor([0, b - a], dtype=torch.int32)
        ref, ref_lse = oracle.attention(q[a:b].cpu(), k[a:b].cpu(), v[a:b].cpu(), one, scale=w.scale,
                                        window=window, causal=causal)
        _parity(out[a:b], ref, f"config3 {kind} seq {i} ({b - a} tokens)")
        _lse(lse[:, a:b], ref_lse, f"config3 {kind} seq {i}")


def test_config2_sampled_sequences_match_oracle():
    """Query batch (4096 x U[8,64], packed several per 128-row tile): sampled sequences."""
    import packed_encoders_b200 as pe

    w = wl.config2()
    q, k, v, cu = _batch(w)
    out, lse = pe.packed_attention(q, k, v, cu.cuda(), max(w.lengths), scale=w.scale, return_lse=True)
    torch.cuda.synchronize()
    assert pe.device_error_word() == 0
    for i in list(range(0, len(w.lengths), 257)) + [len(w.lengths) - 1]:
        a, b = int(cu[i]), int(cu[i + 1])
        one = torch.tensor([0, b - a], dtype=torch.int32)
        ref, ref_lse = oracle.attention(q[a:b].cpu(), k[a:b].cpu(), v[a:b].cpu(), one, scale=w.scale)
        _parity(out[a:b], ref, f"config2 seq {i} ({b - a} tokens)")
        _lse(lse[:, a:b], ref_lse, f"config2 seq {i}")


def test_config5_rows_equal_standalone_calls_and_oracle():
    """GQA 8/2, head_dim 256, causal, 256 x U[128, 4096] (543k tokens)."""
    import packed_encoders_b200 as pe

    w = wl.config5()
    q, k, v, cu = _batch(w)
    out = pe.packed_attention(q, k, v, cu.cuda(), max(w.lengths), scale=w.scale, causal=True)
    torch.cuda.synchronize()
    assert pe.device_error_word() == 0
    for i in _long_sample(w.lengths, n=4):
        a, b = int(cu[i]), int(cu[i + 1])
        one = torch.tensor([0, b - a], dtype=torch.int32, device="cuda")
        o1 = pe.packed_attention(q[a:b].contiguous(), k[a:b].contiguous(), v[a:b].contiguous(), one, b - a,
                                 scale=w.scale, causal=True)
        assert torch.equal(out[a:b], o1), (i, b - a)
    i = min(range(len(w.lengths)), key=lambda j: w.lengths[j])
    a, b = int(cu[i]), int(cu[i + 1])
    ref, _ = oracle.attention(q[a:b].cpu(), k[a:b].cpu(), v[a:b].cpu(), torch.tensor([0, b - a], dtype=torch.int32),
                              scale=w.scale, causal=True)
    _parity(out[a:b], ref, f"config5 seq {i} ({b - a} tokens)")
