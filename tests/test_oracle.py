"""Pin the CPU oracle before trusting it: golden vectors from the reference itself, and
the reference's own C kernel compiled from its source (oracle/_ref)."""

from __future__ import annotations

import pytest
import torch

import oracle
from conftest import golden_names, load_golden, load_rope_golden, packed_inputs, rope_golden_names

# fp32 restatement vs the reference's fp32 paths: both are fp32-exact to rounding.
ATOL = 2e-5


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_golden(name):
    g = load_golden(name)
    out, lse = oracle.attention_prefixed(g["q"], g["k"], g["v"], g["cu_q"], g["cu_k"], scale=g["scale"],
                                         window=g["window"], causal=g["causal"], threads=4)
    torch.testing.assert_close(out, g["out"], atol=ATOL, rtol=ATOL)
    assert torch.isfinite(lse).all()


def _lse_reference(q, k, cu, scale, window, causal):
    """Natural-log LSE restated with torch (float64) for the oracle's LSE output."""
    heads, kv = q.shape[1], k.shape[1]
    rows = []
    for s in range(cu.numel() - 1):
        a, b = int(cu[s]), int(cu[s + 1])
        if b == a:
            continue
        qs = q[a:b].double().permute(1, 0, 2)
        ks = k[a:b].double().repeat_interleave(heads // kv, 1).permute(1, 2, 0)
        scores = (qs @ ks) * scale
        pos = torch.arange(b - a)
        delta = pos[:, None] - pos[None, :]
        allowed = torch.ones(b - a, b - a, dtype=torch.bool)
        right = 0 if causal else window[1]
        if window[0] >= 0:
            allowed &= delta <= window[0]
        if right >= 0:
            allowed &= delta >= -right
        rows.append(scores.masked_fill(~allowed, float("-inf")).logsumexp(-1))
    return torch.cat(rows, dim=1).float()


@pytest.mark.parametrize("window,causal", [((-1, -1), False), ((64, 64), False), ((-1, -1), True), ((8, 3), False)])
def test_oracle_lse(window, causal):
    q, k, v, cu = packed_inputs([1, 40, 0, 129, 7], 4, 64, kv_heads=2, seed=3)
    _, lse = oracle.attention(q, k, v, cu, scale=0.125, window=window, causal=causal, threads=2)
    torch.testing.assert_close(lse, _lse_reference(q, k, cu, 0.125, window, causal), atol=1e-5, rtol=1e-5)


@pytest.mark.skipif(oracle.available_reference() is None, reason="reference C kernel not built for this host")
@pytest.mark.parametrize("half", [0, 15, 64, 10_000])
@pytest.mark.parametrize("lengths", [[1, 2, 31, 32, 33, 63, 64, 65, 127, 128], [7, 65, 66, 1, 130, 200],
                                     [16, 32, 1, 15, 17, 31, 33, 65]])
def test_oracle_matches_reference_kernel(lengths, half):
    """The restatement agrees with the reference's own pe_local_attention on the same inputs."""
    q, k, v, cu = packed_inputs(lengths, 3, 64, seed=11, logit_scale=2.0)
    half_eff = min(half, max(lengths))
    window = (-1, -1) if half_eff >= max(lengths) else (half_eff, half_eff)
    ours, _ = oracle.attention(q, k, v, cu, scale=0.125, window=window, threads=4)
    ref = oracle.reference_local_attention(*(t.float().permute(1, 0, 2) for t in (q, k, v)), lengths, half_eff,
                                           threads=4)
    torch.testing.assert_close(ours, ref.permute(1, 0, 2), atol=ATOL, rtol=ATOL)
    # token-major output of the reference (local_attention_x86.c:212,218) is the same numbers
    ref_tm = oracle.reference_local_attention(*(t.float().permute(1, 0, 2) for t in (q, k, v)), lengths, half_eff,
                                              threads=4, token_major=True)
    torch.testing.assert_close(ref_tm.view_as(ours), ref.permute(1, 0, 2), atol=0, rtol=0)


def test_oracle_rejects_bad_arguments():
    q, k, v, cu = packed_inputs([3, 4], 2, 64)
    bad = cu.clone()
    bad[-1] = 6  # total does not match
    with pytest.raises(ValueError):
        oracle.attention(q, k, v, bad, scale=0.125)
    with pytest.raises(ValueError):  # heads not a multiple of kv heads
        oracle.attention(q, k[:, :1].expand(-1, 1, -1).repeat(1, 3, 1)[:, :3], v[:, :1].repeat(1, 3, 1), cu,
                         scale=0.125)


def test_useful_pairs_counts():
    cu = torch.tensor([0, 3, 3, 203], dtype=torch.int32)
    assert oracle.useful_pairs(cu) == 9 + 200 * 200
    assert oracle.useful_pairs(cu, causal=True) == 6 + 200 * 201 // 2
    # |i-j| <= 64 inside a 200-token sequence
    band = sum(min(199, i + 64) - max(0, i - 64) + 1 for i in range(200))
    assert oracle.useful_pairs(cu, window=(64, 64)) == 9 + band


def test_empty_batch_is_fine():
    q, k, v, cu = packed_inputs([0, 0], 2, 64)
    out, lse = oracle.attention(q, k, v, cu, scale=0.125)
    assert out.shape == (0, 2, 64) and lse.shape == (2, 0)


@pytest.mark.parametrize("name", rope_golden_names())
def test_rope_restatement_matches_reference(name):
    """oracle.rope_bshd (fp32 rotate-half, rounded to bf16) against the reference's own CPU RoPE
    (CPUAttention.rope_layout, fp32): equal up to the final bf16 rounding; and the reference's
    attention over its rotated q/k is reproduced by the oracle over the restated rotation."""
    g = load_rope_golden(name)
    for x, ref in ((g["q"], g["rq"]), (g["k"], g["rk"])):
        got = oracle.rope_bshd(x, g["cos"], g["sin"]).float()
        assert ((got - ref).abs() <= ref.abs() * 2.0 ** -8 + 1e-6).all()
    rq, rk = oracle.rope_bshd(g["q"], g["cos"], g["sin"]), oracle.rope_bshd(g["k"], g["cos"], g["sin"])
    out, _ = oracle.attention(rq, rk, g["v"], g["cu_q"], scale=g["scale"], window=g["window"])
    assert (out - g["out"]).abs().max().item() <= 2e-2

